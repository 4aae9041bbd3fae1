"""Host-side restatement of the B-spline kernels' span evaluation (csrc/kat_bspline.cu), checked
on the CPU in float64 against the oracle's recursion:

  - the padded shared-memory tables (knot rows j + kOrder holding t_clamp(j), clamped differences
    and reciprocals at rows (k - 1, j + kOrder)) and the windows a span reads from them, without
    index clamping;
  - the fixed-step span search over the bits of the index (largest i <= n - 2 with t_i <= x);
  - the backward's derivative identity dB^K_j/dx = K (B^{K-1}_j / d_j - B^{K-1}_{j+1} / d_{j+1}),
    d_j = max(t_{j+K} - t_j, 1e-8), against autograd through the reference recursion, on uniform
    grids and grids with repeated knots, orders 1..5."""

import pytest
import torch

from oracle import bspline_oracle as bs

EPS = 1e-8


def tables(t, K):
    n = len(t)
    knots = [t[min(max(row - K, 0), n - 1)] for row in range(n + 2 * K)]
    recip = [[0.0] * (n + K) for _ in range(K)]
    diff = [[1.0] * (n + K) for _ in range(K)]
    for k in range(1, K + 1):
        for row in range(n + K):
            j = row - K
            if j >= 0 and j + k < n:
                diff[k - 1][row] = max(t[j + k] - t[j], EPS)
                recip[k - 1][row] = 1.0 / diff[k - 1][row]
    return knots, recip, diff


def find_span(t, n, x):
    i, step = 0, 1 << ((n - 2).bit_length() - 1)
    while step:
        if i + step <= n - 2 and t[i + step] <= x:
            i += step
        step >>= 1
    return i


def span_values(t, K, levels, x):
    """B^levels values on x's span from the padded tables, as the kernels index them."""
    n = len(t)
    knots, recip, diff = tables(t, K)
    i = find_span(t, n, x)
    xl = [x - knots[i + 1 + q] for q in range(K)]
    xr = [knots[i + 1 + q + K] - x for q in range(K)]
    rw = [[recip[k - 1][i - k + 1 + m + K] for m in range(k)] for k in range(1, K + 1)]
    dw = [[diff[k - 1][i - k + 1 + m + K] for m in range(k)] for k in range(1, K + 1)]
    prev = [1.0]
    for k in range(1, levels + 1):
        cur = []
        for m in range(k + 1):
            j = i - k + m
            v = 0.0
            if 0 <= j <= n - 2 - k:
                if m >= 1:
                    assert abs(dw[k - 1][m - 1] * rw[k - 1][m - 1] - 1.0) < 1e-12
                    v += xl[K - 1 - k + m] / dw[k - 1][m - 1] * prev[m - 1]
                if m <= k - 1:
                    v += xr[m] / dw[k - 1][m] * prev[m]
            cur.append(v)
        prev = cur
    return i, prev, rw


def grids(K):
    out = []
    for gs in (3, 5, 8):
        out.append(bs.make_grid(1, gs, K).double()[0].tolist())
        g = torch.Generator().manual_seed(10 * K + gs)
        adap = torch.sort(torch.randn(gs + 2 * K + 1, generator=g).double())[0]
        adap[K + 1] = adap[K]                      # a repeated knot
        out.append(adap.tolist())
    return out


@pytest.mark.parametrize("K", [1, 2, 3, 4, 5])
def test_padded_tables_and_span_search_match_the_recursion(K):
    for t in grids(K):
        n, nb = len(t), len(t) - 1 - K
        tt = torch.tensor(t, dtype=torch.float64).view(1, -1)
        xs = torch.linspace(t[0], t[-1], 203, dtype=torch.float64)[:-1].tolist() + t[:-1]
        ref = bs.b_splines(torch.tensor(xs, dtype=torch.float64).view(-1, 1), tt, K).view(len(xs), -1)
        for row, x in enumerate(xs):
            i, vals, _ = span_values(t, K, K, x)
            assert t[i] <= x and (i == n - 2 or x < t[i + 1])
            out = [0.0] * nb
            for m, v in enumerate(vals):
                if 0 <= i - K + m < nb:
                    out[i - K + m] = v
            assert max(abs(a - b) for a, b in zip(out, ref[row].tolist())) < 1e-12


@pytest.mark.parametrize("K", [1, 2, 3, 4, 5])
def test_backward_derivative_identity(K):
    for t in grids(K):
        n, nb = len(t), len(t) - 1 - K
        tt = torch.tensor(t, dtype=torch.float64).view(1, -1)
        xs = torch.linspace(t[0], t[-1], 151, dtype=torch.float64)[:-1]
        x = xs.view(-1, 1).clone().requires_grad_(True)
        B = bs.b_splines(x, tt, K)
        dB = torch.stack([torch.autograd.grad(B[..., j].sum(), x, retain_graph=True)[0].view(-1)
                          for j in range(nb)], dim=-1)
        for row, xv in enumerate(xs.tolist()):
            i, lower, rw = span_values(t, K, K - 1, xv)
            got = [0.0] * nb
            for m in range(K + 1):
                j = i - K + m
                if 0 <= j < nb:
                    left = lower[m - 1] * rw[K - 1][m - 1] if m >= 1 else 0.0
                    right = lower[m] * rw[K - 1][m] if m <= K - 1 else 0.0
                    got[j] = K * (left - right)
            want = dB[row].tolist()
            scale = max(1.0, sum(abs(v) for v in want))
            assert max(abs(a - b) for a, b in zip(got, want)) < 1e-9 * scale
