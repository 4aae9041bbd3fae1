/*
 * kat_bspline.h — C ABI of the B-spline basis kernels in libkat_rational.so (sm_100a).
 *
 * The B-spline basis of a KAN layer (efficient-KAN's KANLinear.b_splines, fused by the
 * reference in rational_kat_cu/bspline_basis.py): for every input element x[b, d] and the
 * channel's knot vector t = grid[d, 0..n_knots-1], the Cox-de Boor recursion
 *
 *     B^0_i(x) = 1 if t_i <= x < t_{i+1}, else 0                       (i = 0 .. n_knots-2)
 *     B^k_i(x) = (x - t_i) / max(t_{i+k} - t_i, 1e-8) * B^{k-1}_i(x)
 *              + (t_{i+k+1} - x) / max(t_{i+k+1} - t_{i+1}, 1e-8) * B^{k-1}_{i+1}(x)
 *
 * up to k = spline_order, giving n_basis = n_knots - 1 - spline_order values per element.
 * Each term is evaluated as ((numerator / clamped difference) * lower-order value) and the two
 * terms added, without fused multiply-adds — the operation order of the reference's PyTorch
 * definition (tests/test_bspline.py:11-24), so fp32 results match it bit for bit.
 *
 * Layout: x [batch, features] fp32 contiguous; grid [features, n_knots] fp32 contiguous;
 * bases [batch, features, n_basis] fp32 contiguous.  1 <= spline_order <= 5,
 * spline_order + 2 <= n_knots <= 64.  Same conventions as kat_rational.h: the caller owns
 * every buffer, nothing is allocated, work is enqueued on `stream` of the current device, the
 * return value is KAT_OK (0) or a KAT_ERR_* code (kat_rational_strerror), and argument errors
 * are reported before anything is enqueued.
 */
#ifndef KAT_BSPLINE_H_
#define KAT_BSPLINE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Forward: bases[b, d, :] = B^{spline_order}_{0..n_basis-1}(x[b, d]) on grid[d, :].
 * Replaces rational_kat_cu/bspline_basis.py:262-296 (bspline_basis_fwd), which is limited to
 * n_knots <= 15 and spline order 3 in its unrolled kernel.
 */
int kat_bspline_basis_fwd(const float* x, const float* grid, float* bases,
                          int64_t batch, int64_t features, int32_t n_knots,
                          int32_t spline_order, void* stream);

/*
 * Backward: grad_x[b, d] = sum_j grad_bases[b, d, j] * d B_j / dx (x[b, d]), the derivative
 * torch autograd takes through the recursion above (the indicator functions contribute
 * nothing; each term contributes +-B^{k-1} / clamped difference plus its factor times the
 * lower-order derivative), evaluated with the B-spline derivative identity
 * dB^K_j/dx = K (B^{K-1}_j / max(t_{j+K} - t_j, 1e-8) - B^{K-1}_{j+1} / max(t_{j+K+1} - t_{j+1}, 1e-8)),
 * which equals that autograd value up to rounding.  Replaces
 * rational_kat_cu/bspline_basis.py:562-599 (bspline_basis_bwd).  The grid gets no gradient, as in
 * the reference.
 */
int kat_bspline_basis_bwd(const float* x, const float* grid, const float* grad_bases,
                          float* grad_x, int64_t batch, int64_t features, int32_t n_knots,
                          int32_t spline_order, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KAT_BSPLINE_H_ */
