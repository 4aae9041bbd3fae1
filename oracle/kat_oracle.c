/*
 * ORACLE — test infrastructure only.  Built into oracle/_build/libkat_oracle.so and loaded
 * by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg; never by the library.
 *
 * Float64 restatement of the reference's group-rational formula
 * (kat_rational/kat_1dgroup_torch.py:27-78 of felippe-alves/rational_kat_cu):
 *
 *   P(x) = sum_{k=0..5} a_k x^k                       (:57-60, powers by repeated product :7-24)
 *   Q(x) = 1 + sum_{i=1..4} |b_i| x^i                 (:63-69, abs on coefficients, raw x)
 *   y    = P / Q                                      (:72)
 *
 * and of the gradients torch autograd derives for it (abs backward = sgn, sgn(0) = 0):
 *
 *   dx       = go (P' Q - P Q') / Q^2
 *   d a[g,k] = sum_{elements of group g} go x^k / Q
 *   d b[g,i] = sgn(b[g,i]) sum_{elements of group g} -go P x^(i+1) / Q^2   (b index i = 0..3)
 *
 * Layout: contiguous [batch, channels, inner]; channel c is in group c / (channels/groups).
 * Besides the values, every routine returns "magnitudes": first-order bounds, in units of
 * the unit roundoff, on how far any fp32 evaluation of the same expression (any term order,
 * Horner or stacked powers) can drift.  With Pm = sum |a_k||x|^k, Qm = 1 + sum |b_i||x|^i
 * (and P'm, Q'm likewise) and the cancellation ratio rq = Qm / |Q|:
 *   y_mag  = (Pm + |y| Qm) / |Q|
 *   dx_mag = |go| / |Q| (P'm + (y_mag + |y|) Q'm) + |dx| rq
 *   numerator-gradient term k:   |go x^k / Q| (1 + rq)
 *   denominator-gradient term i: |go| (Pm + 2 |P| rq) |x|^i / Q^2
 * The tests scale their tolerances by these (a pole, Q -> 0, makes them large).
 *
 * Coefficient-gradient sums are accumulated per fixed chunk of rows and the chunk results
 * are added in chunk order, so the output does not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define NUM 6
#define DEN 4
#define ROWS_PER_CHUNK 64

typedef struct {
  double a[NUM];
  double c[DEN];   /* |b_i| */
} coef_t;

static void load_coef(const float* num, const float* den, int64_t g, coef_t* k) {
  for (int i = 0; i < NUM; ++i) k->a[i] = (double)num[g * NUM + i];
  for (int i = 0; i < DEN; ++i) k->c[i] = fabs((double)den[g * DEN + i]);
}

/* One element: values and magnitudes of P, Q, P', Q'. */
typedef struct {
  double p, q, dp, dq;
  double p_mag, q_mag, dp_mag, dq_mag;
} eval_t;

static inline void eval_elem(double x, const coef_t* k, eval_t* e) {
  double pw[NUM];           /* x^0 .. x^5 by repeated product */
  pw[0] = 1.0;
  for (int i = 1; i < NUM; ++i) pw[i] = pw[i - 1] * x;
  const double ax = fabs(x);
  double apw[NUM];
  apw[0] = 1.0;
  for (int i = 1; i < NUM; ++i) apw[i] = apw[i - 1] * ax;
  e->p = 0.0; e->p_mag = 0.0;
  for (int i = 0; i < NUM; ++i) {
    e->p += k->a[i] * pw[i];
    e->p_mag += fabs(k->a[i]) * apw[i];
  }
  e->q = 1.0; e->q_mag = 1.0;
  for (int i = 0; i < DEN; ++i) {
    e->q += k->c[i] * pw[i + 1];
    e->q_mag += k->c[i] * apw[i + 1];
  }
  e->dp = 0.0; e->dp_mag = 0.0;
  for (int i = 1; i < NUM; ++i) {
    e->dp += (double)i * k->a[i] * pw[i - 1];
    e->dp_mag += (double)i * fabs(k->a[i]) * apw[i - 1];
  }
  e->dq = 0.0; e->dq_mag = 0.0;
  for (int i = 0; i < DEN; ++i) {
    e->dq += (double)(i + 1) * k->c[i] * pw[i];
    e->dq_mag += (double)(i + 1) * k->c[i] * apw[i];
  }
}

/* y[n] = P/Q and its magnitude y_mag[n] (either output may be NULL). */
void kat_oracle_forward(const float* x, int64_t batch, int64_t channels, int64_t inner,
                        int64_t groups, const float* num, const float* den,
                        double* y, double* y_mag) {
  const int64_t per = channels / groups;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < batch; ++b) {
    for (int64_t ch = 0; ch < channels; ++ch) {
      coef_t k;
      load_coef(num, den, ch / per, &k);
      const int64_t base = (b * channels + ch) * inner;
      for (int64_t s = 0; s < inner; ++s) {
        eval_t e;
        eval_elem((double)x[base + s], &k, &e);
        const double yv = e.p / e.q;
        if (y) y[base + s] = yv;
        if (y_mag) y_mag[base + s] = (e.p_mag + fabs(yv) * e.q_mag) / fabs(e.q);
      }
    }
  }
}

/*
 * Backward.  dx / dx_mag may be NULL.  d_num [G,6], d_den [G,4] receive the coefficient
 * gradients (d_den with the sgn(b) factor applied); d_num_mag / d_den_mag (may be NULL)
 * receive the sums of absolute terms.
 */
void kat_oracle_backward(const float* x, const float* grad_out, int64_t batch,
                         int64_t channels, int64_t inner, int64_t groups, const float* num,
                         const float* den, double* dx, double* dx_mag, double* d_num,
                         double* d_den, double* d_num_mag, double* d_den_mag) {
  const int64_t per = channels / groups;
  const int64_t n_chunks = (batch + ROWS_PER_CHUNK - 1) / ROWS_PER_CHUNK;
  const int64_t acc_len = groups * 20;   /* 10 sums + 10 magnitude sums per group */
  double* part = (double*)calloc((size_t)(n_chunks > 0 ? n_chunks : 1) * (size_t)acc_len,
                                 sizeof(double));
#pragma omp parallel for schedule(static)
  for (int64_t chunk = 0; chunk < n_chunks; ++chunk) {
    double* acc = part + chunk * acc_len;
    const int64_t b1 = (chunk + 1) * ROWS_PER_CHUNK < batch ? (chunk + 1) * ROWS_PER_CHUNK : batch;
    for (int64_t b = chunk * ROWS_PER_CHUNK; b < b1; ++b) {
      for (int64_t ch = 0; ch < channels; ++ch) {
        const int64_t g = ch / per;
        coef_t k;
        load_coef(num, den, g, &k);
        double* ag = acc + g * 20;
        const int64_t base = (b * channels + ch) * inner;
        for (int64_t s = 0; s < inner; ++s) {
          const double xv = (double)x[base + s];
          const double go = (double)grad_out[base + s];
          eval_t e;
          eval_elem(xv, &k, &e);
          const double u = go / e.q;               /* go / Q */
          const double yv = e.p / e.q;
          const double w = u * yv;                 /* go P / Q^2 */
          const double dxv = u * (e.dp - yv * e.dq);
          const double rq = e.q_mag / fabs(e.q);
          if (dx) dx[base + s] = dxv;
          if (dx_mag) {
            const double ymag = (e.p_mag + fabs(yv) * e.q_mag) / fabs(e.q);
            dx_mag[base + s] = fabs(u) * (e.dp_mag + (ymag + fabs(yv)) * e.dq_mag) + fabs(dxv) * rq;
          }
          const double num_m = fabs(u) * (1.0 + rq);
          const double den_m = fabs(go) * (e.p_mag + 2.0 * fabs(e.p) * rq) / (e.q * e.q);
          double pw = 1.0, apw = 1.0;
          for (int i = 0; i < NUM; ++i) {
            ag[i] += u * pw;
            ag[10 + i] += num_m * apw;
            if (i >= 1 && i <= DEN) {
              ag[NUM + i - 1] += -w * pw;
              ag[10 + NUM + i - 1] += den_m * apw;
            }
            pw *= xv;
            apw *= fabs(xv);
          }
        }
      }
    }
  }
  for (int64_t g = 0; g < groups; ++g) {
    double s[20];
    memset(s, 0, sizeof(s));
    for (int64_t chunk = 0; chunk < n_chunks; ++chunk)
      for (int i = 0; i < 20; ++i) s[i] += part[chunk * acc_len + g * 20 + i];
    for (int i = 0; i < NUM; ++i) {
      d_num[g * NUM + i] = s[i];
      if (d_num_mag) d_num_mag[g * NUM + i] = s[10 + i];
    }
    for (int i = 0; i < DEN; ++i) {
      const double b = (double)den[g * DEN + i];
      const double sg = b > 0.0 ? 1.0 : (b < 0.0 ? -1.0 : b * 0.0);
      d_den[g * DEN + i] = sg * s[NUM + i];
      if (d_den_mag) d_den_mag[g * DEN + i] = s[10 + NUM + i];
    }
  }
  free(part);
}

int kat_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
