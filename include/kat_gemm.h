/*
 * kat_gemm.h — C ABI of the tensor-core GEMMs with a fused group-rational epilogue in
 * libkat_rational.so (sm_100a: tcgen05 MMA with the accumulator in tensor memory, TMA tile
 * loads and stores, one persistent CTA per SM).
 *
 * The reference's GR-KAN block (README.md:20-51) runs
 *     act1 ('identity' KAT) -> drop -> fc1 -> act2 ('gelu' KAT) -> drop -> fc2
 * so the activation act2 (kat_rational/kat_1dgroup_triton.py:80-87 -> rational_triton.py:241-297)
 * sits between two GEMMs: its forward consumes fc1's output and its backward consumes fc2's
 * input gradient.  These entry points compute the GEMM and the activation in one kernel, so the
 * [rows, hidden] activation tensor does not make an extra round trip through HBM:
 *
 *   kat_gemm_rational_fwd:  h = A B^T + bias,  y = P(h) / Q(h)          (fc1 + act2 forward)
 *   kat_gemm_rational_bwd:  g = A B^T,  dh = g * dy/dh (h),  d_num, d_den (fc2 dgrad + act2 backward)
 *   kat_gemm_bf16:          C = A B^T + bias                           (the same GEMM, no epilogue)
 *
 * A [M, K] and B [N, K] are bf16 row-major (both K-contiguous: for fc1, A = the block input and
 * B = fc1.weight; for fc2's input gradient, A = dL/d(fc2 output) and B = fc2.weight transposed to
 * [hidden, out]).  Accumulation is fp32 in tensor memory; outputs are bf16 row-major [M, N].
 * The rational function is the KAT formula of kat_rational.h (or the abs-after-sum one) with
 * group g = column / (N / num_groups), coefficients num [G, 6] and den [G, 4] fp32.
 *
 * Rounding contract (what the tests check bit for bit): h is the fp32 accumulator plus the bf16
 * bias, rounded to bf16; y is exactly what kat_rational_fwd gives for that bf16 h.  In the
 * backward, g is the fp32 accumulator rounded to bf16 (what kat_gemm_bf16 returns for the same
 * operands) and dh is exactly what kat_rational_bwd gives for (h, g); the coefficient gradients
 * are fixed-order fp64 sums of fp32 per-thread partials, bit-reproducible on one GPU model.
 *
 * Shapes: M >= 0 (M = 0 is a no-op; the backward then writes zero coefficient gradients); N a
 * multiple of 256; K a multiple of 64; N / num_groups a multiple of 32;
 * M, N, K below 2^31.  Pointers (bias included) 16-byte aligned, else KAT_ERR_BAD_SHAPE (a TMA
 * tensor map needs it).  Same conventions as
 * kat_rational.h: the caller owns every buffer (the backward's workspace included), nothing is
 * allocated, work is enqueued on `stream` of the current device, argument errors are reported
 * before anything is enqueued, and the return value is KAT_OK or a KAT_ERR_* code.
 */
#ifndef KAT_GEMM_H_
#define KAT_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* C = A B^T (+ bias[N] if bias != NULL), bf16 out.  The mainloop shared by the two fused
 * entry points; kat_gemm_rational_bwd's g equals this C for bias == NULL. */
int kat_gemm_bf16(const void* a, const void* b, const void* bias, void* c,
                  int64_t m, int64_t n, int64_t k, void* stream);

/* fc1 + act2 forward: h = A B^T + bias (bias may be NULL), y = rational(h).  Replaces the
 * GEMM followed by kat_rational/kat_1dgroup_triton.py:80-87 (KAT_Group.forward) on its output;
 * h is kept for the backward as the reference's autograd keeps the activation input
 * (rational_triton.py:250-251).  h may be NULL when no backward follows (inference): only y is
 * written. */
int kat_gemm_rational_fwd(const void* a, const void* b, const void* bias,
                          const float* num, const float* den, void* h, void* y,
                          int64_t m, int64_t n, int64_t k, int32_t num_groups,
                          int32_t formula, void* stream);

/* Workspace bytes kat_gemm_rational_bwd needs for this shape on `device` (fp64 per-CTA
 * partial sums of the coefficient gradients). */
size_t kat_gemm_rational_bwd_workspace_bytes(int64_t m, int64_t n, int32_t num_groups,
                                             int device);

/* fc2 input-gradient GEMM + act2 backward: g = A B^T (not stored), dh = g * y'(h), d_num [G, 6]
 * and d_den [G, 4] (fp32) the activation's coefficient gradients over all M x N elements.
 * Replaces the dgrad GEMM followed by rational_triton.py:271-297 (RationalTriton1DGroup
 * backward) on its output. */
int kat_gemm_rational_bwd(const void* a, const void* b, const void* h,
                          const float* num, const float* den, void* dh,
                          float* d_num, float* d_den, void* workspace, size_t workspace_bytes,
                          int64_t m, int64_t n, int64_t k, int32_t num_groups,
                          int32_t formula, void* stream);

/* Sticky device status of these kernels on `device` (0 = ok; KAT_DEVICE_WAIT_TIMEOUT when a
 * pipeline wait ran out — the kernel then stopped without finishing its tiles), optionally
 * reset to 0.  Synchronous (reads a device word). */
int kat_gemm_device_status(int device, int reset, int* status);

/* Test only: on != 0 makes every following GEMM launch in this process stall its MMA issuer on
 * a barrier that nothing completes, so the launch exercises its bounded-wait path (returns
 * after about two seconds with KAT_DEVICE_WAIT_TIMEOUT in the status word and undefined
 * outputs); on == 0 turns it off again.  Off by default; nothing but a test calls it.
 * No counterpart in the reference, whose kernels have no device-side waits. */
int kat_gemm_set_test_stall(int on);

#ifdef __cplusplus
}
#endif

#endif /* KAT_GEMM_H_ */
