/*
 * kat_rational.h — C ABI of the B200 (sm_100a) group-rational activation library
 * (libkat_rational.so).
 *
 * The activation is KAT's group rational function, evaluated exactly as the
 * reference's PyTorch path does (kat_rational/kat_1dgroup_torch.py:27-78):
 *
 *     y = P(x) / Q(x),   P(x) = a0 + a1 x + a2 x^2 + a3 x^3 + a4 x^4 + a5 x^5
 *                        Q(x) = 1 + |b1| x + |b2| x^2 + |b3| x^3 + |b4| x^4
 *
 * with one coefficient set (a[g,0..5], b[g,0..3]) per channel group g.  The
 * absolute value is taken on the denominator coefficients only; the powers of x
 * are raw (kat_1dgroup_torch.py:63-69), so Q can reach zero for x < 0.
 *
 * Tensor layout.  Every data tensor is contiguous and viewed as
 * [batch, channels, inner]:
 *   - channels-last input [B, L, C] or [B, C]  -> batch = B*L (or B), inner = 1
 *   - NCHW input [B, C, H, W]                  -> batch = B,   inner = H*W
 * Channel c belongs to group c / (channels / num_groups).
 *
 * Conventions.
 *   - The caller owns every buffer (inputs, outputs and the backward workspace).
 *     The library allocates no device memory, never synchronises the host and
 *     enqueues work only on the given stream (a cudaStream_t passed as void*;
 *     NULL = the legacy default stream) of the current CUDA device.
 *   - Coefficients are fp32: numerator [num_groups, 6], denominator [num_groups, 4].
 *   - Data tensors (x, y, grad_out, grad_x) share one dtype (KAT_DTYPE_*); all
 *     arithmetic is fp32 and a 16-bit output is rounded once, to nearest even.
 *   - Pointers of any alignment are accepted; 16-byte-aligned tensors whose group
 *     width is a multiple of the vector width take the 128-bit vector path.
 *   - Every entry point returns KAT_OK (0) or a KAT_ERR_* code; kat_rational_strerror()
 *     describes it.  Argument errors are detected before anything is enqueued.
 *   - Coefficient gradients are reduced in a fixed order (per-thread fp32 sums,
 *     then fp64 per-block and grid sums, no floating-point atomics): for a given
 *     shape, dtype and GPU model the results are bit-identical run to run.
 */
#ifndef KAT_RATIONAL_H_
#define KAT_RATIONAL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KAT_RATIONAL_ABI_VERSION 3

/* Data-tensor element types. */
#define KAT_DTYPE_F32 0
#define KAT_DTYPE_F16 1
#define KAT_DTYPE_BF16 2

/* Status codes. */
#define KAT_OK 0
#define KAT_ERR_NULL_POINTER 1      /* a required pointer is NULL */
#define KAT_ERR_BAD_DTYPE 2         /* dtype is not one of KAT_DTYPE_* */
#define KAT_ERR_BAD_SHAPE 3         /* negative extent, or size overflow */
#define KAT_ERR_BAD_GROUPS 4        /* num_groups < 1 or channels % num_groups != 0 */
#define KAT_ERR_WORKSPACE 5         /* workspace NULL or smaller than required */
#define KAT_ERR_CUDA 6              /* CUDA runtime / launch error */
#define KAT_ERR_SCRATCH_LIMIT 7     /* kat_rational_bwd_noalloc: problem exceeds its fixed scratch */
#define KAT_ERR_BAD_FORMULA 8       /* formula is not one of KAT_FORMULA_* */

/* Denominator formulas (the *_formula entry points). */
#define KAT_FORMULA_KAT 0      /* Q = 1 + sum_i |b_i| x^i       (kat_rational/kat_1dgroup_torch.py) */
#define KAT_FORMULA_ABS_SUM 1  /* Q = 1 + |sum_i b_i x^i|       (rational_kat_cu rat_cuda) */
/* Flag or-ed into `formula` of kat_rational_fwd_formula / kat_rational_bwd_formula: `numerator`
 * is ONE row of 6 coefficients used by every group (the modules' weight_numerator [1, 6],
 * which the reference repeats per group on every forward: kat_rational/kat_1dgroup_triton.py:86),
 * and the backward writes grad_numerator as ONE row [6], the sum over groups of the per-group
 * gradients (added in fp64 in a fixed order, rounded once) — the gradient the reference's
 * repeat backward produces, without the repeat and the sum as separate launches.  Also accepted
 * by kat_rational_bwd_allreduce_formula (data parallel). */
#define KAT_SHARED_NUMERATOR 0x100

/*
 * Forward: y = P(x)/Q(x).
 * Replaces the reference's forward launchers
 *   kat_rational/rational_triton.py:76-94   (rational_fwd_triton, [B,L,C] / [B,C])
 *   kat_rational/rational_triton2d.py:71-91 (rational_fwd_triton_2d, [B,C,H,W])
 * with the formula of kat_rational/kat_1dgroup_torch.py:27-78.
 */
int kat_rational_fwd(const void* x, void* y,
                     const float* numerator,    /* [num_groups, 6] */
                     const float* denominator,  /* [num_groups, 4] */
                     int64_t batch, int64_t channels, int64_t inner,
                     int64_t num_groups, int dtype, void* stream);

/*
 * Backward: grad_x = dy/dx * grad_out, and the coefficient gradients
 *   grad_numerator[g,k]   = sum over group g of grad_out * x^k / Q
 *   grad_denominator[g,i] = sgn(b[g,i]) * sum over group g of -grad_out * P * x^(i+1) / Q^2
 * (sgn(0) = 0, as torch's abs backward).  Both coefficient gradients are fully
 * overwritten (no accumulation into existing values).  grad_x may be NULL, in
 * which case only the coefficient gradients are produced.
 * `workspace` must hold at least kat_rational_bwd_workspace_size() bytes and be
 * 16-byte aligned; its contents on entry are irrelevant.
 * Replaces kat_rational/rational_triton.py:217-238 (rational_bwd_triton) and
 * kat_rational/rational_triton2d.py:194-220 (rational_bwd_triton_2d); the
 * gradients are those torch autograd derives for kat_1dgroup_torch.py:27-78.
 * Launches two kernels on `stream`: the fused elementwise/partial-sum kernel and
 * the fixed-order grid reduction.
 */
int kat_rational_bwd(const void* x, const void* grad_out, void* grad_x,
                     const float* numerator, const float* denominator,
                     float* grad_numerator,     /* [num_groups, 6] */
                     float* grad_denominator,   /* [num_groups, 4] */
                     void* workspace, size_t workspace_bytes,
                     int64_t batch, int64_t channels, int64_t inner,
                     int64_t num_groups, int dtype, void* stream);

/*
 * The same forward and backward with a selectable denominator formula.
 * formula = KAT_FORMULA_KAT is exactly kat_rational_fwd / kat_rational_bwd.
 * formula = KAT_FORMULA_ABS_SUM is the `rat_cuda` front end of the reference:
 *     Q(x) = 1 + |D(x)|,  D(x) = b0 x + b1 x^2 + b2 x^3 + b3 x^4  (raw coefficients,
 *     absolute value after the sum; D by Horner, then times x)
 * forward as kat_rational/rational_triton.py:22-72 (rational_fwd_triton, called by
 * rational_kat_cu/__init__.py:29), backward as rational_kat_cu/rational_bwd_triton.py:
 *     grad_x                = (P' Q - P sgn(D) D') / Q^2 * grad_out
 *     grad_numerator[g,k]   = sum over group g of grad_out * x^k / Q
 *     grad_denominator[g,j] = sum over group g of -grad_out * P * sgn(D) * x^(j+1) / Q^2
 * with sgn(D) = -1 where D < 0 and +1 elsewhere (D = 0 included), as the reference
 * kernels' where(D < 0, -1, 1).  Same layout, workspace (kat_rational_bwd_workspace_size
 * covers both formulas), determinism and error rules as the KAT entry points.
 * Replaces rational_kat_cu/__init__.py:29-40 (the Triton launchers of _RationalGroupedFn).
 */
int kat_rational_fwd_formula(const void* x, void* y,
                             const float* numerator, const float* denominator,
                             int64_t batch, int64_t channels, int64_t inner,
                             int64_t num_groups, int dtype, int formula, void* stream);

int kat_rational_bwd_formula(const void* x, const void* grad_out, void* grad_x,
                             const float* numerator, const float* denominator,
                             float* grad_numerator, float* grad_denominator,
                             void* workspace, size_t workspace_bytes,
                             int64_t batch, int64_t channels, int64_t inner,
                             int64_t num_groups, int dtype, int formula, void* stream);

/*
 * Forward in float64 for float64 tensors, either formula: x, y and the coefficients
 * (numerator [num_groups, 6], denominator [num_groups, 4]) are all double and every
 * operation is float64.  For gradient checking: the reference's Triton forward loads its
 * input without a cast and so evaluates float64 inputs in float64
 * (kat_rational/rational_triton.py:36-72).  A plain grid-stride kernel (no vector path);
 * no float64 backward is provided (the reference's backward kernels compute in fp32, and
 * the Python wrappers run float64 backward through the fp32 entry points).
 */
int kat_rational_fwd_f64(const double* x, double* y,
                         const double* numerator, const double* denominator,
                         int64_t batch, int64_t channels, int64_t inner,
                         int64_t num_groups, int formula, void* stream);

/*
 * Backward without any device allocation, for callers that cannot allocate where they run
 * it: plugin hosts whose operator interface hands the operator its input and output
 * buffers but no allocator, and fixed-budget real-time loops where a cudaMalloc in the
 * middle of a run could stall the device or fail.  Same arguments and results as
 * kat_rational_bwd minus the workspace: the partial sums go to a fixed 2 MiB file-scope
 * device array instead, which every GPU that loads this library holds until the process
 * exits.
 *   - Problems whose backward needs more than 2 MiB of scratch
 *     (kat_rational_bwd_workspace_size) are rejected with KAT_ERR_SCRATCH_LIMIT before
 *     anything is enqueued.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current) and caches it for the life of the
 *     process; make that first call before any stream capture.  The cached address belongs
 *     to the device's current primary context: after cudaDeviceReset (or anything else that
 *     destroys that context) do not call this entry point again in the same process.  No
 *     call allocates (no cudaMalloc / cudaFree).
 *   - Every call on a device shares the one array and leaves the last call's partial sums in
 *     it; each call writes every entry it later reads, so nothing needs clearing.  Calls
 *     that can overlap on the GPU (different streams, or different host threads) race on
 *     the array: order them on one stream.
 * No counterpart in the reference, whose backward allocates with torch.zeros in its launcher.
 */
int kat_rational_bwd_noalloc(const void* x, const void* grad_out, void* grad_x,
                             const float* numerator, const float* denominator,
                             float* grad_numerator, float* grad_denominator,
                             int64_t batch, int64_t channels, int64_t inner,
                             int64_t num_groups, int dtype, void* stream);

/*
 * Bytes of workspace kat_rational_bwd needs for this problem on `device`
 * (an upper bound over every pointer alignment).  No counterpart in the
 * reference, whose backward allocates with torch.zeros inside the launcher
 * (kat_rational/rational_triton.py:224-226).
 */
int kat_rational_bwd_workspace_size(int64_t batch, int64_t channels, int64_t inner,
                                    int64_t num_groups, int dtype, int device,
                                    size_t* bytes);

/*
 * Sticky device-side status word of `device`: 0, or KAT_DEVICE_WAIT_TIMEOUT when a
 * pipelined kernel gave up on a bounded wait (its outputs are then undefined).  Reads the
 * word synchronously (waits for the device's pending work); reset != 0 clears it.
 * No counterpart in the reference, whose kernels have no device-side waits.
 */
#define KAT_DEVICE_WAIT_TIMEOUT 1
/* Set only by the bounds-checked debug build of this library (libkat_rational_debug.so,
 * compiled with -DKAT_DEBUG_BOUNDS=1): a kernel found a global access, a workspace slot or a
 * plan invariant out of range and skipped the access instead of making it. */
#define KAT_DEVICE_BOUNDS 3
int kat_rational_device_status(int device, int reset, int* status);

/*
 * Data-parallel backward: kat_rational_bwd whose coefficient gradients are, in the same
 * call, exchanged with every other rank over NVLink peer memory and added in rank order
 * (optionally averaged), so every rank ends with the same bit-identical gradients.  grad_x
 * stays local.  `peers` describes the ranks of one node: buffers[r] is rank r's exchange
 * buffer (kat_rational_exchange_buffer_bytes(num_groups) bytes, 16-byte aligned,
 * zero-filled once before the first call) as mapped into this process (peer access or IPC);
 * buffers[rank] is this rank's own.  Every rank must make the same sequence of calls: the
 * k-th call of each rank pairs with the k-th call of the others.  A rank that does not
 * arrive within timeout_ms makes the others set KAT_DEVICE_EXCHANGE_TIMEOUT in the device
 * status word and write NaN gradients (the kernel returns; the context stays usable).
 * Failure is fail-stop: a rank whose wait ran out marks its own exchange buffer broken, and
 * every later call with that buffer writes NaN gradients and stores nothing to any peer, so
 * no rank ever adds data of two different calls.  Rebuild the buffers (every rank) to go on.
 * Replaces the reference's (absent) distributed layer; no counterpart there.
 */
#define KAT_MAX_PEERS 8
#define KAT_DEVICE_EXCHANGE_TIMEOUT 2
typedef struct kat_rational_peers {
  int32_t world_size;               /* 1 .. KAT_MAX_PEERS */
  int32_t rank;                     /* this process's rank */
  int32_t average;                  /* nonzero: divide the sum by world_size */
  int32_t timeout_ms;               /* bound on the wait for the other ranks */
  void* buffers[KAT_MAX_PEERS];     /* every rank's exchange buffer, mapped here */
} kat_rational_peers;

size_t kat_rational_exchange_buffer_bytes(int64_t num_groups);

/* Let kernels on `device` access memory of `peer_device` (NVLink peer access; idempotent). */
int kat_rational_enable_peer_access(int device, int peer_device);

/*
 * Exchange-buffer set-up for kat_rational_bwd_allreduce across processes (one per GPU),
 * outside the per-step path (these calls allocate / map memory and synchronise):
 *   create   cudaMalloc a zeroed local buffer of kat_rational_exchange_buffer_bytes(G) on the
 *            current device and write its 64-byte CUDA IPC handle to `ipc_handle`;
 *   open     map a peer's buffer from its handle on the current device (lazy peer access),
 *            then check it is reachable (pointer attributes + a 16-byte copy into the
 *            caller's 16-byte `local_probe` device buffer) — an unreachable mapping is an
 *            error here, never a kernel fault later;
 *   close / destroy  undo open / create.
 */
int kat_rational_exchange_create(int64_t num_groups, void** buffer, void* ipc_handle);
int kat_rational_exchange_open(const void* ipc_handle, void* local_probe, void** peer_buffer);
int kat_rational_exchange_close(void* peer_buffer);
int kat_rational_exchange_destroy(void* buffer);

int kat_rational_bwd_allreduce(const void* x, const void* grad_out, void* grad_x,
                               const float* numerator, const float* denominator,
                               float* grad_numerator, float* grad_denominator,
                               void* workspace, size_t workspace_bytes,
                               int64_t batch, int64_t channels, int64_t inner,
                               int64_t num_groups, int dtype,
                               const kat_rational_peers* peers, void* stream);

/*
 * kat_rational_bwd_allreduce with a `formula` argument: KAT_FORMULA_KAT, optionally or-ed with
 * KAT_SHARED_NUMERATOR (one numerator row [6] for every group; grad_numerator [6] is the sum
 * over groups of the rank-summed per-group gradients, added in the same fixed fp64 order as
 * kat_rational_bwd_formula's, so at world size 1 both give the same bits).  The abs-after-sum
 * formula is refused (KAT_ERR_BAD_FORMULA).  No counterpart in the reference.
 */
int kat_rational_bwd_allreduce_formula(const void* x, const void* grad_out, void* grad_x,
                                       const float* numerator, const float* denominator,
                                       float* grad_numerator, float* grad_denominator,
                                       void* workspace, size_t workspace_bytes,
                                       int64_t batch, int64_t channels, int64_t inner,
                                       int64_t num_groups, int dtype, int formula,
                                       const kat_rational_peers* peers, void* stream);

/*
 * The exchange step alone, for callers that reduce their coefficient gradients themselves (the
 * host-buffer pipeline sums its row chunks' gradients first): grad_numerator [num_groups, 6]
 * and grad_denominator [num_groups, 4] (fp32, this rank's gradients, device memory) are
 * replaced in place by the rank-order fp64 sum over every rank of `peers` (divided by
 * world_size when peers->average), rounded once to fp32, the same bits on every rank.  It
 * shares the exchange buffers, the epoch counter and the fail-stop rules of
 * kat_rational_bwd_allreduce: each call of either entry point is one exchange, and every rank
 * makes the same sequence of calls.  On failure the gradients become NaN and the status word
 * reads KAT_DEVICE_EXCHANGE_TIMEOUT.  Replaces the reference's (absent) distributed layer; no
 * counterpart there.
 */
int kat_rational_exchange_grads(float* grad_numerator, float* grad_denominator,
                                int64_t num_groups, const kat_rational_peers* peers,
                                void* stream);

/* Human-readable text for a status code (static storage). */
const char* kat_rational_strerror(int status);

/* KAT_RATIONAL_ABI_VERSION of the loaded library. */
int kat_rational_abi_version(void);

/*
 * Launch geometry chosen for a problem, for inspection and tests.  Pure host
 * arithmetic: it touches no GPU.  `sm_count` and `ctas_per_sm` stand in for the
 * device's multiprocessor count and the kernel's occupancy; `vec` is the
 * elements-per-vector the kernels would use (0 = the widest the shape allows).
 */
typedef struct kat_rational_plan {
  int64_t rows;          /* batch */
  int64_t width;         /* channels * inner: elements per row */
  int64_t group_width;   /* (channels / num_groups) * inner */
  int64_t num_groups;
  int32_t vec;           /* elements per vector load */
  int32_t threads;       /* threads per block = tile_cols * tile_rows */
  int32_t tile_cols;     /* vector columns per block */
  int32_t tile_rows;     /* rows a block advances per step */
  int64_t col_blocks;    /* blocks across a row */
  int64_t items;         /* col_blocks * rows: the units split across blocks */
  int64_t blocks;        /* grid size */
  int32_t max_segments;  /* column blocks one block can touch */
  int32_t max_local_groups;  /* groups one column block can touch */
  uint64_t workspace_bytes;  /* backward partial-sum buffer */
  /* Block split: 0 = the items are split evenly over all blocks; > 0 = each block stays in
   * one column block, the first `col_block_extra` column blocks get col_block_blocks + 1
   * blocks and the others col_block_blocks, and a column block's rows are split evenly. */
  int64_t col_block_blocks;
  int64_t col_block_extra;
} kat_rational_plan;

int kat_rational_make_plan(int64_t batch, int64_t channels, int64_t inner,
                           int64_t num_groups, int dtype, int vec,
                           int sm_count, int ctas_per_sm,
                           kat_rational_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* KAT_RATIONAL_H_ */
