/*
 * flashslice_b200 -- C ABI of the B200 (sm_100a) slice/deslice coupling.
 *
 * The reference (Shizheng-Wen/flashslice v0.3.0) exposes this path as Python
 * functions that launch Triton kernels; each entry point below replaces one
 * of its host launchers, with the same argument meaning:
 *
 *   fs_slice_fwd    <- _slice_impl            flashslice/kernels/slice_ops.py:804-819
 *                      _slice_blk_impl        flashslice/kernels/blocked.py:1346-1368
 *   fs_deslice_fwd  <- _deslice_impl          slice_ops.py:846-859
 *                      _deslice_blk_impl      blocked.py:1406-1433
 *   fs_slice_bwd    <- _slice_bwd_impl        slice_ops.py:822-843
 *                      _slice_blk_bwd_impl    blocked.py:1371-1403
 *   fs_deslice_bwd  <- _deslice_bwd_impl      slice_ops.py:862-885
 *                      _deslice_blk_bwd_impl  blocked.py:1436-1469
 *   fs_compute_stats<- compute_stats          blocked.py:1329-1343
 *   fs_workspace_bytes: the partial-sum buffers the reference allocates with
 *                      torch.empty inside each launcher (slice_ops.py:811-814).
 *
 * Conventions
 *   - Shapes: x_mid (B, N, H, D); fx_mid, d_out, out (B, N, H, DV);
 *     tokens, z_num, dz_num, dtokens (B, H, G, DV) fp32 contiguous;
 *     s, ds (B, H, G) fp32 contiguous; tau, dtau (H,) fp32;
 *     stats (B, H, 2, N) fp32 contiguous: [.., 0, n] row max m, [.., 1, n]
 *     sum of exponentials l (blocked.py:293-346).
 *   - The slice weight is fp32 contiguous of shape (w_batch, w_heads, G, D)
 *     with w_batch in {1, B} and w_heads in {1, H}: (G, D), (H, G, D) and
 *     (B, H, G, D) of the reference (slice_ops.py:503-526). The bias is
 *     fp32 contiguous (b_batch, b_heads, G); a missing bias is zeros(G).
 *     dW / db are returned in those same shapes, summed over the shared axes
 *     (slice_ops.py:481-500).
 *   - The point tensors (fs_tensor4) are read and written through arbitrary
 *     element strides (b, n, h, width) in act_dtype.
 *   - Every call enqueues on `stream` (a cudaStream_t) and returns at once.
 *     Results are bitwise deterministic for a given shape: no atomics; every
 *     reduction runs in a fixed order.
 *   - Workspace: caller-allocated device memory of at least
 *     fs_workspace_bytes(op, p) bytes, 256-byte aligned.
 *   - Return value: FS_OK or an fs_status code; fs_last_error() describes the
 *     last failure of the calling thread.
 */
#ifndef FLASHSLICE_B200_H
#define FLASHSLICE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FS_ABI_VERSION 2

#if defined(__GNUC__)
#define FS_API __attribute__((visibility("default")))
#else
#define FS_API
#endif

typedef enum fs_dtype { FS_F32 = 0, FS_BF16 = 1, FS_F16 = 2 } fs_dtype;

typedef enum fs_status {
  FS_OK = 0,
  FS_ERR_SHAPE = 1,       /* bad extents / layout (reference: ValueError)   */
  FS_ERR_ARGUMENT = 2,    /* null pointer, bad enum, bad mode               */
  FS_ERR_WORKSPACE = 3,   /* workspace too small or misaligned              */
  FS_ERR_CUDA = 4,        /* a CUDA launch or runtime call failed           */
  FS_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up             */
  FS_ERR_UNSUPPORTED = 6  /* dims outside the supported range (D, DV > 256) */
} fs_status;

typedef enum fs_op {
  FS_OP_SLICE_FWD = 0,
  FS_OP_DESLICE_FWD = 1,
  FS_OP_SLICE_BWD = 2,
  FS_OP_DESLICE_BWD = 3,
  FS_OP_STATS = 4
} fs_op;

/* Family: which reference kernel family's contract the call follows.
 * FS_FAMILY_SINGLE forms the softmax whole per point and neither takes nor
 * returns statistics (slice_ops.py); FS_FAMILY_BLOCKED works from the
 * per-point statistics (m, l), takes them when given and returns them
 * (blocked.py). */
typedef enum fs_family { FS_FAMILY_SINGLE = 0, FS_FAMILY_BLOCKED = 1 } fs_family;

typedef struct fs_problem {
  int64_t B, N, H, D, DV, G;
  int32_t act_dtype;   /* fs_dtype of the point tensors                        */
  int32_t dot;         /* dot level 0 ieee .. 4 tf32x3 (slice_ops.py:336-360)  */
  int32_t family;      /* fs_family                                            */
  int32_t stats_mode;  /* 0 online, 1 two-pass (blocked.py:101-120)            */
  int32_t w_batch, w_heads; /* weight leading extents: 1 or B, 1 or H          */
  int32_t b_batch, b_heads; /* bias leading extents: 1 or B, 1 or H            */
  int32_t flags;       /* FS_FLAG_* : which optional statistics buffers the
                          call passes; part of the workspace size contract    */
  int32_t engine;      /* FS_ENGINE_*: 0 lets the library choose */
  /* Ragged samples (NULL: B dense samples of N points each). Otherwise a
   * HOST array of B + 1 non-decreasing row offsets, row_splits[0] = 0 and
   * row_splits[B] = N: the point tensors hold one batch entry of N rows and
   * sample b owns rows [row_splits[b], row_splits[b + 1]); weight, bias,
   * tokens, z_num, s and the parameter gradients keep their per-sample
   * (B, ...) layouts. Served by the tensor-core engine (FS_MAX_SPLITS samples
   * at most a call); other problems return FS_ERR_UNSUPPORTED. The reference
   * plans this in ROADMAP.md:66-68 ("Ragged batching"). */
  const int64_t* row_splits;
} fs_problem;

#define FS_MAX_SPLITS 128

/* Engine selection. FS_ENGINE_AUTO runs the tensor-core kernels where they
 * serve the problem (single-tile family with fp32 or bf16 points, D = DV = 32
 * and G = 32 or 64, TMA-friendly strides; the blocked family for bf16 points
 * in the bf16 dot mode with D = 32, DV = 32 or 64, G a multiple of 128) and
 * the exact-fp32 FMA kernels elsewhere; FS_ENGINE_FMA forces the FMA kernels
 * (every product an fp32 FMA). Both meet the ieee contract. */
#define FS_ENGINE_AUTO 0
#define FS_ENGINE_FMA 1

#define FS_FLAG_STATS_IN 1  /* stats_in is given (non-NULL)   */
#define FS_FLAG_STATS_OUT 2 /* stats_out is given (non-NULL)  */

typedef struct fs_tensor4 {
  void* data;
  int64_t stride[4]; /* element strides along (b, n, h, width) */
} fs_tensor4;

/* Library ABI version (FS_ABI_VERSION). */
FS_API int fs_version(void);

/* Description of the last failure on the calling thread ("" if none). */
FS_API const char* fs_last_error(void);

/* Number of kernels this library has launched in this process (all
 * devices and threads); a diagnostic for benchmarks, no reference
 * counterpart. */
FS_API uint64_t fs_launch_count(void);

/* Of those, the tensor-core (tcgen05) kernels. Diagnostic, no reference
 * counterpart. */
FS_API uint64_t fs_tc_launch_count(void);

/* The current device's status word: 0, or 1 when a bounded device-side wait
 * of a tensor-core kernel (on a TMA load or an MMA completion) gave up after
 * 2 s since the last reset; the kernel then finished without the data it was
 * waiting for, so its outputs are not valid. Synchronises the device; clears
 * the word when reset != 0. A diagnostic of this library, no reference
 * counterpart. */
FS_API int fs_device_status(int reset);

/* Self-test of the bounded-wait path: launches on `stream` one kernel whose
 * single wait (on an mbarrier nothing arrives at) gives up after limit_ns
 * (at most 2e9) and sets the status word to 1, as a kernel's timed-out wait
 * does; the kernel then returns and the context stays usable. No reference
 * counterpart. */
FS_API int fs_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* How long one device-side wait of the tensor-core kernels launched from now
 * on may take, in ns (at most 2e9); 0 restores the default 2e9. A short
 * limit makes real kernels' waits run out on a healthy GPU: the status word
 * is set, every later wait of a thread whose wait gave up returns at once,
 * the issuing thread stops issuing and lets what it issued land, and the
 * kernel returns (its outputs not valid). For tests of that path; a
 * diagnostic of this library, no reference counterpart. */
FS_API int fs_set_wait_limit_ns(uint64_t limit_ns);

/* Bytes of workspace `op` needs for problem `p` (0 when it needs none). */
FS_API size_t fs_workspace_bytes(int op, const fs_problem* p);

/* Slice forward: z_num (B,H,G,DV), s (B,H,G). Blocked family: stats_in may
 * be NULL (then the statistics are formed first) and stats_out, when not
 * NULL, receives the statistics used (the reference's third output). */
FS_API int fs_slice_fwd(const fs_problem* p, const fs_tensor4* x_mid,
                 const fs_tensor4* fx_mid, const float* weight,
                 const float* bias, const float* tau, const float* stats_in,
                 float* stats_out, float* z_num, float* s, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Deslice forward: out (B,N,H,DV) in act_dtype. Blocked family without
 * stats_in: the online kernel forms out and the statistics in one pass
 * (stats_mode 0) and writes them to stats_out. */
FS_API int fs_deslice_fwd(const fs_problem* p, const fs_tensor4* x_mid,
                   const float* weight, const float* bias, const float* tau,
                   const float* tokens, const float* stats_in, float* stats_out,
                   const fs_tensor4* out, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Slice backward for upstream dz_num (B,H,G,DV) and ds (B,H,G):
 * dx_mid, dfx_mid (act_dtype, strided), dW, db (parameter shapes), dtau (H).
 * Blocked family: stats_in is required. */
FS_API int fs_slice_bwd(const fs_problem* p, const fs_tensor4* x_mid,
                 const fs_tensor4* fx_mid, const float* weight,
                 const float* bias, const float* tau, const float* stats_in,
                 const float* dz_num, const float* ds, const fs_tensor4* dx_mid,
                 const fs_tensor4* dfx_mid, float* dW, float* db, float* dtau,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Deslice backward for upstream d_out (B,N,H,DV): dx_mid, dtokens
 * (B,H,G,DV), dW, db, dtau. Blocked family: stats_in is required. */
FS_API int fs_deslice_bwd(const fs_problem* p, const fs_tensor4* x_mid,
                   const float* weight, const float* bias, const float* tau,
                   const float* tokens, const float* stats_in,
                   const fs_tensor4* d_out, const fs_tensor4* dx_mid,
                   float* dtokens, float* dW, float* db, float* dtau,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Slice forward without any device allocation by the caller or the library:
 * the same values as fs_slice_fwd to fp32 rounding (it always runs the
 * exact-fp32 FMA slice forward, where fs_slice_fwd may run the tensor-core
 * kernel, so the two may differ in the last bits), with the per-CTA partial
 * sums kept in a fixed scratch array inside this library instead of a
 * caller workspace.
 * No counterpart in the reference. For callers that cannot allocate device
 * memory -- a host that owns and pre-plans all device memory (an engine
 * plugin, an FFI caller with no device allocator at hand) or a code path
 * where a cudaMalloc, which may synchronise the device, is not acceptable.
 *
 *  - Serves the single-tile family only: family FS_FAMILY_SINGLE, G <= 32,
 *    D and DV <= 64, flags 0 (no statistics). Problems whose partial sums
 *    need more than FS_NOALLOC_SCRATCH_BYTES are rejected with
 *    FS_ERR_UNSUPPORTED; use fs_slice_fwd with a workspace for those.
 *  - The scratch (FS_NOALLOC_SCRATCH_BYTES) is a static device array: every
 *    GPU that loads this library holds it until the process exits.
 *  - Every call looks up the array's device address in the calling
 *    thread's current context (cudaGetSymbolAddress: a host-side query, no
 *    allocation); the scratch is per context. The first call in a context
 *    loads the library's device code into it, so make that first call
 *    before any stream capture. No call allocates or frees device memory.
 *  - All calls share the one scratch array: calls that overlap on the GPU
 *    (different streams, or different host threads on one device) race and
 *    give wrong results. Serialise them. Every partial the kernel reads is
 *    written by the same call first, so nothing needs clearing between calls.
 */
#define FS_NOALLOC_SCRATCH_BYTES (8u << 20)
FS_API int fs_slice_fwd_noalloc(const fs_problem* p, const fs_tensor4* x_mid,
                                const fs_tensor4* fx_mid, const float* weight,
                                const float* bias, const float* tau, float* z_num,
                                float* s, void* stream);

/* Backward of a coupling round -- z_num, s = slice(x_mid, fx_mid); tokens =
 * any function of z_num / (s + eps); out = deslice(x_mid, tokens) -- for
 * both ops at once, given the upstream d_out of the deslice and dz_num, ds
 * of the slice (from the tokens' gradient, which the caller forms with
 * fs_slice_fwd(x_mid, d_out): dtokens = sum_n w^T d_out). Writes dx_mid and
 * dfx_mid (the totals over both ops, so no second dx is summed) and dW, db,
 * dtau (the totals). The reference runs the two backward ops separately
 * (slice_ops.py:822-885) and autograd adds their dx; the results agree to
 * rounding. Serves only what fs_coupled_supported accepts (otherwise
 * FS_ERR_UNSUPPORTED); the workspace is fs_workspace_bytes(FS_OP_SLICE_BWD).
 * No reference counterpart as one call. */
FS_API int fs_coupled_bwd(const fs_problem* p, const fs_tensor4* x_mid,
                          const fs_tensor4* fx_mid, const fs_tensor4* d_out,
                          const float* weight, const float* bias, const float* tau,
                          const float* tokens, const float* dz_num, const float* ds,
                          const fs_tensor4* dx_mid, const fs_tensor4* dfx_mid, float* dW,
                          float* db, float* dtau, void* workspace, size_t workspace_bytes,
                          void* stream);

/* 1 when fs_coupled_bwd serves problem p: single-tile family, fp32 or bf16
 * points, D = DV = 32, G = 32 or 64, engine auto, no statistics flags; 0
 * otherwise. */
FS_API int fs_coupled_supported(const fs_problem* p);

/* Per-point softmax statistics (B,H,2,N) of the slice logits, in
 * stats_mode's form (online or two-pass). */
FS_API int fs_compute_stats(const fs_problem* p, const fs_tensor4* x_mid,
                     const float* weight, const float* bias, const float* tau,
                     float* stats, void* stream);

/* out[e] = sum over r = 0 .. world-1, in that order, of parts[r * n + e]:
 * the rank-order sum of a (world, n) fp32 buffer gathered from the ranks of a
 * process group, one launch on `stream`. Replaces the per-rank Python adds
 * of the multi-GPU wrapper (the reference plans the sharded coupling in
 * ROADMAP.md:69-73 and has no kernel for it). */
FS_API int fs_rank_sum(const float* parts, float* out, int world, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHSLICE_B200_H */
