// flashslice_b200 -- tensor-core (tcgen05) kernels of the single-tile family
// for the hot shape: fp32 point tensors, D = DV = G = 32.
//
// Every product is formed on the tensor cores from an exact three-way bf16
// split of each fp32 operand, x = hi + mid + lo (8 + 8 + 8 significant bits):
// all nine partial products are formed, each exact in the fp32 accumulator,
// so the result differs from an exact-arithmetic dot only by the
// accumulation's rounding. The parts are stacked so that one MMA forms
// several partial products at once:
//  * "wide" products (M = the 128 points of a tile): the small operand's
//    parts are stacked along N ([B_hi | B_mid | B_lo], N = 96) and the three
//    parts of the point operand are accumulated into them one after the
//    other (lo, mid, hi: the tensor core truncates when it adds to its
//    accumulator, so the small terms go first); the three column groups are
//    added in registers.
//  * "pool" products (sums over the tile's points, M = slots): the slot
//    operand's parts are stacked along M ([A_lo; A_mid; A_hi; 0], M = 128)
//    and the point operand's along N ([B_lo | B_mid | B_hi (| 1)], N = 96 or
//    112 with a ones column for the plain sums s and db): one MMA per 16
//    points; each warp reads one A part's 32 slots and adds its column
//    groups, and the per-tile pool is drained into fp32 registers with
//    round-to-nearest adds before the next tile.
//
// One CTA = one warpgroup (128 threads); thread t owns point row t of a
// 128-point tile and TMEM lane t. Tiles arrive by TMA (128B swizzle) one tile
// ahead; one thread issues the MMAs and commits them to an mbarrier.
//
// Operand layouts (no swizzle, core matrices of 8 rows x 16 bytes):
//  * per-point rows are written split into "stacked" buffers: for every group
//    of 8 points, the lo, mid and hi parts of the 32 values (64 bytes each,
//    4 core matrices) at +0, +512, +1024, and in 2048-byte groups a fourth
//    block at +1536 that holds zeros (pool A) or a ones column (pool B). The
//    same bytes serve as a K-major A operand (M = points, K = 32) and as an
//    MN-major operand over points (K = points, M or N = 32 per part).
//  * small operands (W, tokens, dz_num and their transposes, 32 x 32) are
//    split into one K-major N = 96 buffer: rows 0-31 hi, 32-63 mid, 64-95 lo.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>

#include "fs_launch.h"
#include "fs_tc.cuh"
#include "fs_tc_launch.h"

namespace fs {
namespace tcx {

using namespace fs::tc;

constexpr int kTile = 128;
constexpr int kRS3 = 1536;    // stacked buffer, 8-row group stride, three parts
constexpr int kRS4 = 2048;    // stacked buffer with a fourth (zero or ones) block
constexpr uint32_t kIdWide = idesc_bf16(128, 96, 0, 0);    // M = points, N = 3 B parts
constexpr uint32_t kIdPool = idesc_bf16(128, 96, 1, 1);    // M = 4 A parts, N = 3 B parts
constexpr uint32_t kIdPool1 = idesc_bf16(128, 112, 1, 1);  // ... plus the ones column

// ------------------------------------------------------------ row helpers
// This thread's row of a 128 x 32 fp32 tile loaded by TMA with 128B swizzle.
__device__ __forceinline__ void read_row(const uint8_t* tile, int t, float (&v)[32]) {
  const uint8_t* row = tile + t * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4 q = *(const float4*)(row + ((c ^ (t & 7)) << 4));
    v[4 * c] = q.x;
    v[4 * c + 1] = q.y;
    v[4 * c + 2] = q.z;
    v[4 * c + 3] = q.w;
  }
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}

// Split row t's 32 values into bf16 lo / mid / hi and store them in a stacked
// buffer with 8-row group stride rs.
__device__ __forceinline__ void put_row_split(uint8_t* buf, int rs, int t, const float (&v)[32]) {
  uint8_t* base = buf + (t >> 3) * rs + (t & 7) * 16;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t hw[4], mw[4], lw[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float a = v[8 * j + 2 * q], c = v[8 * j + 2 * q + 1];
      const __nv_bfloat162 h2 = __floats2bfloat162_rn(a, c);
      const float ra = a - __low2float(h2), rc = c - __high2float(h2);
      const __nv_bfloat162 m2 = __floats2bfloat162_rn(ra, rc);
      const __nv_bfloat162 l2 =
          __floats2bfloat162_rn(ra - __low2float(m2), rc - __high2float(m2));
      hw[q] = bf2_bits(h2);
      mw[q] = bf2_bits(m2);
      lw[q] = bf2_bits(l2);
    }
    *(uint4*)(base + 1024 + j * 128) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *(uint4*)(base + 512 + j * 128) = make_uint4(mw[0], mw[1], mw[2], mw[3]);
    *(uint4*)(base + j * 128) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

// A 32 x 32 fp32 matrix M (row-major, row stride 32) split into the N = 96
// K-major small operand at dst: operand row n + 32 * part (part 0 hi, 1 mid,
// 2 lo), column k, is M[n][k], or M[k][n] when transposed.
__device__ __forceinline__ void put_small_split(uint8_t* dst, const float* M, bool transposed) {
  for (int i = threadIdx.x; i < 32 * 32; i += 128) {
    const int n = i >> 5, k = i & 31;
    const float v = transposed ? M[k * 32 + n] : M[n * 32 + k];
    __nv_bfloat16 h, m, l;
    split3(v, h, m, l);
    *(__nv_bfloat16*)(dst + kmajor_off(n, k, 32)) = h;
    *(__nv_bfloat16*)(dst + kmajor_off(n + 32, k, 32)) = m;
    *(__nv_bfloat16*)(dst + kmajor_off(n + 64, k, 32)) = l;
  }
}

// The fourth block of a 2048-stride stacked buffer: zeros (pool A), or the
// ones column of a pool B (MN-group 12: column 96 = 1, 97-111 = 0).
__device__ __forceinline__ void init_fourth_block(uint8_t* buf, bool ones) {
  for (int i = threadIdx.x; i < 16 * 128; i += 128) {
    const int grp = i >> 7, w = i & 127;  // 128 words of 4 bytes per 8-row group
    uint32_t v = 0u;
    if (ones && w < 32 && (w & 3) == 0) v = 0x3F80u;  // element 0 of each 16-byte row
    *(uint32_t*)(buf + grp * kRS4 + 1536 + w * 4) = v;
  }
}

// ------------------------------------------------------------ MMA schedules
// D (128 x 96) = sum over the point operand's parts (lo, mid, hi) of
// A_part (points x 32) * [B_hi | B_mid | B_lo]^T; two K steps of 16 each.
// ad / bd: descriptors of the A buffer (K-major, SBO = its group stride) and
// of the small B buffer at their bases.
__device__ __forceinline__ void mma_wide(uint32_t d, uint64_t ad, uint64_t bd) {
#pragma unroll
  for (int q = 0; q < 3; ++q)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_bf16(d, ad + ((q * 512 + ks * 256) >> 4), bd + ((ks * 256) >> 4), kIdWide, q | ks);
}

// D (128 x N) = pool over the tile's 128 points: A = [lo; mid; hi; 0] slot
// parts (MN-major, M = 128), B = point parts (MN-major, N = 96 or 112);
// eight K steps of 16 points.
__device__ __forceinline__ void mma_pool(uint32_t d, uint64_t ad, uint64_t bd, int rsb,
                                         uint32_t idesc) {
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
    mma_bf16(d, ad + ((ks * 2 * kRS4) >> 4), bd + ((ks * 2 * rsb) >> 4), idesc, ks > 0);
}

// TMEM loads without their wait (issue several, then tmem_wait once)
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld1_nw(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The three column groups of a 96-wide result row, added small first:
// (group 2 + group 1) + group 0, with the groups in [B_hi | B_mid | B_lo]
// order for wide products.
__device__ __forceinline__ void ld_wide(uint32_t taddr, float (&v)[32]) {
  uint32_t a[32], b[32];
  tmem_ld32_nw(taddr + 64, a);
  tmem_ld32_nw(taddr + 32, b);
  tmem_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(a[i]) + __uint_as_float(b[i]);
  tmem_ld32_nw(taddr, a);
  tmem_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(a[i]);
}

// Add this lane's pool row (column groups [B_lo | B_mid | B_hi], lo first)
// into acc; with ones, also column 96 into acc1.
__device__ __forceinline__ void ld_pool(uint32_t taddr, float (&acc)[32], bool ones,
                                        float* acc1) {
  uint32_t a[32], b[32];
  tmem_ld32_nw(taddr, a);
  tmem_ld32_nw(taddr + 32, b);
  tmem_wait();
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(a[i]) + __uint_as_float(b[i]);
  tmem_ld32_nw(taddr + 64, a);
  uint32_t s = 0u;
  if (ones) tmem_ld1_nw(taddr + 96, s);
  tmem_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] += v[i] + __uint_as_float(a[i]);
  if (ones) *acc1 += __uint_as_float(s);
}

// all threads' shared writes visible to the tensor core, TMEM reads done
__device__ __forceinline__ void to_async_barrier() {
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

__device__ __forceinline__ void wait_mma(uint64_t* bar, uint32_t& phase, int* status) {
  mbar_wait(bar, phase, status);
  phase ^= 1;
  tc_fence_after();
}

// logits -> softmax weights in place (rows past N get zero weights); keeps
// logit - rowmax in lgc when given
__device__ __forceinline__ void softmax_row(float (&lg)[32], const float* bias, float inv_tau,
                                            bool valid, float* lgc) {
  float m = -INFINITY;
#pragma unroll
  for (int g = 0; g < 32; ++g) {
    lg[g] = (lg[g] + bias[g]) * inv_tau;
    m = fmaxf(m, lg[g]);
  }
  float tmp[32];
#pragma unroll
  for (int g = 0; g < 32; ++g) {
    const float c = lg[g] - m;
    if (lgc) lgc[g] = c;
    lg[g] = exp2f(c * kLog2e);
    tmp[g] = lg[g];
  }
  const float r = valid ? __frcp_rn(tree_sum(tmp)) : 0.f;
#pragma unroll
  for (int g = 0; g < 32; ++g) lg[g] *= r;
}

// softmax Jacobian of one row: dl = w (dw - sum w dw); returns
// sum_g dl (logit - m) (centred: sum_g dl = 0 exactly, so this is
// sum_g dl * logit, without a common offset multiplying the rounding residue
// of sum_g dl) and leaves dl / tau in dw
__device__ __forceinline__ float jacobian_row(const float (&w)[32], float (&dw)[32],
                                              const float (&lgc)[32], float inv_tau) {
  float tmp[32];
#pragma unroll
  for (int g = 0; g < 32; ++g) tmp[g] = w[g] * dw[g];
  const float gs = tree_sum(tmp);
#pragma unroll
  for (int g = 0; g < 32; ++g) {
    const float dl = w[g] * (dw[g] - gs);
    tmp[g] = dl * lgc[g];
    dw[g] = dl * inv_tau;
  }
  return tree_sum(tmp);
}

__device__ __forceinline__ void store_row(float* base, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *(float4*)(base + 4 * c) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// The TMA 128B-swizzle destinations need 1024-byte alignment. The dynamic
// shared window of a CTA is only 16-byte aligned when several CTAs share an
// SM, so every kernel asks for kSmemPad bytes more and aligns its base here.
constexpr int kSmemPad = 1024;
__device__ __forceinline__ uint8_t* align_smem(uint8_t* raw) {
  const uint32_t a = smem_u32(raw);
  return raw + (((a + 1023u) & ~1023u) - a);
}

// Pool partials: warp w (A part lo, mid, hi for w = 0, 1, 2) holds slot
// `lane`'s sums; add the parts small first through xch and write the 32 x n
// partial (n = 32, or 1 for a scalar per slot).
__device__ __forceinline__ void pool_write(float* xch, const float* acc, int n, float* part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (warp < 3)
    for (int i = 0; i < n; ++i) xch[(warp * 32 + lane) * 33 + i] = acc[i];
  __syncthreads();
  if (warp == 0)
    for (int i = 0; i < n; ++i)
      part[lane * n + i] =
          (xch[lane * 33 + i] + xch[(32 + lane) * 33 + i]) + xch[(64 + lane) * 33 + i];
}

__device__ __forceinline__ float cta_sum128(float v, float* red) {
  __syncthreads();
  red[threadIdx.x] = v;
  __syncthreads();
#pragma unroll
  for (int s = 64; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  return red[0];
}

// Kernel prologue shared by all four kernels: TMEM, barriers, bias.
struct Ctl {
  uint64_t* bar_tma;
  uint64_t* bar_mma;
  uint32_t tmem;
  uint32_t ph_tma, ph_mma;
};

template <int NCOLS>
__device__ __forceinline__ Ctl prologue_begin(uint8_t* sm, int bar_off) {
  Ctl c;
  c.bar_tma = (uint64_t*)(sm + bar_off);
  c.bar_mma = c.bar_tma + 1;
  uint32_t* tslot = (uint32_t*)(c.bar_tma + 2);
  if ((threadIdx.x >> 5) == 0) {
    tmem_alloc(tslot, NCOLS);
    // Give up the right to allocate again: until a CTA does, the SM admits
    // no other CTA that allocates (measured: without it, CTAs of these
    // kernels run one at a time per SM).
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    mbar_init(c.bar_tma, 1);
    mbar_init(c.bar_mma, 1);
    fence_barrier_init();
  }
  c.ph_tma = c.ph_mma = 0;
  c.tmem = 0;
  return c;
}

__device__ __forceinline__ void prologue_end(Ctl& c) {
  to_async_barrier();
  c.tmem = *(const uint32_t*)(c.bar_tma + 2);
}

template <int NCOLS>
__device__ __forceinline__ void epilogue(Ctl& c) {
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) tmem_dealloc(c.tmem, NCOLS);
}

// issue the TMA loads of one tile (one or two point tensors) on bar_tma
__device__ __forceinline__ void tma_tile(const TcParams& p, uint8_t* st0, uint8_t* st1, int h,
                                         int tile, int b, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, st1 ? 2 * 16384 : 16384);
  tma_load_4d(st0, &p.mx, 0, h, tile * kTile, b, bar);
  if (st1) tma_load_4d(st1, &p.mv, 0, h, tile * kTile, b, bar);
}

// Prefetch the tile after `tile` into the staging buffers. Called by one
// thread after a barrier that every thread reached only after its reads of
// the staging rows were consumed (their values stored into the split
// buffers) and after a proxy fence: a barrier alone does not order
// generic-proxy shared loads still in flight before the TMA's async-proxy
// writes, and with two CTAs per SM such loads were seen returning the next
// tile's bytes.
__device__ __forceinline__ void prefetch(const TcParams& p, uint8_t* st0, uint8_t* st1, int h,
                                         int tile, int b, uint64_t* bar) {
  if (tile + p.P < p.ntiles) tma_tile(p, st0, st1, h, tile + p.P, b, bar);
}

// ------------------------------------------------------------ slice forward
// smem: [stage x 16K][stage fx 16K][X split / w pool-A 32K][FX pool-B 32K]
//       [W small 6K][bias 128B][barriers]
constexpr int kSfStageX = 0, kSfStageF = 16384, kSfX = 32768, kSfF = 65536, kSfWs = 98304,
              kSfBias = 104448, kSfBar = 104576, kSfBytes = 104576 + 64;

__global__ void __launch_bounds__(128, 1) k_tc_slice_fwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  Ctl c = prologue_begin<256>(sm, kSfBar);
  float* bias_s = (float*)(sm + kSfBias);
  put_small_split(sm + kSfWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh, false);
  if (t < 32) bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
  init_fourth_block(sm + kSfX, false);  // w pool A: zeros
  init_fourth_block(sm + kSfF, true);   // fx pool B: ones column (s)
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tP = c.tmem + 128, lane_off = (uint32_t)(warp * 32) << 16;
  const uint64_t dX = smem_desc(smem_u32(sm + kSfX), 128, kRS4);      // K-major A
  const uint64_t dWs = smem_desc(smem_u32(sm + kSfWs), 128, 512);     // small B
  const uint64_t dWp = smem_desc(smem_u32(sm + kSfX), kRS4, 128);     // pool A (w)
  const uint64_t dFp = smem_desc(smem_u32(sm + kSfF), kRS4, 128);     // pool B (fx)
  float accz[32], accs = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) accz[i] = 0.f;
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) tma_tile(p, sm + kSfStageX, sm + kSfStageF, h, tile, b, c.bar_tma);
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    mbar_wait(c.bar_tma, c.ph_tma, p.status);
    c.ph_tma ^= 1;
    {
      float x[32], f[32];
      read_row(sm + kSfStageX, t, x);
      read_row(sm + kSfStageF, t, f);
      put_row_split(sm + kSfX, kRS4, t, x);
      put_row_split(sm + kSfF, kRS4, t, f);
    }
    to_async_barrier();
    if (t == 0) {
      prefetch(p, sm + kSfStageX, sm + kSfStageF, h, tile, b, c.bar_tma);
      mma_wide(tL, dX, dWs);
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float lg[32];
      ld_wide(tL + lane_off, lg);
      softmax_row(lg, bias_s, inv_tau, n0 + t < p.N, nullptr);
      put_row_split(sm + kSfX, kRS4, t, lg);  // w, over the consumed X split
    }
    to_async_barrier();
    if (t == 0) {
      mma_pool(tP, dWp, dFp, kRS4, kIdPool1);
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    if (warp < 3) ld_pool(tP + lane_off, accz, true, &accs);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kSfF);
  tc_fence_before();
  pool_write(xch, accz, 32, p.partA + slot * 32 * 32);
  pool_write(xch, &accs, 1, p.partS + slot * 32);
  epilogue<256>(c);
}

// ------------------------------------------------------------ deslice forward
// smem: [stage x 16K][X split / w split 24K][W small 6K][tok^T small 6K][bias][barriers]
constexpr int kDfStageX = 0, kDfX = 16384, kDfWs = 40960, kDfTs = 47104, kDfBias = 53248,
              kDfBar = 53376, kDfBytes = 53376 + 64;

__global__ void __launch_bounds__(128, 1) k_tc_deslice_fwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  Ctl c = prologue_begin<128>(sm, kDfBar);
  float* bias_s = (float*)(sm + kDfBias);
  put_small_split(sm + kDfWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh, false);
  put_small_split(sm + kDfTs, p.M + (int64_t)bh * 32 * 32, true);
  if (t < 32) bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, lane_off = (uint32_t)(warp * 32) << 16;
  const uint64_t dX = smem_desc(smem_u32(sm + kDfX), 128, kRS3);
  const uint64_t dWs = smem_desc(smem_u32(sm + kDfWs), 128, 512);
  const uint64_t dTs = smem_desc(smem_u32(sm + kDfTs), 128, 512);
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) tma_tile(p, sm + kDfStageX, nullptr, h, tile, b, c.bar_tma);
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    mbar_wait(c.bar_tma, c.ph_tma, p.status);
    c.ph_tma ^= 1;
    {
      float x[32];
      read_row(sm + kDfStageX, t, x);
      put_row_split(sm + kDfX, kRS3, t, x);
    }
    to_async_barrier();
    if (t == 0) {
      prefetch(p, sm + kDfStageX, nullptr, h, tile, b, c.bar_tma);
      mma_wide(tL, dX, dWs);
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float lg[32];
      ld_wide(tL + lane_off, lg);
      softmax_row(lg, bias_s, inv_tau, true, nullptr);
      put_row_split(sm + kDfX, kRS3, t, lg);
    }
    to_async_barrier();
    if (t == 0) {
      mma_wide(tL, dX, dTs);  // out = w tokens, over the consumed logits
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    float o[32];
    ld_wide(tL + lane_off, o);
    if (n0 + t < p.N)
      store_row(p.out + (int64_t)b * p.so[0] + (int64_t)(n0 + t) * p.so[1] + (int64_t)h * p.so[2],
                o);
  }
  epilogue<128>(c);
}

// ------------------------------------------------------------ deslice backward
// smem: [stage x 16K][stage dout 16K][X 32K (RS4, ones)][DO 24K (RS3)]
// [WP 32K (RS4, zeros)][UP 32K (RS4, zeros)][W 6K][tok 6K][W^T 6K][bias][red][bars]
constexpr int kDbStageX = 0, kDbStageO = 16384, kDbX = 32768, kDbO = 65536, kDbWp = 90112,
              kDbUp = 122880, kDbWs = 155648, kDbTs = 161792, kDbWt = 167936,
              kDbBias = 174080, kDbRed = 174208, kDbBar = 174720, kDbBytes = 174720 + 64;

__global__ void __launch_bounds__(128, 1) k_tc_deslice_bwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  Ctl c = prologue_begin<512>(sm, kDbBar);
  float* bias_s = (float*)(sm + kDbBias);
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;
  put_small_split(sm + kDbWs, Wb, false);                             // logits: W
  put_small_split(sm + kDbTs, p.M + (int64_t)bh * 32 * 32, false);    // dw: tok
  put_small_split(sm + kDbWt, Wb, true);                              // dx: W^T
  if (t < 32) bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
  init_fourth_block(sm + kDbX, true);
  init_fourth_block(sm + kDbWp, false);
  init_fourth_block(sm + kDbUp, false);
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  // TMEM: logits / dx at 0, dw / dtok-pool at 128, dW-pool at 256
  const uint32_t tA = c.tmem, tB = c.tmem + 128, tC = c.tmem + 256;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint64_t dXa = smem_desc(smem_u32(sm + kDbX), 128, kRS4);
  const uint64_t dOa = smem_desc(smem_u32(sm + kDbO), 128, kRS3);
  const uint64_t dUa = smem_desc(smem_u32(sm + kDbUp), 128, kRS4);
  const uint64_t dWs = smem_desc(smem_u32(sm + kDbWs), 128, 512);
  const uint64_t dTs = smem_desc(smem_u32(sm + kDbTs), 128, 512);
  const uint64_t dWt = smem_desc(smem_u32(sm + kDbWt), 128, 512);
  const uint64_t dWpP = smem_desc(smem_u32(sm + kDbWp), kRS4, 128);
  const uint64_t dUpP = smem_desc(smem_u32(sm + kDbUp), kRS4, 128);
  const uint64_t dOb = smem_desc(smem_u32(sm + kDbO), kRS3, 128);
  const uint64_t dXb = smem_desc(smem_u32(sm + kDbX), kRS4, 128);
  float acct[32], accw[32], accb = 0.f, dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) acct[i] = accw[i] = 0.f;
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) tma_tile(p, sm + kDbStageX, sm + kDbStageO, h, tile, b, c.bar_tma);
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + t < p.N;
    mbar_wait(c.bar_tma, c.ph_tma, p.status);
    c.ph_tma ^= 1;
    {
      float x[32], o[32];
      read_row(sm + kDbStageX, t, x);
      read_row(sm + kDbStageO, t, o);
      put_row_split(sm + kDbX, kRS4, t, x);
      put_row_split(sm + kDbO, kRS3, t, o);
    }
    to_async_barrier();
    if (t == 0) {
      prefetch(p, sm + kDbStageX, sm + kDbStageO, h, tile, b, c.bar_tma);
      mma_wide(tA, dXa, dWs);  // logits = x W^T
      mma_wide(tB, dOa, dTs);  // dw = d_out tok^T
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float w[32], lgc[32], dw[32];
      ld_wide(tA + lane_off, w);
      softmax_row(w, bias_s, inv_tau, valid, lgc);
      ld_wide(tB + lane_off, dw);
      const float rdt = jacobian_row(w, dw, lgc, inv_tau);
      if (valid) dt_acc += rdt;
      put_row_split(sm + kDbWp, kRS4, t, w);
      put_row_split(sm + kDbUp, kRS4, t, dw);  // dl / tau
    }
    to_async_barrier();
    if (t == 0) {
      mma_wide(tA, dUa, dWt);                      // dx = (dl/tau) W
      mma_pool(tB, dWpP, dOb, kRS3, kIdPool);      // dtokens += w^T d_out
      mma_pool(tC, dUpP, dXb, kRS4, kIdPool1);     // dW += (dl/tau)^T x, db
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float v[32];
      ld_wide(tA + lane_off, v);
      if (valid)
        store_row(p.out + (int64_t)b * p.so[0] + (int64_t)(n0 + t) * p.so[1] +
                      (int64_t)h * p.so[2],
                  v);
    }
    if (warp < 3) {
      ld_pool(tB + lane_off, acct, false, nullptr);
      ld_pool(tC + lane_off, accw, true, &accb);
    }
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kDbX);
  tc_fence_before();
  pool_write(xch, acct, 32, p.partB + slot * 32 * 32);
  pool_write(xch, accw, 32, p.partA + slot * 32 * 32);
  pool_write(xch, &accb, 1, p.partS + slot * 32);
  const float tot = cta_sum128(dt_acc, (float*)(sm + kDbRed));
  if (t == 0) p.partDt[slot] = -inv_tau * tot;
  epilogue<512>(c);
}

// ------------------------------------------------------------ slice backward
// smem: [stage x 16K][stage fx 16K][X 32K (RS4, ones)][F / w 24K (RS3)]
// [UP 32K (RS4, zeros)][W 6K][dzn 6K][dzn^T 6K][W^T 6K][bias][ds][red][bars]
constexpr int kSbStageX = 0, kSbStageF = 16384, kSbX = 32768, kSbF = 65536, kSbUp = 90112,
              kSbWs = 122880, kSbZs = 129024, kSbZt = 135168, kSbWt = 141312,
              kSbBias = 147456, kSbDs = 147584, kSbRed = 147712, kSbBar = 148224,
              kSbBytes = 148224 + 64;

__global__ void __launch_bounds__(128, 1) k_tc_slice_bwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int t = threadIdx.x, warp = t >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  Ctl c = prologue_begin<512>(sm, kSbBar);
  float* bias_s = (float*)(sm + kSbBias);
  float* ds_s = (float*)(sm + kSbDs);
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;
  const float* dzb = p.M + (int64_t)bh * 32 * 32;
  put_small_split(sm + kSbWs, Wb, false);   // logits: W
  put_small_split(sm + kSbZs, dzb, false);  // dw: dz_num
  put_small_split(sm + kSbZt, dzb, true);   // dfx: dz_num^T
  put_small_split(sm + kSbWt, Wb, true);    // dx: W^T
  if (t < 32) {
    bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
    ds_s[t] = p.ds[(int64_t)bh * 32 + t];
  }
  init_fourth_block(sm + kSbX, true);
  init_fourth_block(sm + kSbUp, false);
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  // TMEM: logits / dfx at 0, dw / dx at 128, dW-pool at 256
  const uint32_t tA = c.tmem, tB = c.tmem + 128, tC = c.tmem + 256;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint64_t dXa = smem_desc(smem_u32(sm + kSbX), 128, kRS4);
  const uint64_t dFa = smem_desc(smem_u32(sm + kSbF), 128, kRS3);
  const uint64_t dUa = smem_desc(smem_u32(sm + kSbUp), 128, kRS4);
  const uint64_t dWs = smem_desc(smem_u32(sm + kSbWs), 128, 512);
  const uint64_t dZs = smem_desc(smem_u32(sm + kSbZs), 128, 512);
  const uint64_t dZt = smem_desc(smem_u32(sm + kSbZt), 128, 512);
  const uint64_t dWt = smem_desc(smem_u32(sm + kSbWt), 128, 512);
  const uint64_t dUpP = smem_desc(smem_u32(sm + kSbUp), kRS4, 128);
  const uint64_t dXb = smem_desc(smem_u32(sm + kSbX), kRS4, 128);
  float accw[32], accb = 0.f, dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) accw[i] = 0.f;
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) tma_tile(p, sm + kSbStageX, sm + kSbStageF, h, tile, b, c.bar_tma);
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + t < p.N;
    mbar_wait(c.bar_tma, c.ph_tma, p.status);
    c.ph_tma ^= 1;
    {
      float x[32], f[32];
      read_row(sm + kSbStageX, t, x);
      read_row(sm + kSbStageF, t, f);
      put_row_split(sm + kSbX, kRS4, t, x);
      put_row_split(sm + kSbF, kRS3, t, f);
    }
    to_async_barrier();
    if (t == 0) {
      prefetch(p, sm + kSbStageX, sm + kSbStageF, h, tile, b, c.bar_tma);
      mma_wide(tA, dXa, dWs);  // logits = x W^T
      mma_wide(tB, dFa, dZs);  // dw = fx dz_num^T
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float w[32], lgc[32], dw[32];
      ld_wide(tA + lane_off, w);
      softmax_row(w, bias_s, inv_tau, valid, lgc);
      ld_wide(tB + lane_off, dw);
#pragma unroll
      for (int g = 0; g < 32; ++g) dw[g] += ds_s[g];
      const float rdt = jacobian_row(w, dw, lgc, inv_tau);
      if (valid) dt_acc += rdt;
      put_row_split(sm + kSbF, kRS3, t, w);    // over the consumed fx split
      put_row_split(sm + kSbUp, kRS4, t, dw);  // dl / tau
    }
    to_async_barrier();
    if (t == 0) {
      mma_wide(tA, dFa, dZt);                   // dfx = w dz_num
      mma_wide(tB, dUa, dWt);                   // dx = (dl/tau) W
      mma_pool(tC, dUpP, dXb, kRS4, kIdPool1);  // dW += (dl/tau)^T x, db
      mma_commit(c.bar_mma);
    }
    wait_mma(c.bar_mma, c.ph_mma, p.status);
    {
      float v[32];
      ld_wide(tA + lane_off, v);
      if (valid)
        store_row(p.out2 + (int64_t)b * p.so2[0] + (int64_t)(n0 + t) * p.so2[1] +
                      (int64_t)h * p.so2[2],
                  v);
      ld_wide(tB + lane_off, v);
      if (valid)
        store_row(p.out + (int64_t)b * p.so[0] + (int64_t)(n0 + t) * p.so[1] +
                      (int64_t)h * p.so[2],
                  v);
    }
    if (warp < 3) ld_pool(tC + lane_off, accw, true, &accb);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kSbX);
  tc_fence_before();
  pool_write(xch, accw, 32, p.partA + slot * 32 * 32);
  pool_write(xch, &accb, 1, p.partS + slot * 32);
  const float tot = cta_sum128(dt_acc, (float*)(sm + kSbRed));
  if (t == 0) p.partDt[slot] = -inv_tau * tot;
  epilogue<512>(c);
}

// ------------------------------------------------------------ host side

static __device__ int fs_tc_status_word;

int* device_status() {
  static int* ptrs[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, fs_tc_status_word) != cudaSuccess) return nullptr;
    ptrs[dev] = (int*)p;
  }
  return ptrs[dev];
}

bool make_point_map(CUtensorMap* map, const void* data, int64_t B, int64_t N, int64_t H,
                    const int64_t stride[4]) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        !fn)
      return false;
    encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  if (stride[3] != 1 || ((uintptr_t)data & 15)) return false;
  for (int i = 0; i < 3; ++i)
    if (stride[i] <= 0 || (stride[i] * 4) % 16 || stride[i] * 4 >= ((int64_t)1 << 40))
      return false;
  // The encoder is a driver call and needs a current context on this thread;
  // a thread that has made no runtime call yet (an autograd worker on its
  // first backward op) has none until the runtime binds the device's primary
  // context, which cudaSetDevice does.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return false;
  cuuint64_t dims[4] = {32, (cuuint64_t)H, (cuuint64_t)N, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)(stride[2] * 4), (cuuint64_t)(stride[1] * 4),
                        (cuuint64_t)(stride[0] * 4)};
  cuuint32_t box[4] = {32, 1, kTile, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  // the encoder wants a 64-byte aligned map; do not rely on the caller's stack
  unsigned char raw[sizeof(CUtensorMap) + 64];
  CUtensorMap* aligned = (CUtensorMap*)(((uintptr_t)raw + 63) & ~(uintptr_t)63);
  const CUresult r = encode(aligned, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(data),
                            dims, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::memcpy(map, aligned, sizeof(CUtensorMap));
  return true;
}

// Dynamic shared memory size, and the full shared carveout: without it the
// runtime may size the L1/shared split for one CTA per SM.
static cudaError_t set_smem(const void* k, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

std::atomic<uint64_t> g_tc_launches{0};

cudaError_t run_tc(TcKind k, const TcParams& p, cudaStream_t s) {
  const dim3 grid(p.P, p.B * p.H);
  cudaError_t e = cudaSuccess;
  switch (k) {
    case TcKind::SliceFwd:
      e = set_smem((const void*)k_tc_slice_fwd, kSfBytes + kSmemPad);
      if (e != cudaSuccess) return e;
      k_tc_slice_fwd<<<grid, 128, kSfBytes + kSmemPad, s>>>(p);
      break;
    case TcKind::DesliceFwd:
      e = set_smem((const void*)k_tc_deslice_fwd, kDfBytes + kSmemPad);
      if (e != cudaSuccess) return e;
      k_tc_deslice_fwd<<<grid, 128, kDfBytes + kSmemPad, s>>>(p);
      break;
    case TcKind::SliceBwd:
      e = set_smem((const void*)k_tc_slice_bwd, kSbBytes + kSmemPad);
      if (e != cudaSuccess) return e;
      k_tc_slice_bwd<<<grid, 128, kSbBytes + kSmemPad, s>>>(p);
      break;
    case TcKind::DesliceBwd:
      e = set_smem((const void*)k_tc_deslice_bwd, kDbBytes + kSmemPad);
      if (e != cudaSuccess) return e;
      k_tc_deslice_bwd<<<grid, 128, kDbBytes + kSmemPad, s>>>(p);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

// Co-resident CTAs per SM each kernel is sized for (shared memory and TMEM):
// slice fwd 102 KB + 256 columns, deslice fwd 52 KB + 128 columns, the
// backward kernels 145 / 171 KB + all 512 columns.
int tc_ctas_per_sm(TcKind k) {
  switch (k) {
    case TcKind::SliceFwd: return 2;
    case TcKind::DesliceFwd: return 4;
    default: return 1;
  }
}

}  // namespace tcx
}  // namespace fs
