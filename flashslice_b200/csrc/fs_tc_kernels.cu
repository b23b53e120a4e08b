// flashslice_b200 -- tensor-core (tcgen05) kernels of the single-tile family
// for the hot shape: fp32 point tensors, D = DV = 32, G = 32.
//
// Every product is formed on the tensor cores from an exact three-way bf16
// split of each fp32 operand, x = hi + mid + lo (8 + 8 + 8 significant bits),
// keeping the six partial products whose weight is above 2^-24 of the full
// product (hi*hi, hi*mid, mid*hi, hi*lo, mid*mid, lo*hi); each bf16 product
// is exact in the fp32 accumulator. The tensor core truncates when it adds
// to its accumulator, so the small products are issued first and the big
// one last, and sums over points are drained every tile into fp32 registers
// with round-to-nearest adds. Measured on a B200 the split dot is closer to
// the float64 value than a sequential fp32 FMA dot (0.4 vs 0.7 median ulp).
//
// One CTA = one warpgroup (128 threads); thread t owns point row t of a
// 128-point tile and TMEM lane t. Tiles arrive by TMA (128B swizzle) one tile
// ahead; one thread issues the MMAs and commits them to an mbarrier.
//
// Operand layouts (no swizzle, core matrices of 8 rows x 16 bytes):
//  * per-point rows (x, fx, weights w, ...) are written split into "stacked"
//    buffers: for every group of 8 points, the lo, mid and hi parts of the 32
//    values (64 bytes each as 4 core matrices) at +0, +512, +1024 and, in
//    pool-A buffers, 512 zero bytes at +1536. The same bytes serve as a
//    K-major A operand (M = points, K = 32) and as an MN-major operand over
//    points (K = points, M or N = 32); three consecutive parts form the
//    M = 64 windows [lo; mid], [mid; hi], [hi; 0] of a pool's A operand.
//  * small operands (W, tokens, dz_num and their transposes, 32 x 32) are
//    split into three K-major 2 KB buffers.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "fs_launch.h"
#include "fs_tc.cuh"
#include "fs_tc_launch.h"

namespace fs {
namespace tcx {

using namespace fs::tc;

constexpr int kTile = 128;
constexpr int kRS3 = 1536;   // stacked buffer, 8-row group stride, three parts
constexpr int kRS4 = 2048;   // stacked buffer with a zero part (pool A)
constexpr int kSmall = 2048; // one part of a 32 x 32 small operand
constexpr uint32_t kIdWide = idesc_bf16(128, 32, 0, 0);  // M = points
constexpr uint32_t kIdPool = idesc_bf16(64, 32, 1, 1);   // M = 64 slot window, N = 32
constexpr uint32_t kIdPool8 = idesc_bf16(64, 8, 1, 1);   // N = 8 (ones column)

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

// A 32 x 32 fp32 matrix M (row-major, row stride ld) split into three K-major
// small operands at dst (hi, mid, lo, kSmall bytes apart); operand row n,
// column k is M[n][k], or M[k][n] when transposed.
template <int NT>
__device__ __forceinline__ void put_small_split(uint8_t* dst, const float* M, int ld,
                                                bool transposed) {
  for (int i = threadIdx.x; i < 32 * 32; i += NT) {
    const int n = i >> 5, k = i & 31;
    const float v = transposed ? M[k * ld + n] : M[n * ld + k];
    __nv_bfloat16 h, m, l;
    split3(v, h, m, l);
    const uint32_t off = kmajor_off(n, k, 32);
    *(__nv_bfloat16*)(dst + off) = h;
    *(__nv_bfloat16*)(dst + kSmall + off) = m;
    *(__nv_bfloat16*)(dst + 2 * kSmall + off) = l;
  }
}

// ------------------------------------------------------------ MMA schedules
// D (128 x 32) = A (points x 32, stacked, stride rs) * B^T (small, 32 x 32):
// the six split products, small first, two K steps of 16 each.
__device__ __forceinline__ void mma_wide(uint32_t d, uint32_t a, int rs, uint32_t b) {
  // (A part, B part) with 0 = hi, 1 = mid, 2 = lo
  const int pa[6] = {2, 1, 0, 1, 0, 0};
  const int pb[6] = {0, 1, 2, 0, 1, 0};
#pragma unroll
  for (int q = 0; q < 6; ++q)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const uint64_t ad = smem_desc(a + (2 - pa[q]) * 512 + ks * 256, 128, rs);
      const uint64_t bd = smem_desc(b + pb[q] * kSmall + ks * 256, 128, 512);
      mma_bf16(d, ad, bd, kIdWide, q | ks);
    }
}

// Pool (64 x 32 in TMEM, M = 64 layout): sum over the tile's 128 points of
// A^T B with A the stacked pool buffer (stride kRS4) and B a stacked point
// buffer (stride rsb) read as MN-major over points. Windows [lo; mid] x hi,
// [mid; hi] x mid, [hi; 0] x lo, [hi; 0] x hi: rows 0-31 of D (top) and
// 32-63 (bottom) add up to the six split products.
__device__ __forceinline__ void mma_pool(uint32_t d, uint32_t a, uint32_t b, int rsb) {
  const int win[4] = {0, 512, 1024, 1024};
  const int bp[4] = {1024, 512, 0, 1024};
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint64_t ad = smem_desc(a + win[g] + ks * 2 * kRS4, kRS4, 128);
      const uint64_t bd = smem_desc(b + bp[g] + ks * 2 * rsb, rsb, 128);
      mma_bf16(d, ad, bd, kIdPool, g | ks);
    }
}

// Column sums of the pool's A over the tile's points, against a ones column
// (N = 8, column 0 is one): windows [lo; mid] and [hi; 0].
__device__ __forceinline__ void mma_pool_ones(uint32_t d, uint32_t a, uint32_t ones) {
  const int win[2] = {0, 1024};
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint64_t ad = smem_desc(a + win[g] + ks * 2 * kRS4, kRS4, 128);
      const uint64_t bd = smem_desc(ones + ks * 256, 128, 128);
      mma_bf16(d, ad, bd, kIdPool8, g | ks);
    }
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
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

__device__ __forceinline__ float softmax_row(float (&lg)[32], const float* bias, float inv_tau,
                                             bool valid) {
#pragma unroll
  for (int g = 0; g < 32; ++g) lg[g] = (lg[g] + bias[g]) * inv_tau;
  float m = lg[0];
#pragma unroll
  for (int g = 1; g < 32; ++g) m = fmaxf(m, lg[g]);
  float tmp[32];
#pragma unroll
  for (int g = 0; g < 32; ++g) {
    lg[g] = exp2f((lg[g] - m) * kLog2e);
    tmp[g] = lg[g];
  }
  const float r = valid ? __frcp_rn(tree_sum(tmp)) : 0.f;
#pragma unroll
  for (int g = 0; g < 32; ++g) lg[g] *= r;
  return m;
}

__device__ __forceinline__ void store_row(float* base, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *(float4*)(base + 4 * c) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// ------------------------------------------------------------ slice forward
// smem: [stage x 16K][stage fx 16K][X split / w pool 32K (aliased; both with
//       the 2048-byte group stride, so X never touches the zero blocks)]
//       [FX split 24K][W small 6K][ones 2K][bias 128B][barriers]
constexpr int kSfStageX = 0, kSfStageF = 16384, kSfX = 32768, kSfW = 32768, kSfF = 65536,
              kSfWs = 90112, kSfOnes = 96256, kSfBias = 98304, kSfBar = 98432,
              kSfBytes = 98432 + 64;

// The TMA 128B-swizzle destinations need 1024-byte alignment; the dynamic
// shared window is checked instead of assumed.
__device__ __forceinline__ bool smem_misaligned(const uint8_t* sm, int* status) {
  if (smem_u32(sm) & 1023) {
    if (threadIdx.x == 0) atomicExch(status, 2);
    return true;
  }
  return false;
}

__global__ void __launch_bounds__(128, 1) k_tc_slice_fwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  if (smem_misaligned(sm, p.status)) return;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  uint64_t* bar_tma = (uint64_t*)(sm + kSfBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tslot = (uint32_t*)(bar_tma + 2);
  float* bias_s = (float*)(sm + kSfBias);
  if (warp == 0) tmem_alloc(tslot, 128);
  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_barrier_init();
  }
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;
  put_small_split<128>(sm + kSfWs, Wb, 32, false);
  if (t < 32) bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
  // zero part of the pool buffer and the ones column
  for (int i = t; i < 16 * 128; i += 128)
    *(uint32_t*)(sm + kSfW + (i >> 7) * kRS4 + 1536 + (i & 127) * 4) = 0u;
  for (int i = t; i < 512; i += 128) {
    // ones: MN-major, N = 8, K = points; column 0 of point k at (k>>3)*128 + (k&7)*16
    const int k = i >> 2, w = i & 3;
    *(uint32_t*)(sm + kSfOnes + (k >> 3) * 128 + (k & 7) * 16 + w * 4) = w == 0 ? 0x3F80u : 0u;
  }
  const float inv_tau = __frcp_rn(p.tau[h]);
  to_async_barrier();
  const uint32_t tb = *tslot;
  const uint32_t tL = tb, tZ = tb + 32, tS = tb + 64, lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t aX = smem_u32(sm + kSfX), aF = smem_u32(sm + kSfF), aW = smem_u32(sm + kSfW);
  const uint32_t aWs = smem_u32(sm + kSfWs), aOnes = smem_u32(sm + kSfOnes);
  uint32_t ph_tma = 0, ph_mma = 0;
  float accz[32], accs = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) accz[i] = 0.f;
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) {
    mbar_arrive_expect_tx(bar_tma, 2 * 16384);
    tma_load_4d(sm + kSfStageX, &p.mx, 0, h, tile * kTile, b, bar_tma);
    tma_load_4d(sm + kSfStageF, &p.mv, 0, h, tile * kTile, b, bar_tma);
  }
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    mbar_wait(bar_tma, ph_tma, p.status);
    ph_tma ^= 1;
    float x[32], f[32];
    read_row(sm + kSfStageX, t, x);
    read_row(sm + kSfStageF, t, f);
    __syncthreads();  // staging consumed: prefetch the next tile into it
    if (t == 0 && tile + p.P < p.ntiles) {
      mbar_arrive_expect_tx(bar_tma, 2 * 16384);
      tma_load_4d(sm + kSfStageX, &p.mx, 0, h, (tile + p.P) * kTile, b, bar_tma);
      tma_load_4d(sm + kSfStageF, &p.mv, 0, h, (tile + p.P) * kTile, b, bar_tma);
    }
    put_row_split(sm + kSfX, kRS4, t, x);
    put_row_split(sm + kSfF, kRS3, t, f);
    to_async_barrier();
    if (t == 0) {
      mma_wide(tL, aX, kRS4, aWs);
      mma_commit(bar_mma);
    }
    wait_mma(bar_mma, ph_mma, p.status);
    float lg[32];
    tmem_ld32(tL + lane_off, lg);
    softmax_row(lg, bias_s, inv_tau, n0 + t < p.N);
    put_row_split(sm + kSfW, kRS4, t, lg);  // over the consumed X split
    to_async_barrier();
    if (t == 0) {
      mma_pool(tZ, aW, aF, kRS3);
      mma_pool_ones(tS, aW, aOnes);
      mma_commit(bar_mma);
    }
    wait_mma(bar_mma, ph_mma, p.status);
    float z[32], s8[8];
    tmem_ld32(tZ + lane_off, z);
    tmem_ld8(tS + lane_off, s8);
#pragma unroll
    for (int i = 0; i < 32; ++i) accz[i] += z[i];
    accs += s8[0];
  }
  // rows of the pool live in lanes 0-15 of each warp: warps 0, 1 hold slots
  // 0-31 of the top half, warps 2, 3 the bottom half; add the halves
  float* xch = (float*)(sm + kSfF);  // 32 x 33 floats, the FX split is free now
  tc_fence_before();
  __syncthreads();
  if (warp >= 2 && lane < 16) {
    const int g = (warp - 2) * 16 + lane;
#pragma unroll
    for (int i = 0; i < 32; ++i) xch[g * 33 + i] = accz[i];
    xch[g * 33 + 32] = accs;
  }
  __syncthreads();
  if (warp < 2 && lane < 16) {
    const int g = warp * 16 + lane;
    const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
    float* pz = p.partA + (slot * 32 + g) * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) pz[i] = accz[i] + xch[g * 33 + i];
    p.partS[slot * 32 + g] = accs + xch[g * 33 + 32];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 128);
}

// ------------------------------------------------------------ deslice forward
// smem: [stage x 16K][X split / w split 24K][W small 6K][tok^T small 6K][bias][barriers]
constexpr int kDfStageX = 0, kDfX = 16384, kDfWs = 40960, kDfTs = 47104, kDfBias = 53248,
              kDfBar = 53376, kDfBytes = 53376 + 64;

__global__ void __launch_bounds__(128, 1) k_tc_deslice_fwd(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t sm[];
  if (smem_misaligned(sm, p.status)) return;
  const int t = threadIdx.x, warp = t >> 5;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  uint64_t* bar_tma = (uint64_t*)(sm + kDfBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tslot = (uint32_t*)(bar_tma + 2);
  float* bias_s = (float*)(sm + kDfBias);
  if (warp == 0) tmem_alloc(tslot, 64);
  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_barrier_init();
  }
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;
  put_small_split<128>(sm + kDfWs, Wb, 32, false);
  put_small_split<128>(sm + kDfTs, p.M + (int64_t)bh * 32 * 32, 32, true);
  if (t < 32) bias_s[t] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + t];
  const float inv_tau = __frcp_rn(p.tau[h]);
  to_async_barrier();
  const uint32_t tb = *tslot;
  const uint32_t tL = tb, tO = tb + 32, lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t aX = smem_u32(sm + kDfX), aWs = smem_u32(sm + kDfWs),
                 aTs = smem_u32(sm + kDfTs);
  uint32_t ph_tma = 0, ph_mma = 0;
  int tile = blockIdx.x;
  if (t == 0 && tile < p.ntiles) {
    mbar_arrive_expect_tx(bar_tma, 16384);
    tma_load_4d(sm + kDfStageX, &p.mx, 0, h, tile * kTile, b, bar_tma);
  }
  for (; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    mbar_wait(bar_tma, ph_tma, p.status);
    ph_tma ^= 1;
    float x[32];
    read_row(sm + kDfStageX, t, x);
    __syncthreads();
    if (t == 0 && tile + p.P < p.ntiles) {
      mbar_arrive_expect_tx(bar_tma, 16384);
      tma_load_4d(sm + kDfStageX, &p.mx, 0, h, (tile + p.P) * kTile, b, bar_tma);
    }
    put_row_split(sm + kDfX, kRS3, t, x);
    to_async_barrier();
    if (t == 0) {
      mma_wide(tL, aX, kRS3, aWs);
      mma_commit(bar_mma);
    }
    wait_mma(bar_mma, ph_mma, p.status);
    float lg[32];
    tmem_ld32(tL + lane_off, lg);
    softmax_row(lg, bias_s, inv_tau, true);
    put_row_split(sm + kDfX, kRS3, t, lg);
    to_async_barrier();
    if (t == 0) {
      mma_wide(tO, aX, kRS3, aTs);
      mma_commit(bar_mma);
    }
    wait_mma(bar_mma, ph_mma, p.status);
    float o[32];
    tmem_ld32(tO + lane_off, o);
    if (n0 + t < p.N)
      store_row(p.out + (int64_t)b * p.so[0] + (int64_t)(n0 + t) * p.so[1] + (int64_t)h * p.so[2],
                o);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 64);
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
  cuuint64_t dims[4] = {32, (cuuint64_t)H, (cuuint64_t)N, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)(stride[2] * 4), (cuuint64_t)(stride[1] * 4),
                        (cuuint64_t)(stride[0] * 4)};
  cuuint32_t box[4] = {32, 1, kTile, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(data),
                            dims, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static cudaError_t set_smem(const void* k, int bytes) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

cudaError_t run_tc(TcKind k, const TcParams& p, cudaStream_t s) {
  const dim3 grid(p.P, p.B * p.H);
  cudaError_t e = cudaSuccess;
  switch (k) {
    case TcKind::SliceFwd:
      e = set_smem((const void*)k_tc_slice_fwd, kSfBytes);
      if (e != cudaSuccess) return e;
      k_tc_slice_fwd<<<grid, 128, kSfBytes, s>>>(p);
      break;
    case TcKind::DesliceFwd:
      e = set_smem((const void*)k_tc_deslice_fwd, kDfBytes);
      if (e != cudaSuccess) return e;
      k_tc_deslice_fwd<<<grid, 128, kDfBytes, s>>>(p);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

std::atomic<uint64_t> g_tc_launches{0};

int tc_ctas_per_sm(TcKind k) {
  switch (k) {
    case TcKind::SliceFwd: return 2;
    case TcKind::DesliceFwd: return 4;
    default: return 1;
  }
}

}  // namespace tcx
}  // namespace fs
