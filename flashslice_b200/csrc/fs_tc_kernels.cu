// flashslice_b200 -- tensor-core (tcgen05) kernels of the single-tile family
// for the hot shape: D = DV = 32, G = 32 (and the G = 64 round further down),
// fp32 or bf16 point tensors (the kernels are templated on the point type; a
// bf16 value is its own exact hi part), and of the blocked family's bf16
// shapes.
//
// Every product is formed on the tensor cores from an exact three-way bf16
// split of each fp32 operand, x = hi + mid + lo (8 + 8 + 8 significant bits);
// each partial product is exact in the fp32 accumulator, so the result
// differs from an exact-arithmetic dot only by the accumulation's rounding.
// The tensor core truncates when it adds to its accumulator, so small terms
// go first everywhere.
//
// An MMA instruction (M = 128, K = 16) costs about 47 cycles whether N is 32
// or 96 (measured on this part: N = 32 47, N = 96 48-57, N = 256 127), so the
// schedules minimise instructions:
//  * "wide" products (M = the 128 points of a tile, K = 32): with NW = 96 the
//    small operand's parts are stacked along N ([B_lo | B_mid | B_hi]) and the
//    point operand's parts lo, mid, hi accumulated one after the other (six
//    MMAs, all nine partial products); the three column groups are added in
//    registers. Where TMEM is short, NW = 64 accumulates [x B_mid | x B_hi]
//    (eight MMAs: A hi times B_lo goes into the B_mid group) and NW = 32 the
//    six partial products above the fp32 rounding level (lo*lo, lo*mid and
//    mid*lo are below 2^-26 of the result) in one 32-column accumulator
//    (twelve MMAs). The point operand is read from TMEM, where each thread
//    writes its own row: a tensor-core read of shared memory runs at about
//    128 bytes per clock.
//  * "pool" products (sums over the tile's points, M = slots): the slot
//    operand's parts are stacked along M ([A_lo; A_mid; A_hi; unused], M =
//    128) and the point operand's along N ([B_lo | B_mid | B_hi], N = 96):
//    one MMA per 16 points gives all nine part products; the threads of TMEM
//    lanes 0-95 add the three column groups of their A part, and the per-tile
//    pool is drained into fp32 registers with round-to-nearest adds before
//    the next tile. Plain sums (s, db) are added up by the threads that own
//    the rows.
//
// Threads: T threads share each of the 128 point rows of a tile (T = 2 or 4;
// 128 * T threads per CTA). Warp w serves TMEM lanes 32 (w % 4) .. +31 and
// the columns [C (w / 4), C (w / 4) + C) of every 32-column result, C = 32 /
// T; row maxima and sums are combined across the T threads of a row through
// shared memory. Row arithmetic uses the paired fp32 instructions (two
// values per instruction). Tiles arrive by TMA (128B swizzle) one tile
// ahead; one thread issues the MMAs and commits them to an mbarrier.
//
// Operand layouts (no swizzle, core matrices of 8 rows x 16 bytes):
//  * "stacked" buffers: for every group of 8 rows, the lo, mid and hi parts
//    of the 32 values (64 bytes each, 4 core matrices) at +0, +512, +1024
//    (group stride 1536). Point rows stored so serve as an N-stacked MN-major
//    B operand over points and as an M-stacked MN-major A operand over points;
//    the latter reads 512 bytes past each group (the next group's lo part, and
//    a tail after the buffer) into TMEM lanes 96-127, which nothing reads. A
//    small matrix stored so (rows r) is the N-stacked MN-major operand of its
//    transpose.
//  * a point operand in TMEM holds, in its thread's lane, the lo, mid and hi
//    parts at columns +0, +16, +32 (two bf16 per column, even k low).
//  * "small" operands (W, tokens, dz_num; 32 x 32, row-major M[r][c]) split
//    into three K-major parts (rows r, k = c) at +0 (lo), +2048 (mid), +4096
//    (hi): one N = 96 K-major operand ([B_lo | B_mid | B_hi]), or three
//    N = 32 ones, and each part is also the MN-major operand of the transpose
//    (K = r, N = c).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <type_traits>
#include <cstring>

#include "fs_launch.h"
#include "fs_tc.cuh"
#include "fs_tc_launch.h"

namespace fs {
namespace tcx {

using namespace fs::tc;

constexpr int kTile = 128;
constexpr int kRS = 1536;               // stacked buffer: 8-row group stride
constexpr int kSplit = 16 * kRS;        // one 128-point tile split (24 KB)
constexpr int kTail = 512;              // read past an M-stacked operand (ignored)
constexpr int kSmall = 3 * 2048;        // one 32 x 32 matrix, three parts
constexpr int kSmallStk = 4 * kRS;      // one 32 x 32 matrix, stacked
constexpr int kStage = kTile * 128;     // one fp32 TMA tile (16 KB)
constexpr float kLn2 = 0.6931471805599453f;

constexpr uint32_t kIdPool = idesc_bf16(128, 96, 1, 1);  // M = 4 A parts, N = 3 B parts

// the six partial products of a 32-wide product, small first: (A part, B
// part) with parts 0 = lo, 1 = mid, 2 = hi
__host__ __device__ constexpr int part_a(int i) { return i == 0 ? 0 : i == 1 ? 2 : i < 4 ? 1 : 2; }
__host__ __device__ constexpr int part_b(int i) {
  return i == 0 ? 2 : i == 1 ? 0 : i == 2 ? 1 : i == 3 ? 2 : i == 4 ? 1 : 2;
}

// ------------------------------------------------------------ threads
template <int T>
struct Th {
  static constexpr int NT = 128 * T;  // threads per CTA
  static constexpr int C = 32 / T;    // columns per thread
  int row, cs, q;
  uint32_t lane_off;
  __device__ __forceinline__ Th() {
    const int w = threadIdx.x >> 5;
    q = w & 3;
    cs = w >> 2;
    row = 32 * q + (threadIdx.x & 31);
    lane_off = (uint32_t)(32 * q) << 16;
  }
};

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 2^x with the hardware's base-2 exponential (ex2.approx, subnormal results
// flushed to zero): the softmax only needs it for x <= 0, where a flushed
// result is a weight below 2^-126 of the row's largest.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------ paired fp32
__device__ __forceinline__ float2 f2(const float* v, int k) { return make_float2(v[2 * k], v[2 * k + 1]); }
__device__ __forceinline__ void put2(float* v, int k, float2 x) {
  v[2 * k] = x.x;
  v[2 * k + 1] = x.y;
}

// sum of N values (N even) by pairs, fixed order
template <int N>
__device__ __forceinline__ float tree_sum2(const float (&v)[N]) {
  float2 p[N / 2];
#pragma unroll
  for (int k = 0; k < N / 2; ++k) p[k] = f2(v, k);
#pragma unroll
  for (int s = N / 4; s > 0; s >>= 1) {
#pragma unroll
    for (int i = 0; i < s; ++i) p[i] = __fadd2_rn(p[i], p[i + s]);
  }
  return p[0].x + p[0].y;
}

// ------------------------------------------------------------ TMEM I/O
template <int N>
__device__ __forceinline__ void tld(uint32_t a, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tld<8>(uint32_t a, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(a));
}
template <>
__device__ __forceinline__ void tld<16>(uint32_t a, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(a));
}
template <>
__device__ __forceinline__ void tld<32>(uint32_t a, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(a));
}
__device__ __forceinline__ void tld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tst(uint32_t a, const uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tst<4>(uint32_t a, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
template <>
__device__ __forceinline__ void tst<8>(uint32_t a, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(a),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
template <>
__device__ __forceinline__ void tst<16>(uint32_t a, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(a),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tst_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// This thread's C columns of a wide result at taddr (lane included): one
// 32-column accumulator (NW = 32), or the sum of the column groups of an
// N-stacked one, added small first (NW = 64: groups x B_mid, x B_hi; NW = 96:
// x B_lo, x B_mid, x B_hi).
template <int NW, int C>
__device__ __forceinline__ void ld_wide(uint32_t taddr, int cs, float (&v)[C]) {
  if constexpr (NW == 32) {
    uint32_t r[C];
    tld<C>(taddr + cs * C, r);
    tld_wait();
#pragma unroll
    for (int i = 0; i < C; ++i) v[i] = __uint_as_float(r[i]);
  } else if constexpr (NW == 64) {
    uint32_t a[C], b[C];
    tld<C>(taddr + cs * C, a);
    tld<C>(taddr + 32 + cs * C, b);
    tld_wait();
#pragma unroll
    for (int k = 0; k < C / 2; ++k)
      put2(v, k, __fadd2_rn(make_float2(__uint_as_float(a[2 * k]), __uint_as_float(a[2 * k + 1])),
                            make_float2(__uint_as_float(b[2 * k]), __uint_as_float(b[2 * k + 1]))));
  } else {
    uint32_t a[C], b[C], c[C];
    tld<C>(taddr + cs * C, a);
    tld<C>(taddr + 32 + cs * C, b);
    tld<C>(taddr + 64 + cs * C, c);
    tld_wait();
#pragma unroll
    for (int k = 0; k < C / 2; ++k) {
      const float2 s = __fadd2_rn(make_float2(__uint_as_float(a[2 * k]), __uint_as_float(a[2 * k + 1])),
                                  make_float2(__uint_as_float(b[2 * k]), __uint_as_float(b[2 * k + 1])));
      put2(v, k, __fadd2_rn(s, make_float2(__uint_as_float(c[2 * k]), __uint_as_float(c[2 * k + 1]))));
    }
  }
}

// ------------------------------------------------------------ row helpers
// This thread's C columns of row `row` of a 128 x 32 fp32 tile loaded by TMA
// with 128B swizzle (16-byte chunk j of row r sits at chunk j ^ (r % 8)).
template <int C>
__device__ __forceinline__ void read_cols(const uint8_t* tile, int row, int cs, float (&v)[C]) {
  const uint8_t* r = tile + row * 128;
#pragma unroll
  for (int i = 0; i < C / 4; ++i) {
    const int j = cs * (C / 4) + i;
    const float4 f = *(const float4*)(r + ((j ^ (row & 7)) << 4));
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}

// (a, c) -> packed bf16 pairs of their hi, mid and lo parts (a in the low
// half); the residuals are exact, so a = hi + mid + lo exactly
__device__ __forceinline__ void split_pair(float2 v, uint32_t& hw, uint32_t& mw, uint32_t& lw) {
  const float2 neg1 = make_float2(-1.f, -1.f);
  const __nv_bfloat162 h2 = __float22bfloat162_rn(v);
  const float2 r = __ffma2_rn(__bfloat1622float2(h2), neg1, v);
  const __nv_bfloat162 m2 = __float22bfloat162_rn(r);
  const float2 r2 = __ffma2_rn(__bfloat1622float2(m2), neg1, r);
  hw = bf2_bits(h2);
  mw = bf2_bits(m2);
  lw = bf2_bits(__float22bfloat162_rn(r2));
}

// A row's C values split into packed bf16 pairs of their lo, mid and hi parts
// (formed once, stored wherever the row serves as an operand).
template <int C>
struct Split {
  uint32_t hw[C / 2], mw[C / 2], lw[C / 2];
  __device__ __forceinline__ explicit Split(const float (&v)[C]) {
#pragma unroll
    for (int k = 0; k < C / 2; ++k) split_pair(f2(v, k), hw[k], mw[k], lw[k]);
  }
  // values that are bf16 already: they are their own hi part, mid = lo = 0
  __device__ __forceinline__ explicit Split(const uint32_t (&bf16_pairs)[C / 2]) {
#pragma unroll
    for (int k = 0; k < C / 2; ++k) {
      hw[k] = bf16_pairs[k];
      mw[k] = lw[k] = 0u;
    }
  }
  // into a stacked buffer as row `row`, columns [C cs, C cs + C)
  __device__ __forceinline__ void to_smem(uint8_t* buf, int row, int cs) const {
    uint8_t* base = buf + (row >> 3) * kRS + (row & 7) * 16;
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      const int j = cs * (C / 8) + i;
      *(uint4*)(base + 1024 + j * 128) =
          make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
      *(uint4*)(base + 512 + j * 128) =
          make_uint4(mw[4 * i], mw[4 * i + 1], mw[4 * i + 2], mw[4 * i + 3]);
      *(uint4*)(base + j * 128) = make_uint4(lw[4 * i], lw[4 * i + 1], lw[4 * i + 2], lw[4 * i + 3]);
    }
  }
  // into the TMEM point operand at taddr (lane included): parts lo, mid, hi
  // at +0, +16, +32 columns. The caller waits (tst_wait) before the MMA is
  // issued.
  __device__ __forceinline__ void to_tmem(uint32_t taddr, int cs) const {
    const uint32_t a = taddr + cs * (C / 2);
    tst<C / 2>(a, lw);
    tst<C / 2>(a + 16, mw);
    tst<C / 2>(a + 32, hw);
  }
};

// This thread's C columns of one row of a point tile staged by TMA, in the
// tile's type: fp32 (128-byte rows, 128B swizzle: chunk j at j ^ (r % 8)),
// split three ways, or bf16 (64-byte rows, 64B swizzle: chunk j at
// j ^ ((r / 2) % 4)), exact as its own hi part. Read into registers first
// (load), split where the caller consumes them.
template <int C, typename PT>
struct RowVals;
template <int C>
struct RowVals<C, float> {
  float v[C];
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int cs) {
    read_cols<C>(tile, row, cs, v);
  }
  __device__ __forceinline__ Split<C> split() const { return Split<C>(v); }
};
template <int C>
struct RowVals<C, __nv_bfloat16> {
  uint32_t w[C / 2];
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int cs) {
    const uint8_t* r = tile + row * 64;
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      const int j = cs * (C / 8) + i;
      const uint4 q = *(const uint4*)(r + ((j ^ ((row >> 1) & 3)) << 4));
      w[4 * i] = q.x;
      w[4 * i + 1] = q.y;
      w[4 * i + 2] = q.z;
      w[4 * i + 3] = q.w;
    }
  }
  __device__ __forceinline__ Split<C> split() const { return Split<C>(w); }
};

// bytes of one staged point tile of type PT (128 points x 32 values)
template <typename PT>
__host__ __device__ constexpr int stage_bytes() {
  return kTile * 32 * (int)sizeof(PT);
}

// point tensors of type PT have only a hi part (bf16: each value is its own
// hi part, mid and lo are zero), so the MMAs of their other parts are skipped
template <typename PT>
constexpr bool kHi = std::is_same<PT, __nv_bfloat16>::value;

// two result values of a row stored in the point tensor's type
__device__ __forceinline__ void store2(float* p, float2 v) { *(float2*)p = v; }
__device__ __forceinline__ void store2(__nv_bfloat16* p, float2 v) {
  *(__nv_bfloat162*)p = __float22bfloat162_rn(v);
}


// A 32 x 32 fp32 matrix M (row-major) split into the three-part small
// operand at dst: part p (0 lo, 1 mid, 2 hi) at +2048 p, K-major with rows r
// and k = c.
template <int NT>
__device__ __forceinline__ void put_small(uint8_t* dst, const float* M) {
  for (int i = threadIdx.x; i < 32 * 32; i += NT) {
    const int r = i >> 5, c = i & 31;
    __nv_bfloat16 h, m, l;
    split3(M[i], h, m, l);
    const uint32_t o = kmajor_off(r, c, 32);
    *(__nv_bfloat16*)(dst + o) = l;
    *(__nv_bfloat16*)(dst + 2048 + o) = m;
    *(__nv_bfloat16*)(dst + 4096 + o) = h;
  }
}

// The same matrix as a stacked buffer over its rows r (the N-stacked MN-major
// operand of its transpose: K = r, N = part * 32 + c).
template <int NT>
__device__ __forceinline__ void put_small_stacked(uint8_t* dst, const float* M) {
  for (int i = threadIdx.x; i < 32 * 32; i += NT) {
    const int r = i >> 5, c = i & 31;
    __nv_bfloat16 h, m, l;
    split3(M[i], h, m, l);
    const uint32_t o = (r >> 3) * kRS + (r & 7) * 16 + (c >> 3) * 128 + (c & 7) * 2;
    *(__nv_bfloat16*)(dst + o) = l;
    *(__nv_bfloat16*)(dst + 512 + o) = m;
    *(__nv_bfloat16*)(dst + 1024 + o) = h;
  }
}

// A result tile written to a point tensor with whole 32-byte sectors: this
// warp's 32 rows (lanes 32 q ..) and C columns (from cs C) are read back from
// TMEM in the 16x256b shape, in which thread t holds rows 16 half + t / 4 and
// 16 half + 8 + t / 4 and columns 2 (t % 4), +1 of each 8-column chunk, so
// four threads store 32 contiguous bytes of a row. (Stored straight from the
// 32x32b shape, each thread's row is a different point, 1 KB or more apart,
// and every store instruction half-fills 32 sectors.) The result is one
// 32-column accumulator (NW = 32) or an N-stacked one whose column groups
// are added small first (NW = 64, 96). Rows at or past `nvalid` are not
// written.
template <int NW, int C, typename PT>
__device__ __forceinline__ void store_result(uint32_t tcol, int q, int cs, PT* row0,
                                             int64_t row_stride, int nvalid) {
  const int t = threadIdx.x & 31;
  constexpr int J = C / 8;
  constexpr int NG = NW / 32;
  uint32_t r[2][J][NG][4];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf)
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int g = 0; g < NG; ++g) {
        const uint32_t a =
            tcol + ((uint32_t)(32 * q + 16 * hf) << 16) + cs * C + 8 * j + 32 * g;
        asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(r[hf][j][g][0]), "=r"(r[hf][j][g][1]), "=r"(r[hf][j][g][2]),
                       "=r"(r[hf][j][g][3])
                     : "r"(a));
      }
  tld_wait();
#pragma unroll
  for (int hf = 0; hf < 2; ++hf)
#pragma unroll
    for (int sub = 0; sub < 2; ++sub) {
      const int row = 32 * q + 16 * hf + 8 * sub + (t >> 2);
      if (row < nvalid) {
        PT* rp = row0 + (int64_t)row * row_stride + cs * C + 2 * (t & 3);
#pragma unroll
        for (int j = 0; j < J; ++j) {
          float2 v = make_float2(__uint_as_float(r[hf][j][0][2 * sub]),
                                 __uint_as_float(r[hf][j][0][2 * sub + 1]));
#pragma unroll
          for (int g = 1; g < NG; ++g)
            v = __fadd2_rn(v, make_float2(__uint_as_float(r[hf][j][g][2 * sub]),
                                          __uint_as_float(r[hf][j][g][2 * sub + 1])));
          store2(rp + 8 * j, v);
        }
      }
    }
}

// ------------------------------------------------------------ MMA schedules
// Descriptors: a stacked buffer as M-stacked / N-stacked MN-major operand;
// a small operand in its K-major or (per part) MN-major view.
__device__ __forceinline__ uint64_t desc_stacked(const void* p) {
  return smem_desc(smem_u32(p), kRS, 128);
}
__device__ __forceinline__ uint64_t desc_smallK(const void* p) {
  return smem_desc(smem_u32(p), 128, 512);
}
__device__ __forceinline__ uint64_t desc_smallM(const void* p) {
  return smem_desc(smem_u32(p), 512, 128);
}

// A from TMEM (K-major by construction): D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                       bool accumulate) {
  const uint32_t acc = accumulate ? 1u : 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// The NW = 64 schedule (below) of D = A1 B1^T, or with S = 2 of
// D = A1 B1^T + A2 B2^T into one accumulator, the two products' partial
// products interleaved so that the small ones still go first.
//
// AHI: the point operands have only a hi part (bf16 points: their lo and mid
// parts are zero), so only their hi-part MMAs run: hi x [B_mid | B_hi] first
// (it sets all 64 columns), then hi x B_lo into the B_mid group.
template <bool MN, int S, bool AHI = false>
__device__ __forceinline__ void wide_ts64_pair(uint32_t d, uint32_t a1, uint64_t b1, uint32_t a2,
                                               uint64_t b2) {
  constexpr uint32_t id64 = idesc_bf16(128, 64, 0, MN ? 1 : 0);
  constexpr uint32_t id32 = idesc_bf16(128, 32, 0, MN ? 1 : 0);
  constexpr int kstep = MN ? 2 * kRS : 256;  // bytes per K step of 16
  constexpr int mid = MN ? 512 : 2048;       // offset of B_mid
  const uint32_t a[2] = {a1, a2};
  const uint64_t b[2] = {b1, b2};
  if constexpr (AHI) {
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((mid + ks * kstep) >> 4), id64, (s | ks) != 0);
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((ks * kstep) >> 4), id32, true);
  } else {
#pragma unroll
    for (int pa = 0; pa < 2; ++pa)
#pragma unroll
      for (int s = 0; s < S; ++s)
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
          mma_ts(d, a[s] + pa * 16 + ks * 8, b[s] + ((mid + ks * kstep) >> 4), id64,
                 (pa | s | ks) != 0);
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((ks * kstep) >> 4), id32, true);
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((mid + ks * kstep) >> 4), id64, true);
  }
}

// Wide product D = A B^T, A = point rows in TMEM at `a` (K = 32), B = small
// operand at bd:
//  * NW = 32: twelve MMAs into one 32-column accumulator; bd is the three-part
//    small operand, read K-major (B[n][k] = M[n][k]) or, MN, MN-major per
//    part (B[n][k] = M[k][n]);
//  * NW = 64: eight MMAs into a 64-column accumulator [x B_mid | x B_hi]:
//    A lo and mid times [B_mid | B_hi], A hi times B_lo (into the B_mid
//    group: the same outputs), A hi times [B_mid | B_hi] -- seven of the
//    nine partial products, all above the fp32 rounding level; bd as for
//    NW = 96 (both layouts hold B_mid and B_hi next to each other along N,
//    so [B_mid | B_hi] is one N = 64 operand);
//  * NW = 96: six MMAs into a 96-column N-stacked accumulator; bd is the
//    three-part small operand read K-major (B[n][k] = M[n][k]) or, MN, the
//    stacked copy of M (B[n][k] = M[k][n]).
// An MMA with N <= 96 takes about as long as one with N = 32, so NW = 96
// and NW = 64 cost half and two thirds of NW = 32.
// AHI: the point operand has only a hi part (bf16 points), so only its
// hi-part MMAs run.
template <int NW, bool MN, bool AHI = false>
__device__ __forceinline__ void wide_ts(uint32_t d, uint32_t a, uint64_t bd) {
  if constexpr (NW == 64) {
    wide_ts64_pair<MN, 1, AHI>(d, a, bd, a, bd);
  } else if constexpr (NW == 32) {
    constexpr uint32_t id = idesc_bf16(128, 32, 0, MN ? 1 : 0);
    bool first = true;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      if (AHI && part_a(i) != 2) continue;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        mma_ts(d, a + part_a(i) * 16 + ks * 8,
               bd + ((part_b(i) * 2048 + ks * (MN ? 1024 : 256)) >> 4), id, !first);
        first = false;
      }
    }
  } else {
    constexpr uint32_t id = idesc_bf16(128, 96, 0, MN ? 1 : 0);
    constexpr int pa0 = AHI ? 2 : 0;
#pragma unroll
    for (int pa = pa0; pa < 3; ++pa)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a + pa * 16 + ks * 8, bd + ((ks * (MN ? 2 * kRS : 256)) >> 4), id,
               (pa != pa0) || ks != 0);
  }
}

// Wide product with N = 96 and the point operand in shared memory: A = point
// rows of a stacked buffer read K-major (part p at +512 p), B = the small
// operand's three parts stacked along N (K-major); six MMAs, A parts lo, mid,
// hi accumulated one after the other.
// (AHI: the point rows have only a hi part, bf16 points: only its MMAs run)
template <bool AHI = false>
__device__ __forceinline__ void wide_ss96(uint32_t d, uint64_t ad, uint64_t bd) {
  constexpr uint32_t id = idesc_bf16(128, 96, 0, 0);
  constexpr int pa0 = AHI ? 2 : 0;
#pragma unroll
  for (int pa = pa0; pa < 3; ++pa)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_bf16(d, ad + ((pa * 512 + ks * 256) >> 4), bd + ((ks * 256) >> 4), id,
               (pa != pa0) || ks != 0);
}

__device__ __forceinline__ uint64_t desc_rowsA(const void* p) {
  return smem_desc(smem_u32(p), 128, kRS);
}

// D (128 x 96) = pool over the tile's points: A = M-stacked slot parts, B =
// N-stacked point parts; eight K steps of 16 points.
__device__ __forceinline__ void mma_pool(uint32_t d, uint64_t ad, uint64_t bd) {
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
    mma_bf16(d, ad + ((ks * 2 * kRS) >> 4), bd + ((ks * 2 * kRS) >> 4), kIdPool, ks > 0);
}

// Add this thread's columns of its pool row (column groups lo, mid, hi of the
// B parts, small first) into acc. Lanes 0-95 only (A parts lo, mid, hi).
template <int C>
__device__ __forceinline__ void drain_pool(uint32_t taddr, int cs, float (&acc)[C]) {
  float v[C];
  ld_wide<96, C>(taddr, cs, v);
#pragma unroll
  for (int k = 0; k < C / 2; ++k) put2(acc, k, __fadd2_rn(f2(acc, k), f2(v, k)));
}

// ------------------------------------------------------------ sync
// all threads' shared (and TMEM) writes visible to the tensor core, TMEM
// reads done
__device__ __forceinline__ void to_async_barrier() {
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Kernel control block: the TMA barrier and up to five MMA-completion
// barriers (one per group of MMAs committed together), each completing once
// per tile, with their phases; the wait limit, and whether a wait of this
// thread has given up.
//
// After a wait gives up (status word set), every later wait of that thread
// returns at once, so a kernel whose arrivals are lost finishes after one
// limit per thread instead of one per wait; the issuing thread (thread 0)
// then issues no further TMA or MMA work -- it re-arms a barrier only after
// a completed wait on it, so each barrier has at most one phase it armed and
// did not see complete -- and before the TMEM is freed it waits, with a
// short bound, for the phase each barrier still expects, so that the copies
// and MMAs it issued are done before the CTA exits. Control flow is the same
// for every thread either way: the CTA-wide barriers all meet.
constexpr int kNumBars = 6;
constexpr uint64_t kDrainNs = 50000000ull;  // 50 ms per barrier, failure path only
struct Ctl {
  uint64_t* bar;  // [0] TMA, [1..5] MMA groups
  uint32_t tmem;
  uint32_t ph[kNumBars];
  uint32_t fail;   // a wait of this thread gave up
  uint64_t limit;  // ns a wait may take
  // the thread that issues TMA loads and MMAs, while none of its waits failed
  __device__ __forceinline__ bool issuer() const { return threadIdx.x == 0 && !fail; }
};

__device__ __forceinline__ void wait_bar(Ctl& c, int k, int* status) {
  if (!c.fail) {
    if (mbar_wait(c.bar + k, c.ph[k], status, c.limit))
      c.ph[k] ^= 1;
    else
      c.fail = 1;
  }
  tc_fence_after();
}
__device__ __forceinline__ void commit(Ctl& c, int k) { mma_commit(c.bar + k); }

// ------------------------------------------------------------ row math
// Per-head row constants in shared memory: the logit scale in log2 units
// (log2(e) / tau) and the bias on that scale.
struct RowConst {
  float scale;
  const float* bias2;  // 32 floats: bias * log2(e) / tau
};

template <int NT>
__device__ __forceinline__ RowConst row_const(float* bias_s, const float* bias, float tau) {
  const float inv_tau = __frcp_rn(tau);
  const float scale = inv_tau * kLog2e;
  if (threadIdx.x < 32) bias_s[threadIdx.x] = bias[threadIdx.x] * scale;
  return RowConst{scale, bias_s};
}

// Row statistics combined across the T threads of a row in one exchange
// (fixed order): the row maximum m of the scaled logits, s = sum 2^(l - m)
// and u = sum 2^(l - m) dw. Each thread contributes its columns' values
// relative to its own maximum; `red` holds 3 T 128 floats, not reused until
// a CTA-wide barrier.
struct RowStat {
  float m, s, u;
};
template <int T, bool U>
__device__ __forceinline__ RowStat row_stat(float ml, float sl, float ul, float* red,
                                            const Th<T>& th) {
  if constexpr (T == 1) {
    return RowStat{ml, sl, ul};
  } else {
    red[th.cs * 128 + th.row] = ml;
    red[(T + th.cs) * 128 + th.row] = sl;
    if (U) red[(2 * T + th.cs) * 128 + th.row] = ul;
    named_sync(1 + th.q, 32 * T);
    float mt[T], st[T], ut[T];
#pragma unroll
    for (int c = 0; c < T; ++c) {
      mt[c] = red[c * 128 + th.row];
      st[c] = red[(T + c) * 128 + th.row];
      ut[c] = U ? red[(2 * T + c) * 128 + th.row] : 0.f;
    }
    float m = mt[0];
#pragma unroll
    for (int c = 1; c < T; ++c) m = fmaxf(m, mt[c]);
#pragma unroll
    for (int c = 0; c < T; ++c) {
      const float f = ex2(mt[c] - m);
      st[c] *= f;
      ut[c] *= f;
    }
    return RowStat{m, tree_sum(st), U ? tree_sum(ut) : 0.f};
  }
}

// raw logits (x W^T) -> scaled logits relative to this thread's maximum:
// d = l - max, e = 2^d; returns the thread's maximum
template <int C>
__device__ __forceinline__ float row_exp(const float (&acc)[C], const RowConst& rc, int cs,
                                         float (&d)[C], float (&e)[C]) {
  const float2 sc = make_float2(rc.scale, rc.scale);
  const float2* b2 = (const float2*)(rc.bias2 + cs * C);
  float mx[C / 2];
#pragma unroll
  for (int k = 0; k < C / 2; ++k) {
    const float2 v = __ffma2_rn(f2(acc, k), sc, b2[k]);
    put2(d, k, v);
    mx[k] = fmaxf(v.x, v.y);
  }
#pragma unroll
  for (int s = C / 4; s > 0; s >>= 1)
#pragma unroll
    for (int i = 0; i < s; ++i) mx[i] = fmaxf(mx[i], mx[i + s]);
  const float m = mx[0];
  const float2 nm = make_float2(-m, -m);
#pragma unroll
  for (int k = 0; k < C / 2; ++k) {
    const float2 v = __fadd2_rn(f2(d, k), nm);
    put2(d, k, v);
    put2(e, k, make_float2(ex2(v.x), ex2(v.y)));
  }
  return m;
}

// Softmax (forward): raw logits -> weights in place (rows past N get zero
// weights). One exchange per row.
template <int T, int C>
__device__ __forceinline__ void softmax_fwd(float (&lg)[C], const RowConst& rc, bool valid,
                                            float* red, const Th<T>& th) {
  float d[C], e[C];
  const float ml = row_exp<C>(lg, rc, th.cs, d, e);
  const RowStat st = row_stat<T, false>(ml, tree_sum2(e), 0.f, red, th);
  const float f = valid ? ex2(ml - st.m) / st.s : 0.f;
  const float2 f2v = make_float2(f, f);
#pragma unroll
  for (int k = 0; k < C / 2; ++k) put2(lg, k, __fmul2_rn(f2(e, k), f2v));
}

// Softmax and its Jacobian (backward) in one exchange per row: raw logits in
// lg -> weights w; upstream dw -> dl / tau with dl = w (dw - sum w dw).
// Returns this thread's part of sum_g dl (logit - rowmax), in log2 units
// (centred: sum_g dl = 0 exactly, so this is sum_g dl * logit without a
// common offset multiplying the rounding residue of sum_g dl).
template <int T, int C>
__device__ __forceinline__ float softmax_bwd(float (&lg)[C], float (&dw)[C], const RowConst& rc,
                                             float inv_tau, bool valid, float* red,
                                             const Th<T>& th) {
  float d[C], e[C], tmp[C];
  const float ml = row_exp<C>(lg, rc, th.cs, d, e);
#pragma unroll
  for (int k = 0; k < C / 2; ++k) put2(tmp, k, __fmul2_rn(f2(e, k), f2(dw, k)));
  const RowStat st = row_stat<T, true>(ml, tree_sum2(e), tree_sum2(tmp), red, th);
  const float dm = ml - st.m;
  const float rs = __frcp_rn(st.s);
  const float f = valid ? ex2(dm) * rs : 0.f;
  const float gs = st.u * rs;
  const float2 f2v = make_float2(f, f), ng = make_float2(-gs, -gs), dm2 = make_float2(dm, dm),
               it = make_float2(inv_tau, inv_tau);
#pragma unroll
  for (int k = 0; k < C / 2; ++k) {
    const float2 w = __fmul2_rn(f2(e, k), f2v);
    put2(lg, k, w);
    const float2 dl = __fmul2_rn(w, __fadd2_rn(f2(dw, k), ng));
    put2(tmp, k, __fmul2_rn(dl, __fadd2_rn(f2(d, k), dm2)));
    put2(dw, k, __fmul2_rn(dl, it));
  }
  return tree_sum2(tmp);
}

// The TMA 128B-swizzle destinations need 1024-byte alignment. The dynamic
// shared window of a CTA is only 16-byte aligned when several CTAs share an
// SM, so every kernel asks for kSmemPad bytes more and aligns its base here.
constexpr int kSmemPad = 1024;
__device__ __forceinline__ uint8_t* align_smem(uint8_t* raw) {
  const uint32_t a = smem_u32(raw);
  return raw + (((a + 1023u) & ~1023u) - a);
}

// Pool partials: threads of lanes 0-95 (A part lo, mid, hi = lane quarter)
// hold slot `lane`'s sums over their C columns; add the parts small first
// through xch (96 x 33 floats) and write the 32 x 32 partial.
template <int T>
__device__ __forceinline__ void pool_write(float* xch, const float* acc, float* part,
                                           const Th<T>& th) {
  constexpr int C = Th<T>::C;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  if (th.q < 3) {
#pragma unroll
    for (int i = 0; i < C; ++i) xch[(th.q * 32 + lane) * 33 + th.cs * C + i] = acc[i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 32 * 32; i += Th<T>::NT) {
    const int g = i >> 5, c = i & 31;
    part[i] = (xch[g * 33 + c] + xch[(32 + g) * 33 + c]) + xch[(64 + g) * 33 + c];
  }
}

// Plain sums over the CTA's points (s, db): thread (row, cs) holds its rows'
// sums of columns [C cs, C cs + C); add them over the 128 rows in a fixed
// order through xch (128 x 33 floats) and write the 32 sums.
template <int T>
__device__ __forceinline__ void rowsum_write(float* xch, const float* acc, float* part,
                                             const Th<T>& th) {
  constexpr int C = Th<T>::C;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < C; ++i) xch[th.row * 33 + th.cs * C + i] = acc[i];
  __syncthreads();
  if (threadIdx.x < 32) {
    float s[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s[k] = 0.f;
      for (int r = k; r < 128; r += 8) s[k] += xch[r * 33 + threadIdx.x];
    }
    part[threadIdx.x] = tree_sum(s);
  }
}

template <int NT>
__device__ __forceinline__ float cta_sum_nt(float v, float* red) {
  __syncthreads();
  red[threadIdx.x] = v;
  __syncthreads();
#pragma unroll
  for (int s = NT / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  return red[0];
}

// ------------------------------------------------------------ prologue
constexpr int kBarBytes = 128;  // kNumBars mbarriers and the TMEM address slot

template <int NCOLS>
__device__ __forceinline__ Ctl prologue_begin(uint8_t* sm, int bar_off, uint64_t limit_ns) {
  Ctl c;
  c.fail = 0;
  c.limit = limit_ns ? limit_ns : kWaitNs;
  c.bar = (uint64_t*)(sm + bar_off);
  uint32_t* tslot = (uint32_t*)(c.bar + kNumBars);
  if ((threadIdx.x >> 5) == 0) {
    tmem_alloc(tslot, NCOLS);
    // Give up the right to allocate again: until a CTA does, the SM admits
    // no other CTA that allocates (measured: without it, CTAs of these
    // kernels run one at a time per SM).
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < kNumBars; ++k) mbar_init(c.bar + k, 1);
    fence_barrier_init();
  }
#pragma unroll
  for (int k = 0; k < kNumBars; ++k) c.ph[k] = 0;
  c.tmem = 0;
  return c;
}

__device__ __forceinline__ void prologue_end(Ctl& c) {
  to_async_barrier();
  c.tmem = *(const uint32_t*)(c.bar + kNumBars);
}

template <int NCOLS>
__device__ __forceinline__ void epilogue(Ctl& c) {
  if (c.issuer() && c.fail) {
    // failure path: let the copies and MMAs this thread issued land first
#pragma unroll
    for (int k = 0; k < kNumBars; ++k) mbar_wait(c.bar + k, c.ph[k], nullptr, kDrainNs);
  }
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) tmem_dealloc(c.tmem, NCOLS);
}

// The points of one b: all N rows of batch entry b, or, with row splits
// (ragged samples packed along n), rows [split[b], split[b + 1]) of the one
// batch entry. Tile t covers its rows [128 t, 128 t + 128); rows at or past N
// are masked (they may be the next sample's, or past the tensor: zeros).
struct Span {
  int64_t n0;  // first row in the tensors' n axis
  int bc;      // b coordinate in the point tensors
  int N, ntiles;
  __device__ __forceinline__ int row(int tile) const { return (int)(n0 + (int64_t)tile * kTile); }
};
__device__ __forceinline__ Span span_of(const TcParams& p, int b) {
  if (p.nsplit == 0) return Span{0, b, p.N, p.ntiles};
  const int64_t a = p.split[b], n = p.split[b + 1] - a;
  return Span{a, 0, (int)n, (int)((n + kTile - 1) / kTile)};
}

// issue the TMA loads of one tile (one or two point tensors of type PT) on bar
template <typename PT>
__device__ __forceinline__ void tma_tile(const TcParams& p, uint8_t* st0, uint8_t* st1, int h,
                                         const Span& sp, int tile, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, st1 ? 2 * stage_bytes<PT>() : stage_bytes<PT>());
  tma_load_4d(st0, &p.mx, 0, h, sp.row(tile), sp.bc, bar);
  if (st1) tma_load_4d(st1, &p.mv, 0, h, sp.row(tile), sp.bc, bar);
}

// Prefetch the tile after `tile` into the staging buffers. Called by one
// thread after a barrier that every thread reached only after its reads of
// the staging rows were consumed (their values stored into the split
// buffers or TMEM) and after a proxy fence: a barrier alone does not order
// generic-proxy shared loads still in flight before the TMA's async-proxy
// writes, and with two CTAs per SM such loads were seen returning the next
// tile's bytes.
template <typename PT>
__device__ __forceinline__ void prefetch(const TcParams& p, uint8_t* st0, uint8_t* st1, int h,
                                         const Span& sp, int tile, uint64_t* bar) {
  if (tile + p.P < sp.ntiles) tma_tile<PT>(p, st0, st1, h, sp, tile + p.P, bar);
}

// Per-kernel threads per point row, co-resident CTAs per SM (shared memory,
// TMEM and registers sized for it) and, for deslice forward, the width of its
// wide products. Each can be set at build time (-DFS_TC_SF_T=... etc.).
#ifndef FS_TC_SF_T
#define FS_TC_SF_T 2
#endif
#ifndef FS_TC_DF_T
#define FS_TC_DF_T 1
#endif
#ifndef FS_TC_DF_CTAS
#define FS_TC_DF_CTAS 4
#endif
#ifndef FS_TC_DF_NW
#define FS_TC_DF_NW 64
#endif
#ifndef FS_TC_SB_T
#define FS_TC_SB_T 2
#endif
#ifndef FS_TC_DB_T
#define FS_TC_DB_T 2
#endif
constexpr int kTSliceFwd = FS_TC_SF_T, kTDesliceFwd = FS_TC_DF_T, kTSliceBwd = FS_TC_SB_T,
              kTDesliceBwd = FS_TC_DB_T;
constexpr int kCtasSliceFwd = 2, kCtasDesliceFwd = FS_TC_DF_CTAS, kCtasSliceBwd = 2,
              kCtasDesliceBwd = 2;
constexpr int kNwDf = FS_TC_DF_NW;                 // 32, 64 or 96
constexpr int kDfCols = kNwDf == 96 ? 256 : 128;   // TMEM columns of deslice forward

// MMA-completion barrier groups
enum : int { kBarTma = 0, kG1 = 1, kG2 = 2, kG3 = 3, kG4 = 4, kG5 = 5 };

// bytes of the row-statistics exchange for T threads per row and n values
__host__ __device__ constexpr int red_bytes(int T, int n) { return T == 1 ? 0 : n * T * 512; }

// ------------------------------------------------------------ slice forward
// smem: [stage x][WS split: w][F split: fx, two tiles][W][bias][red][bars]
// Each fx tile is staged inside the F buffer its split will occupy (the
// rows are read into registers, then the split overwrites them).
// TMEM (256 columns): logits (N-stacked) at 0, z pool at 96, the x point
// operand at 192.
// The loop is skewed by one stage: while the tensor core forms tile i's pool,
// the threads split tile i+1 (into the other F buffer) and issue its logits;
// the pool is drained while those run. Tile i+2's fx is loaded into tile i's
// F buffer once tile i's pool is done with it.
// (WS needs no tail: its M-stacked reads past the end land in F.)
constexpr int kSfStageX = 0, kSfWS = kStage, kSfF = kSfWS + kSplit, kSfWs = kSfF + 2 * kSplit,
              kSfBias = kSfWs + kSmall, kSfRed = kSfBias + 128,
              kSfBar = kSfRed + red_bytes(kTSliceFwd, 2), kSfBytes = kSfBar + kBarBytes;
static_assert(kSfF % 1024 == 0 && kSplit % 1024 == 0, "fx staging tiles need 1 KB alignment");

template <typename PT>
__global__ void __launch_bounds__(128 * kTSliceFwd, kCtasSliceFwd)
    k_tc_slice_fwd(const __grid_constant__ TcParams p) {
  constexpr int T = kTSliceFwd, NT = Th<T>::NT, C = Th<T>::C;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kSfBar, p.wait_ns);
  float* red = (float*)(sm + kSfRed);
  put_small<NT>(sm + kSfWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  const RowConst rc = row_const<NT>((float*)(sm + kSfBias),
                                    p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tP = c.tmem + 96, tX = c.tmem + 192;
  const uint64_t dWs = desc_smallK(sm + kSfWs), dWp = desc_stacked(sm + kSfWS);
  uint8_t* stX = sm + kSfStageX;
  auto fbuf = [&](int i) { return sm + kSfF + i * kSplit; };
  float accz[C], accs[C];
#pragma unroll
  for (int i = 0; i < C; ++i) accz[i] = accs[i] = 0.f;
  // split one tile's rows (x into TMEM, fx from its staging in F[buf] into F[buf])
  auto split_tile = [&](int buf) {
    wait_bar(c, kBarTma, p.status);
    RowVals<C, PT> x, f;
    x.load(stX, th.row, th.cs);
    f.load(fbuf(buf), th.row, th.cs);
    __syncthreads();  // every staged fx row is in registers before F[buf] is overwritten
    x.split().to_tmem(tX + th.lane_off, th.cs);
    f.split().to_smem(fbuf(buf), th.row, th.cs);
    tst_wait();
  };
  int tile = blockIdx.x, buf = 0;
  // (a CTA of a sample with fewer tiles than CTAs has none: it writes zero
  // partials; the condition is the same for every thread)
  if (tile < sp.ntiles) {
    if (c.issuer()) tma_tile<PT>(p, stX, fbuf(0), h, sp, tile, c.bar);
    split_tile(0);
    to_async_barrier();
    if (c.issuer()) {
      prefetch<PT>(p, stX, fbuf(1), h, sp, tile, c.bar);  // F[1] is unused yet
      wide_ts<96, false, kHi<PT>>(tL, tX, dWs);  // logits = x W^T
      commit(c, kG1);
    }
  }
  for (; tile < sp.ntiles; tile += p.P, buf ^= 1) {
    const int n0 = tile * kTile;
    const bool more = tile + p.P < sp.ntiles;
    const bool more2 = tile + 2 * p.P < sp.ntiles;
    wait_bar(c, kG1, p.status);
    {
      float lg[C];
      ld_wide<96, C>(tL + th.lane_off, th.cs, lg);
      softmax_fwd<T, C>(lg, rc, n0 + th.row < sp.N, red, th);
      Split<C>(lg).to_smem(sm + kSfWS, th.row, th.cs);
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(accs, k, __fadd2_rn(f2(accs, k), f2(lg, k)));
    }
    to_async_barrier();
    if (c.issuer()) {
      mma_pool(tP, dWp, desc_stacked(fbuf(buf)));  // z += w^T fx
      commit(c, kG2);
    }
    if (more) {
      split_tile(buf ^ 1);
      to_async_barrier();
      if (c.issuer()) {
        if (more2) {  // tile i+2: its x now, its fx once tile i's pool is done with F[buf]
          mbar_arrive_expect_tx(c.bar + kBarTma, 2 * stage_bytes<PT>());
          tma_load_4d(stX, &p.mx, 0, h, sp.row(tile + 2 * p.P), sp.bc, c.bar + kBarTma);
        }
        wide_ts<96, false, kHi<PT>>(tL, tX, dWs);
        commit(c, kG1);
      }
    }
    wait_bar(c, kG2, p.status);
    if (c.issuer() && more2)
      tma_load_4d(fbuf(buf), &p.mv, 0, h, sp.row(tile + 2 * p.P), sp.bc, c.bar + kBarTma);
    if (th.q < 3) drain_pool<C>(tP + th.lane_off, th.cs, accz);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)fbuf(0);
  tc_fence_before();
  pool_write<T>(xch, accz, p.partA + slot * 32 * 32, th);
  rowsum_write<T>(xch, accs, p.partS + slot * 32, th);
  epilogue<256>(c);
}

// ------------------------------------------------------------ deslice forward
// smem: [stage x][W][tokens][bias][red][bars]
// TMEM (kDfCols columns): logits -> out at 0 (NW columns), the point operand
// (x, then w) after it.
static_assert(kSmall == kSmallStk, "tokens buffer holds either layout");
constexpr int kDfStageX = 0, kDfWs = kStage, kDfTs = kDfWs + kSmall,
              kDfBias = kDfTs + kSmall, kDfRed = kDfBias + 128,
              kDfBar = kDfRed + red_bytes(kTDesliceFwd, 2), kDfBytes = kDfBar + kBarBytes;

template <typename PT>
__global__ void __launch_bounds__(128 * kTDesliceFwd, kCtasDesliceFwd)
    k_tc_deslice_fwd(const __grid_constant__ TcParams p) {
  constexpr int T = kTDesliceFwd, NT = Th<T>::NT, C = Th<T>::C;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<kDfCols>(sm, kDfBar, p.wait_ns);
  float* red = (float*)(sm + kDfRed);
  put_small<NT>(sm + kDfWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  if constexpr (kNwDf == 32)
    put_small<NT>(sm + kDfTs, p.M + (int64_t)bh * 32 * 32);
  else
    put_small_stacked<NT>(sm + kDfTs, p.M + (int64_t)bh * 32 * 32);
  const RowConst rc = row_const<NT>((float*)(sm + kDfBias),
                                    p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tA = c.tmem + kNwDf;
  const uint64_t dWs = desc_smallK(sm + kDfWs);
  const uint64_t dTs = kNwDf == 32 ? desc_smallM(sm + kDfTs) : desc_stacked(sm + kDfTs);
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles) tma_tile<PT>(p, sm + kDfStageX, nullptr, h, sp, tile, c.bar);
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<C, PT> x;
      x.load(sm + kDfStageX, th.row, th.cs);
      x.split().to_tmem(tA + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      prefetch<PT>(p, sm + kDfStageX, nullptr, h, sp, tile, c.bar);
      wide_ts<kNwDf, false, kHi<PT>>(tL, tA, dWs);  // logits = x W^T
      commit(c, kG1);
    }
    wait_bar(c, kG1, p.status);
    {
      float lg[C];
      ld_wide<kNwDf, C>(tL + th.lane_off, th.cs, lg);
      softmax_fwd<T, C>(lg, rc, true, red, th);
      Split<C>(lg).to_tmem(tA + th.lane_off, th.cs);  // w, over the consumed x
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide_ts<kNwDf, true>(tL, tA, dTs);  // out = w tokens, over the consumed logits
      commit(c, kG2);
    }
    wait_bar(c, kG2, p.status);
    store_result<kNwDf, C>(tL, th.q, th.cs,
                           (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                               (int64_t)h * p.so[2],
                           p.so[1], sp.N - n0);
  }
  epilogue<kDfCols>(c);
}

// ------------------------------------------------------------ slice backward
// smem: [stage x][stage fx][X split][UP split: dl/tau][W][dz_num][bias][ds][red][bars]
// TMEM (256 columns): logits (N-stacked) at 0, dw at 96, point operands x at
// 160 and fx at 208; then dfx at 0, dx at 32, the dW pool at 64 and point
// operands w at 160 and dl/tau at 208. The operands written at the start of
// a tile are disjoint from the columns read at the end of the previous one.
// MMAs are committed in groups (logits; dw; dfx and dx; the pool) so that
// the threads start on each result while the next group runs.
constexpr int kSbStageX = 0, kSbStageF = kStage, kSbX = 2 * kStage, kSbUp = kSbX + kSplit,
              kSbWs = kSbUp + kSplit + kTail, kSbZs = kSbWs + kSmall, kSbBias = kSbZs + kSmall,
              kSbDs = kSbBias + 128, kSbRed = kSbDs + 128,
              kSbBar = kSbRed + red_bytes(kTSliceBwd, 3), kSbBytes = kSbBar + kBarBytes;

template <typename PT>
__global__ void __launch_bounds__(128 * kTSliceBwd, kCtasSliceBwd)
    k_tc_slice_bwd(const __grid_constant__ TcParams p) {
  constexpr int T = kTSliceBwd, NT = Th<T>::NT, C = Th<T>::C;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kSbBar, p.wait_ns);
  float* ds_s = (float*)(sm + kSbDs);
  float* red = (float*)(sm + kSbRed);
  put_small<NT>(sm + kSbWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  put_small<NT>(sm + kSbZs, p.M + (int64_t)bh * 32 * 32);
  const RowConst rc = row_const<NT>((float*)(sm + kSbBias),
                                    p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  if (threadIdx.x < 32) ds_s[threadIdx.x] = p.ds[(int64_t)bh * 32 + threadIdx.x];
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tDw = c.tmem + 96, tX = c.tmem + 160, tF = c.tmem + 208;
  const uint32_t tDfx = c.tmem, tDx = c.tmem + 32, tP = c.tmem + 64, tW = c.tmem + 160,
                 tU = c.tmem + 208;
  const uint64_t dXb = desc_stacked(sm + kSbX), dUp = desc_stacked(sm + kSbUp);
  const uint64_t dWk = desc_smallK(sm + kSbWs), dWm = desc_smallM(sm + kSbWs);
  const uint64_t dZk = desc_smallK(sm + kSbZs), dZm = desc_smallM(sm + kSbZs);
  float accw[C], accb[C], dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) accw[i] = accb[i] = 0.f;
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles)
    tma_tile<PT>(p, sm + kSbStageX, sm + kSbStageF, h, sp, tile, c.bar);
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + th.row < sp.N;
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<C, PT> x, f;
      x.load(sm + kSbStageX, th.row, th.cs);
      f.load(sm + kSbStageF, th.row, th.cs);
      const Split<C> xs = x.split();
      xs.to_smem(sm + kSbX, th.row, th.cs);
      xs.to_tmem(tX + th.lane_off, th.cs);
      f.split().to_tmem(tF + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      prefetch<PT>(p, sm + kSbStageX, sm + kSbStageF, h, sp, tile, c.bar);
      wide_ts<96, false, kHi<PT>>(tL, tX, dWk);  // logits = x W^T
      commit(c, kG1);
      wide_ts<64, false, kHi<PT>>(tDw, tF, dZk);  // dw = fx dz_num^T
      commit(c, kG2);
    }
    {
      float w[C], dw[C];
      wait_bar(c, kG1, p.status);
      ld_wide<96, C>(tL + th.lane_off, th.cs, w);
      wait_bar(c, kG2, p.status);
      ld_wide<64, C>(tDw + th.lane_off, th.cs, dw);
      const float2* ds2 = (const float2*)(ds_s + th.cs * C);
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(dw, k, __fadd2_rn(f2(dw, k), ds2[k]));
      const float rdt = softmax_bwd<T, C>(w, dw, rc, inv_tau, valid, red, th);
      if (valid) dt_acc += rdt;
      Split<C>(w).to_tmem(tW + th.lane_off, th.cs);
      const Split<C> us(dw);  // dl / tau
      us.to_tmem(tU + th.lane_off, th.cs);
      us.to_smem(sm + kSbUp, th.row, th.cs);
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(accb, k, __fadd2_rn(f2(accb, k), f2(dw, k)));
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide_ts<32, true>(tDfx, tW, dZm);  // dfx = w dz_num
      wide_ts<32, true>(tDx, tU, dWm);   // dx = (dl/tau) W
      commit(c, kG3);
      mma_pool(tP, dUp, dXb);  // dW += (dl/tau)^T x
      commit(c, kG4);
    }
    wait_bar(c, kG3, p.status);
    store_result<32, C>(tDfx, th.q, th.cs,
                        (PT*)p.out2 + (int64_t)sp.bc * p.so2[0] + (sp.n0 + n0) * p.so2[1] +
                            (int64_t)h * p.so2[2],
                        p.so2[1], sp.N - n0);
    store_result<32, C>(tDx, th.q, th.cs,
                        (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                            (int64_t)h * p.so[2],
                        p.so[1], sp.N - n0);
    wait_bar(c, kG4, p.status);
    if (th.q < 3) drain_pool<C>(tP + th.lane_off, th.cs, accw);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kSbX);
  tc_fence_before();
  pool_write<T>(xch, accw, p.partA + slot * 32 * 32, th);
  rowsum_write<T>(xch, accb, p.partS + slot * 32, th);
  const float tot = cta_sum_nt<NT>(dt_acc, (float*)(sm + kSbUp));
  if (threadIdx.x == 0) p.partDt[slot] = -inv_tau * kLn2 * tot;
  epilogue<256>(c);
}

// ------------------------------------------------------------ deslice backward
// Sized for two CTAs per SM (shared memory 111 KB, TMEM 256 columns).
// smem: [X split][O split: dout][WP split: w | stage x][UP split: dl/tau |
//       stage dout][W][tokens][bias][red][bars]
// The staging tiles share the pool operands' buffers: the next tile's x is
// loaded into WP once the dtokens pool is done with it, its d_out into UP
// once the dW pool is.
// TMEM: logits (N-stacked) at 0, dw at 96, point operands x -> dl/tau at
// 160 and dout at 208; then dx at 0 and one pool at 32 (dtokens, then dW).
constexpr int kDbX = 0, kDbO = kSplit, kDbWp = 2 * kSplit, kDbUp = 3 * kSplit,
              kDbWs = 4 * kSplit, kDbTs = kDbWs + kSmall, kDbBias = kDbTs + kSmall,
              kDbRed = kDbBias + 128, kDbBar = kDbRed + red_bytes(kTDesliceBwd, 3),
              kDbBytes = kDbBar + kBarBytes;
static_assert(kDbWp % 1024 == 0 && kDbUp % 1024 == 0, "staging tiles need 1 KB alignment");

template <typename PT>
__global__ void __launch_bounds__(128 * kTDesliceBwd, kCtasDesliceBwd)
    k_tc_deslice_bwd(const __grid_constant__ TcParams p) {
  constexpr int T = kTDesliceBwd, NT = Th<T>::NT, C = Th<T>::C;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kDbBar, p.wait_ns);
  float* red = (float*)(sm + kDbRed);
  put_small<NT>(sm + kDbWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  put_small<NT>(sm + kDbTs, p.M + (int64_t)bh * 32 * 32);
  const RowConst rc = row_const<NT>((float*)(sm + kDbBias),
                                    p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tDw = c.tmem + 96, tX = c.tmem + 160, tO = c.tmem + 208;
  const uint32_t tDx = c.tmem, tP = c.tmem + 32;
  const uint64_t dXb = desc_stacked(sm + kDbX), dOb = desc_stacked(sm + kDbO),
                 dWp = desc_stacked(sm + kDbWp), dUp = desc_stacked(sm + kDbUp);
  const uint64_t dWk = desc_smallK(sm + kDbWs), dWm = desc_smallM(sm + kDbWs),
                 dTk = desc_smallK(sm + kDbTs);
  uint8_t* stX = sm + kDbWp;
  uint8_t* stO = sm + kDbUp;
  float acct[C], accw[C], accb[C], dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) acct[i] = accw[i] = accb[i] = 0.f;
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles) tma_tile<PT>(p, stX, stO, h, sp, tile, c.bar);
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + th.row < sp.N;
    const bool more = tile + p.P < sp.ntiles;
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<C, PT> x, o;
      x.load(stX, th.row, th.cs);
      o.load(stO, th.row, th.cs);
      const Split<C> xs = x.split();
      xs.to_smem(sm + kDbX, th.row, th.cs);
      xs.to_tmem(tX + th.lane_off, th.cs);
      const Split<C> os = o.split();
      os.to_smem(sm + kDbO, th.row, th.cs);
      os.to_tmem(tO + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide_ts<96, false, kHi<PT>>(tL, tX, dWk);  // logits = x W^T
      commit(c, kG1);
      wide_ts<64, false, kHi<PT>>(tDw, tO, dTk);  // dw = d_out tok^T
      commit(c, kG2);
    }
    {
      float w[C], dw[C];
      wait_bar(c, kG1, p.status);
      ld_wide<96, C>(tL + th.lane_off, th.cs, w);
      wait_bar(c, kG2, p.status);
      ld_wide<64, C>(tDw + th.lane_off, th.cs, dw);
      const float rdt = softmax_bwd<T, C>(w, dw, rc, inv_tau, valid, red, th);
      if (valid) dt_acc += rdt;
      Split<C>(w).to_smem(sm + kDbWp, th.row, th.cs);  // over the consumed x stage
      const Split<C> us(dw);                            // dl / tau
      us.to_smem(sm + kDbUp, th.row, th.cs);           // over the consumed dout stage
      us.to_tmem(tX + th.lane_off, th.cs);             // over the consumed x operand
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(accb, k, __fadd2_rn(f2(accb, k), f2(dw, k)));
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide_ts<32, true>(tDx, tX, dWm);  // dx = (dl/tau) W
      commit(c, kG3);
      mma_pool(tP, dWp, dOb);  // dtokens += w^T d_out
      commit(c, kG4);
    }
    wait_bar(c, kG3, p.status);
    store_result<32, C>(tDx, th.q, th.cs,
                        (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                            (int64_t)h * p.so[2],
                        p.so[1], sp.N - n0);
    wait_bar(c, kG4, p.status);
    if (th.q < 3) drain_pool<C>(tP + th.lane_off, th.cs, acct);
    tc_fence_before();
    __syncthreads();  // the pool region is read out; WP is free
    tc_fence_after();
    if (c.issuer()) {
      if (more) {
        mbar_arrive_expect_tx(c.bar + kBarTma, 2 * stage_bytes<PT>());
        tma_load_4d(stX, &p.mx, 0, h, sp.row(tile + p.P), sp.bc, c.bar + kBarTma);
      }
      mma_pool(tP, dUp, dXb);  // dW += (dl/tau)^T x
      commit(c, kG5);
    }
    wait_bar(c, kG5, p.status);
    if (c.issuer() && more)  // UP is free once the dW pool is done
      tma_load_4d(stO, &p.mv, 0, h, sp.row(tile + p.P), sp.bc, c.bar + kBarTma);
    if (th.q < 3) drain_pool<C>(tP + th.lane_off, th.cs, accw);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kDbX);
  tc_fence_before();
  pool_write<T>(xch, acct, p.partB + slot * 32 * 32, th);
  pool_write<T>(xch, accw, p.partA + slot * 32 * 32, th);
  rowsum_write<T>(xch, accb, p.partS + slot * 32, th);
  const float tot = cta_sum_nt<NT>(dt_acc, (float*)(sm + kDbO));
  if (threadIdx.x == 0) p.partDt[slot] = -inv_tau * kLn2 * tot;
  epilogue<256>(c);
}

// ------------------------------------------------------------ coupled backward
// The backward of a whole coupling round (slice -> tokens -> deslice) once
// the dtokens pass has run (dtokens = sum_n w^T d_out is a slice forward with
// d_out in place of fx). Per point the two ops' gradients share the softmax
// and are linear in the upstream dw, so with
//   dw = d_out tok^T + fx dz_num^T + ds,  dl = w (dw - sum_g w dw),
// one pass gives dx = (dl/tau) W, dW = (dl/tau)^T x, db = sum dl/tau and
// dtau = -(1/tau) sum dl (logit - rowmax) for slice and deslice together,
// and dfx = w dz_num; x is read once and dx written once, with no separate
// sum of two dx tensors.
// smem: [stage x][stage fx][X split][UP split: dl/tau | stage d_out][W]
//       [tokens][dz_num][bias][ds][red][bars]
// The d_out staging tile shares UP: the next tile's d_out is loaded once the
// dW pool is done with UP.
// TMEM (256 columns): logits (N-stacked, from the x split in shared memory)
// at 0, d_out tok^T + fx dz_num^T at 96 (one 64-column accumulator), point
// operands fx at 160 and d_out at 208; then dfx at 0, dx
// at 32, the dW pool at 64, point operands w at 160 and dl/tau at 208. The
// operands written at the start of a tile are disjoint from the columns read
// at its end. The pool is issued first in the second group, so that the
// next tile's d_out (staged in UP) loads while dfx and dx are formed.
#ifndef FS_TC_CB_T
#define FS_TC_CB_T 2
#endif
constexpr int kTCoupledBwd = FS_TC_CB_T, kCtasCoupledBwd = 2;
constexpr int kCbStageX = 0, kCbStageF = kStage, kCbX = 2 * kStage, kCbUp = kCbX + kSplit,
              kCbWs = kCbUp + kSplit + kTail, kCbTs = kCbWs + kSmall, kCbZs = kCbTs + kSmall,
              kCbBias = kCbZs + kSmall, kCbDs = kCbBias + 128, kCbRed = kCbDs + 128,
              kCbBar = kCbRed + red_bytes(kTCoupledBwd, 3), kCbBytes = kCbBar + kBarBytes;
static_assert(kCbUp % 1024 == 0, "the d_out staging tile needs 1 KB alignment");

template <typename PT>
__global__ void __launch_bounds__(128 * kTCoupledBwd, kCtasCoupledBwd)
    k_tc_coupled_bwd(const __grid_constant__ TcParams p) {
  constexpr int T = kTCoupledBwd, NT = Th<T>::NT, C = Th<T>::C;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kCbBar, p.wait_ns);
  float* ds_s = (float*)(sm + kCbDs);
  float* red = (float*)(sm + kCbRed);
  put_small<NT>(sm + kCbWs, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  put_small<NT>(sm + kCbTs, p.M + (int64_t)bh * 32 * 32);
  put_small<NT>(sm + kCbZs, p.M2 + (int64_t)bh * 32 * 32);
  const RowConst rc = row_const<NT>((float*)(sm + kCbBias),
                                    p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  if (threadIdx.x < 32) ds_s[threadIdx.x] = p.ds[(int64_t)bh * 32 + threadIdx.x];
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tD = c.tmem + 96, tF = c.tmem + 160, tO = c.tmem + 208;
  const uint32_t tDfx = c.tmem, tDx = c.tmem + 32, tP = c.tmem + 64, tW = c.tmem + 160,
                 tU = c.tmem + 208;
  const uint64_t dXa = desc_rowsA(sm + kCbX), dXb = desc_stacked(sm + kCbX),
                 dUp = desc_stacked(sm + kCbUp);
  const uint64_t dWk = desc_smallK(sm + kCbWs), dWm = desc_smallM(sm + kCbWs);
  const uint64_t dTk = desc_smallK(sm + kCbTs);
  const uint64_t dZk = desc_smallK(sm + kCbZs), dZm = desc_smallM(sm + kCbZs);
  uint8_t* stX = sm + kCbStageX;
  uint8_t* stF = sm + kCbStageF;
  uint8_t* stO = sm + kCbUp;
  float accw[C], accb[C], dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) accw[i] = accb[i] = 0.f;
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles) {
    mbar_arrive_expect_tx(c.bar + kBarTma, 3 * stage_bytes<PT>());
    tma_load_4d(stX, &p.mx, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    tma_load_4d(stF, &p.mv, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    tma_load_4d(stO, &p.mo, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
  }
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + th.row < sp.N;
    const bool more = tile + p.P < sp.ntiles;
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<C, PT> x, f, o;
      x.load(stX, th.row, th.cs);
      f.load(stF, th.row, th.cs);
      o.load(stO, th.row, th.cs);
      x.split().to_smem(sm + kCbX, th.row, th.cs);
      f.split().to_tmem(tF + th.lane_off, th.cs);
      o.split().to_tmem(tO + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      if (more) {  // x and fx of the next tile; its d_out once UP is free
        mbar_arrive_expect_tx(c.bar + kBarTma, 3 * stage_bytes<PT>());
        tma_load_4d(stX, &p.mx, 0, h, sp.row(tile + p.P), sp.bc, c.bar + kBarTma);
        tma_load_4d(stF, &p.mv, 0, h, sp.row(tile + p.P), sp.bc, c.bar + kBarTma);
      }
      wide_ss96<kHi<PT>>(tL, dXa, dWk);  // logits = x W^T
      commit(c, kG1);
      wide_ts64_pair<false, 2, kHi<PT>>(tD, tO, dTk, tF, dZk);  // d_out tok^T + fx dz_num^T
      commit(c, kG2);
    }
    {
      float w[C], dw[C];
      wait_bar(c, kG1, p.status);
      ld_wide<96, C>(tL + th.lane_off, th.cs, w);
      wait_bar(c, kG2, p.status);
      ld_wide<64, C>(tD + th.lane_off, th.cs, dw);
      const float2* ds2 = (const float2*)(ds_s + th.cs * C);
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(dw, k, __fadd2_rn(f2(dw, k), ds2[k]));
      const float rdt = softmax_bwd<T, C>(w, dw, rc, inv_tau, valid, red, th);
      if (valid) dt_acc += rdt;
      Split<C>(w).to_tmem(tW + th.lane_off, th.cs);
      const Split<C> us(dw);  // dl / tau
      us.to_tmem(tU + th.lane_off, th.cs);
      us.to_smem(sm + kCbUp, th.row, th.cs);  // over the consumed d_out stage
#pragma unroll
      for (int k = 0; k < C / 2; ++k) put2(accb, k, __fadd2_rn(f2(accb, k), f2(dw, k)));
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      mma_pool(tP, dUp, dXb);  // dW += (dl/tau)^T x
      commit(c, kG3);
      wide_ts<32, true>(tDfx, tW, dZm);  // dfx = w dz_num
      wide_ts<32, true>(tDx, tU, dWm);   // dx = (dl/tau) W
      commit(c, kG4);
    }
    wait_bar(c, kG3, p.status);
    if (c.issuer() && more)  // UP is free once the dW pool is done
      tma_load_4d(stO, &p.mo, 0, h, sp.row(tile + p.P), sp.bc, c.bar + kBarTma);
    if (th.q < 3) drain_pool<C>(tP + th.lane_off, th.cs, accw);
    wait_bar(c, kG4, p.status);
    store_result<32, C>(tDfx, th.q, th.cs,
                        (PT*)p.out2 + (int64_t)sp.bc * p.so2[0] + (sp.n0 + n0) * p.so2[1] +
                            (int64_t)h * p.so2[2],
                        p.so2[1], sp.N - n0);
    store_result<32, C>(tDx, th.q, th.cs,
                        (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                            (int64_t)h * p.so[2],
                        p.so[1], sp.N - n0);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* xch = (float*)(sm + kCbX);
  tc_fence_before();
  pool_write<T>(xch, accw, p.partA + slot * 32 * 32, th);
  rowsum_write<T>(xch, accb, p.partS + slot * 32, th);
  const float tot = cta_sum_nt<NT>(dt_acc, (float*)(sm + kCbUp));
  if (threadIdx.x == 0) p.partDt[slot] = -inv_tau * kLn2 * tot;
  epilogue<256>(c);
}

// ------------------------------------------------------------ blocked slice forward, bf16 dots
// The slot-owning slice forward of the blocked family (blocked.py:404-462)
// for bf16 point tensors in the bf16 dot mode, D = 32, DV in {32, 64}, G a
// multiple of 128, with the per-point statistics (m, l) given. One CTA owns
// 128 slots of one (b, h) and streams the points:
//  * logits = x W^T on the tensor cores: the bf16 x times W's two bf16 parts
//    (hi, mid: 16 significant bits, four MMAs, N = 128), within 2^-17 of the
//    fp32 logits the statistics are formed from;
//  * w = exp(logit - m) / l per point, rounded to bf16 (the bf16 dot mode's
//    value dot, blocked.py), written as the pool's slot-major operand;
//  * z_num += w^T fx and s += w^T 1 (MMAs with N = DV and N = 16) accumulate
//    in TMEM over the CTA's tiles.
// Point tiles arrive by TMA as 16-byte column boxes, which lays them out as
// the MMAs' operands directly (x K-major, fx point-major), double-buffered.
// Two threads per point row (64 slots each); two CTAs per SM.
// smem: [W parts x 2 (16 KB)][bias][x stage x 2][fx stage x 2][w tile][ones][bars]
// TMEM: logits at 0 (128 columns), z_num at 128 (DV), s at 192 (16).
constexpr int kBgSlots = 128;
constexpr int kBgWs = 0, kBgBias = 2 * 8192, kBgX = kBgBias + 1024, kBgF = kBgX + 2 * 8192,
              kBgW = kBgF + 2 * 16384, kBgOnes = kBgW + 32768, kBgBar = kBgOnes + 4096,
              kBgBytes = kBgBar + kBarBytes;
static_assert(kBgX % 1024 == 0 && kBgF % 1024 == 0 && kBgW % 1024 == 0, "blocked slice layout");

__global__ void __launch_bounds__(256, 2) k_tc_blk_slice_fwd_bf16(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int gb = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh - b * p.H;
  const int g0 = gb * kBgSlots, DV = p.dv;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kBgBar, p.wait_ns);
  // W rows g0 .. g0 + 127, two bf16 parts (mid, hi), K-major (rows g, k = d)
  {
    const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh + (int64_t)g0 * 32;
    for (int i = threadIdx.x; i < kBgSlots * 32; i += 256) {
      const int r = i >> 5, k = i & 31;
      __nv_bfloat16 hi, mi;
      split2(Wb[i], hi, mi);
      const uint32_t o = kmajor_off(r, k, 32);
      *(__nv_bfloat16*)(sm + kBgWs + o) = mi;
      *(__nv_bfloat16*)(sm + kBgWs + 8192 + o) = hi;
    }
    const float inv_tau = __frcp_rn(p.tau[h]);
    float* bias2 = (float*)(sm + kBgBias);
    if (threadIdx.x < kBgSlots)
      bias2[threadIdx.x] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + g0 + threadIdx.x] *
                           inv_tau * kLog2e;
    uint32_t* ones = (uint32_t*)(sm + kBgOnes);
    for (int i = threadIdx.x; i < 1024; i += 256) ones[i] = 0x3F803F80u;  // bf16 1.0 pairs
  }
  prologue_end(c);
  const float scale = __frcp_rn(p.tau[h]) * kLog2e;
  const float* bias2 = (const float*)(sm + kBgBias);
  const uint32_t tL = c.tmem, tZ = c.tmem + 128, tS = c.tmem + 192;
  // two threads per point row (64 slots each); threads 0-127 own a slot each at the end
  const int warp = threadIdx.x >> 5, row = 32 * (warp & 3) + (threadIdx.x & 31), half = warp >> 2;
  const uint32_t tlane = (uint32_t)(32 * (warp & 3)) << 16;  // its TMEM lanes
  const uint32_t stage_b = (uint32_t)(4 + DV / 8) * 2048;  // bytes of one tile's boxes
  auto xs = [&](int k) { return sm + kBgX + (k & 1) * 8192; };
  auto fs = [&](int k) { return sm + kBgF + (k & 1) * 16384; };
  auto load = [&](int k, int tile) {  // tile's x (4 boxes) and fx (DV / 8 boxes), one thread
    mbar_arrive_expect_tx(c.bar + kBarTma, stage_b);
    for (int q = 0; q < 4; ++q)
      tma_load_4d(xs(k) + q * 2048, &p.mx, 8 * q, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    for (int q = 0; q < DV / 8; ++q)
      tma_load_4d(fs(k) + q * 2048, &p.mv, 8 * q, h, sp.row(tile), sp.bc, c.bar + kBarTma);
  };
  const uint32_t id_l = idesc_bf16(128, 128, 0, 0), id_z = idesc_bf16(128, DV == 64 ? 64 : 32, 1, 1),
                 id_s = idesc_bf16(128, 16, 1, 1);
  const int n_my = sp.ntiles > (int)blockIdx.x ? (sp.ntiles - 1 - (int)blockIdx.x) / p.P + 1 : 0;
  if (c.issuer() && n_my > 0) load(0, blockIdx.x);
  for (int k = 0; k < n_my; ++k) {
    const int tile = blockIdx.x + k * p.P, n0 = tile * kTile;
    wait_bar(c, kBarTma, p.status);
    if (c.issuer()) {  // logits: x times W mid, hi (small first)
      for (int part = 0; part < 2; ++part)
        for (int ks = 0; ks < 2; ++ks)
          mma_bf16(tL, smem_desc(smem_u32(xs(k)) + ks * 4096, 2048, 128),
                   smem_desc(smem_u32(sm + kBgWs + part * 8192) + ks * 256, 128, 512), id_l,
                   (part | ks) != 0);
      commit(c, kG1);
    }
    if (k > 0) wait_bar(c, kG2, p.status);  // tile k - 1's pool: its buffers and the w tile free
    if (c.issuer() && k + 1 < n_my) load(k + 1, tile + p.P);
    wait_bar(c, kG1, p.status);
    {
      const int n = n0 + row;
      const bool valid = n < sp.N;
      float m2 = 0.f, inv_l = 0.f;
      if (valid) {
        const float* st = p.stats_in + (int64_t)bh * 2 * p.N;
        const int64_t ni = sp.n0 + n;
        m2 = st[ni] * kLog2e;
        inv_l = __frcp_rn(st[p.N + ni]);
      }
      uint8_t* wrow = sm + kBgW + (row >> 3) * (kBgSlots * 16) + (row & 7) * 16;
#pragma unroll
      for (int hc = 0; hc < 2; ++hc) {
        const int ch = 2 * half + hc;  // this thread's 32-slot chunks
        uint32_t r[32];
        tld<32>(tL + tlane + ch * 32, r);
        tld_wait();
        uint32_t wv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int g = ch * 32 + 2 * j;
          const float a =
              valid ? ex2(__uint_as_float(r[2 * j]) * scale + bias2[g] - m2) * inv_l : 0.f;
          const float e =
              valid ? ex2(__uint_as_float(r[2 * j + 1]) * scale + bias2[g + 1] - m2) * inv_l : 0.f;
          wv[j] = bf2_bits(__floats2bfloat162_rn(a, e));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)  // slots ch*32 + 8q .. +7: one 16-byte chunk
          *(uint4*)(wrow + (ch * 4 + q) * 128) =
              make_uint4(wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
      }
    }
    to_async_barrier();
    if (c.issuer()) {  // z_num += w^T fx, s += w^T 1, 16 points a step
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ad = smem_desc(smem_u32(sm + kBgW) + ks * 2 * (kBgSlots * 16), kBgSlots * 16, 128);
        mma_bf16(tZ, ad, smem_desc(smem_u32(fs(k)) + ks * 256, 128, 2048), id_z, (k | ks) != 0);
        mma_bf16(tS, ad, smem_desc(smem_u32(sm + kBgOnes) + ks * 256, 128, 2048), id_s,
                 (k | ks) != 0);
      }
      commit(c, kG2);
    }
  }
  if (n_my > 0) wait_bar(c, kG2, p.status);
  tc_fence_after();
  // this CTA's partial sums: threads 0-127, slot g0 + row
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* pz = p.partA + (slot * p.G + g0 + row) * DV;
  float* ps = p.partS + slot * p.G + g0 + row;
  if (half == 1) {
  } else if (n_my > 0) {
    uint32_t r[32];
    for (int ch = 0; ch < DV / 32; ++ch) {
      tld<32>(tZ + tlane + ch * 32, r);
      tld_wait();
      for (int j = 0; j < 32; ++j) pz[ch * 32 + j] = __uint_as_float(r[j]);
    }
    tld<32>(tS + tlane, r);  // 16 columns read, the first holds s
    tld_wait();
    *ps = __uint_as_float(r[0]);
  } else {
    for (int j = 0; j < DV; ++j) pz[j] = 0.f;
    *ps = 0.f;
  }
  epilogue<256>(c);
}

// ------------------------------------------------------------ blocked backward, slot-owning, bf16 dots
// The slot-owning half of the blocked backward (slice: dW, db, blocked.py:
// 677-741; deslice: dW, db, dtokens, :819-888) for bf16 point tensors in the
// bf16 dot mode, D = 32, DV in {32, 64}, G a multiple of 128, given the
// statistics and the point-owning pass's delta and row sums. One CTA owns 128
// slots of one (b, h) and streams the points; per tile:
//  * logits = x W^T and dw = v M^T (v = d_out with M = tokens, or v = fx with
//    M = dz_num, plus ds) on the tensor cores, W and M in two bf16 parts (16
//    significant bits; the bf16 x and v are exact), N = 128: the products
//    the point-owning kernels form;
//  * w = exp(logit - m) / l, dl = w (dw - delta) / tau, written as bf16
//    slot-major operands (the bf16 value dots);
//  * dW += dl^T x, db += dl^T 1 and, deslice, dtokens += w^T d_out,
//    accumulated in TMEM over the CTA's tiles.
// Four threads per point row (32 slots each). One CTA per SM (TMEM).
// smem: [W parts][M parts][bias][ds][x stage x 2][v stage x 2][dl tile][w tile][ones][bars]
// TMEM: logits 0, dw 128, dW 256 (32), db 288 (16), dtokens 320 (DV).
constexpr int kBbW = 0, kBbM = 2 * 8192, kBbBias = kBbM + 2 * 16384, kBbDs = kBbBias + 512,
              kBbX = kBbDs + 512 + 1024 - ((kBbDs + 512) % 1024), kBbV = kBbX + 2 * 8192,
              kBbDl = kBbV + 2 * 16384, kBbWt = kBbDl + 32768, kBbOnes = kBbWt + 32768,
              kBbBar = kBbOnes + 4096, kBbBytes = kBbBar + kBarBytes;
static_assert(kBbX % 1024 == 0 && kBbDl % 1024 == 0, "blocked backward layout");

template <bool SLICE>
__global__ void __launch_bounds__(512, 1) k_tc_blk_bwd_g_bf16(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int gb = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh - b * p.H;
  const int g0 = gb * kBgSlots, DV = p.dv;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<512>(sm, kBbBar, p.wait_ns);
  const float inv_tau = __frcp_rn(p.tau[h]);
  {
    // W rows g0 .. g0 + 127 (K = d, 32) and M rows (K = dv) in two bf16 parts
    // (mid, hi)
    const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh + (int64_t)g0 * 32;
    for (int i = threadIdx.x; i < kBgSlots * 32; i += 512) {
      const int r = i >> 5, k = i & 31;
      __nv_bfloat16 hi, mi;
      split2(Wb[i], hi, mi);
      const uint32_t o = kmajor_off(r, k, 32);
      *(__nv_bfloat16*)(sm + kBbW + o) = mi;
      *(__nv_bfloat16*)(sm + kBbW + 8192 + o) = hi;
    }
    const float* Mb = p.M + ((int64_t)bh * p.G + g0) * DV;
    for (int i = threadIdx.x; i < kBgSlots * DV; i += 512) {
      const int r = i / DV, k = i - r * DV;
      __nv_bfloat16 hi, mi;
      split2(Mb[i], hi, mi);
      const uint32_t o = kmajor_off(r, k, DV);
      *(__nv_bfloat16*)(sm + kBbM + o) = mi;
      *(__nv_bfloat16*)(sm + kBbM + 16384 + o) = hi;
    }
    if (threadIdx.x < kBgSlots) {
      float* bias2 = (float*)(sm + kBbBias);
      bias2[threadIdx.x] = p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + g0 + threadIdx.x] *
                           inv_tau * kLog2e;
      ((float*)(sm + kBbDs))[threadIdx.x] = SLICE ? p.ds[(int64_t)bh * p.G + g0 + threadIdx.x] : 0.f;
    }
    uint32_t* ones = (uint32_t*)(sm + kBbOnes);
    for (int i = threadIdx.x; i < 1024; i += 512) ones[i] = 0x3F803F80u;
  }
  prologue_end(c);
  const float scale = inv_tau * kLog2e;
  const float* bias2 = (const float*)(sm + kBbBias);
  const float* dss = (const float*)(sm + kBbDs);
  const uint32_t tL = c.tmem, tD = c.tmem + 128, tW = c.tmem + 256, tB = c.tmem + 288,
                 tT = c.tmem + 320;
  // four threads per point row, a quarter of the slots each
  const int warp = threadIdx.x >> 5, row = 32 * (warp & 3) + (threadIdx.x & 31), quarter = warp >> 2;
  const uint32_t tlane = (uint32_t)(32 * (warp & 3)) << 16;
  const uint32_t stage_b = (uint32_t)(4 + DV / 8) * 2048;
  auto xs = [&](int k) { return sm + kBbX + (k & 1) * 8192; };
  auto vs = [&](int k) { return sm + kBbV + (k & 1) * 16384; };
  auto load = [&](int k, int tile) {
    mbar_arrive_expect_tx(c.bar + kBarTma, stage_b);
    for (int q = 0; q < 4; ++q)
      tma_load_4d(xs(k) + q * 2048, &p.mx, 8 * q, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    for (int q = 0; q < DV / 8; ++q)
      tma_load_4d(vs(k) + q * 2048, &p.mv, 8 * q, h, sp.row(tile), sp.bc, c.bar + kBarTma);
  };
  const uint32_t id_l = idesc_bf16(128, 128, 0, 0);
  const uint32_t id_w = idesc_bf16(128, 32, 1, 1), id_s = idesc_bf16(128, 16, 1, 1),
                 id_t = idesc_bf16(128, DV == 64 ? 64 : 32, 1, 1);
  const int n_my = sp.ntiles > (int)blockIdx.x ? (sp.ntiles - 1 - (int)blockIdx.x) / p.P + 1 : 0;
  if (c.issuer() && n_my > 0) load(0, blockIdx.x);
  for (int k = 0; k < n_my; ++k) {
    const int tile = blockIdx.x + k * p.P, n0 = tile * kTile;
    wait_bar(c, kBarTma, p.status);
    if (c.issuer()) {
      for (int part = 0; part < 2; ++part)  // logits = x W^T (mid, hi of W)
        for (int ks = 0; ks < 2; ++ks)
          mma_bf16(tL, smem_desc(smem_u32(xs(k)) + ks * 4096, 2048, 128),
                   smem_desc(smem_u32(sm + kBbW + part * 8192) + ks * 256, 128, 512), id_l,
                   (part | ks) != 0);
      for (int part = 0; part < 2; ++part)  // dw = v M^T (mid, hi of M)
        for (int ks = 0; ks < DV / 16; ++ks)
          mma_bf16(tD, smem_desc(smem_u32(vs(k)) + ks * 4096, 2048, 128),
                   smem_desc(smem_u32(sm + kBbM + part * 16384) + ks * 256, 128, DV * 16), id_l,
                   (part | ks) != 0);
      commit(c, kG1);
    }
    if (k > 0) wait_bar(c, kG2, p.status);  // tile k - 1's pools: buffers and tiles free
    if (c.issuer() && k + 1 < n_my) load(k + 1, tile + p.P);
    wait_bar(c, kG1, p.status);
    {
      const int n = n0 + row;
      const bool valid = n < sp.N;
      float m2 = 0.f, r = 0.f, delta = 0.f;
      if (valid) {
        const int64_t ni = sp.n0 + n;
        m2 = p.stats_in[(int64_t)bh * 2 * p.N + ni] * kLog2e;
        delta = p.delta[(int64_t)bh * 2 * p.N + ni];
        r = __frcp_rn(p.delta[(int64_t)bh * 2 * p.N + p.N + ni]);
      }
      uint8_t* dlrow = sm + kBbDl + (row >> 3) * (kBgSlots * 16) + (row & 7) * 16;
      uint8_t* wrow = sm + kBbWt + (row >> 3) * (kBgSlots * 16) + (row & 7) * 16;
      {
        const int c0 = quarter * 32;
        uint32_t lr[32], dr[32];
        tld<32>(tL + tlane + c0, lr);
        tld<32>(tD + tlane + c0, dr);
        tld_wait();
        uint32_t dl2[16], w2[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float wv[2], dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int g = c0 + 2 * j + e;
            const float w = valid ? ex2(__uint_as_float(lr[2 * j + e]) * scale + bias2[g] - m2) * r
                                  : 0.f;
            const float dwv = __uint_as_float(dr[2 * j + e]) + dss[g];
            wv[e] = w;
            dv[e] = w * (dwv - delta) * inv_tau;
          }
          dl2[j] = bf2_bits(__floats2bfloat162_rn(dv[0], dv[1]));
          w2[j] = bf2_bits(__floats2bfloat162_rn(wv[0], wv[1]));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (c0 >> 3) + q;
          *(uint4*)(dlrow + chunk * 128) =
              make_uint4(dl2[4 * q], dl2[4 * q + 1], dl2[4 * q + 2], dl2[4 * q + 3]);
          if (!SLICE)
            *(uint4*)(wrow + chunk * 128) =
                make_uint4(w2[4 * q], w2[4 * q + 1], w2[4 * q + 2], w2[4 * q + 3]);
        }
      }
    }
    to_async_barrier();
    if (c.issuer()) {  // dW += dl^T x, db += dl^T 1, dtokens += w^T d_out
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ad = smem_desc(smem_u32(sm + kBbDl) + ks * 4096, 2048, 128);
        mma_bf16(tW, ad, smem_desc(smem_u32(xs(k)) + ks * 256, 128, 2048), id_w, (k | ks) != 0);
        mma_bf16(tB, ad, smem_desc(smem_u32(sm + kBbOnes) + ks * 256, 128, 2048), id_s,
                 (k | ks) != 0);
        if (!SLICE)
          mma_bf16(tT, smem_desc(smem_u32(sm + kBbWt) + ks * 4096, 2048, 128),
                   smem_desc(smem_u32(vs(k)) + ks * 256, 128, 2048), id_t, (k | ks) != 0);
      }
      commit(c, kG2);
    }
  }
  if (n_my > 0) wait_bar(c, kG2, p.status);
  tc_fence_after();
  // partial sums: threads 0-127, one slot each
  if (threadIdx.x < 128) {
    const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
    const int g = g0 + threadIdx.x;
    float* pw = p.partA + (slot * p.G + g) * 32;
    float* pb = p.partS + slot * p.G + g;
    uint32_t rr[32];
    if (n_my > 0) {
      tld<32>(tW + tlane, rr);
      tld_wait();
      for (int j = 0; j < 32; ++j) pw[j] = __uint_as_float(rr[j]);
      tld<32>(tB + tlane, rr);
      tld_wait();
      *pb = __uint_as_float(rr[0]);
      if (!SLICE) {
        float* pt = p.partB + (slot * p.G + g) * DV;
        for (int ch = 0; ch < DV / 32; ++ch) {
          tld<32>(tT + tlane + ch * 32, rr);
          tld_wait();
          for (int j = 0; j < 32; ++j) pt[ch * 32 + j] = __uint_as_float(rr[j]);
        }
      }
    } else {
      for (int j = 0; j < 32; ++j) pw[j] = 0.f;
      *pb = 0.f;
      if (!SLICE)
        for (int j = 0; j < DV; ++j) p.partB[(slot * p.G + g) * DV + j] = 0.f;
    }
  }
  epilogue<512>(c);
}

// ------------------------------------------------------------ blocked point-owning kernels, bf16 dots
// Operand image of one (b, h, block of 64 slots) for the point-owning
// kernels, written once per call by k_tc_blk_image and copied into shared
// memory by one bulk copy wherever a kernel walks that block:
//   [bias log2(e) / tau, 64 floats][ds, 64 floats (zeros without ds)]
//   [W mid][W hi]  64 x 32 bf16 each, K-major rows g (4 KB)
//   [M hi][M mid]  64 x DV bf16 each, K-major rows g
// W and M (tokens or dz_num) in two bf16 parts (16 significant bits); the hi
// parts are also the value dots' bf16 operands, read MN-major. Without M
// (p.M null, the statistics) the M parts are left unwritten.
constexpr int kPnSlots = 64;
constexpr int kImBias = 0, kImDs = 256, kImW = 512, kImM = kImW + 2 * 4096;
__host__ __device__ constexpr int im_mpart(int dv) { return kPnSlots * dv * 2; }
__host__ __device__ constexpr int im_bytes(int dv) { return kImM + 2 * im_mpart(dv); }
static_assert(im_bytes(32) % 16 == 0 && im_bytes(64) % 16 == 0, "image alignment");

__global__ void __launch_bounds__(256) k_tc_blk_image(const __grid_constant__ TcParams p) {
  const int gb = blockIdx.x, bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const int g0 = gb * kPnSlots, DV = p.dv, mp = im_mpart(DV);
  uint8_t* im = p.img + ((int64_t)bh * (p.G / kPnSlots) + gb) * im_bytes(DV);
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh + (int64_t)g0 * 32;
  for (int i = threadIdx.x; i < kPnSlots * 32; i += 256) {
    const int r = i >> 5, k = i & 31;
    __nv_bfloat16 hi, mi;
    split2(Wb[i], hi, mi);
    const uint32_t o = kmajor_off(r, k, 32);
    *(__nv_bfloat16*)(im + kImW + o) = mi;
    *(__nv_bfloat16*)(im + kImW + 4096 + o) = hi;
  }
  const float* Mb = p.M + ((int64_t)bh * p.G + g0) * DV;
  for (int i = threadIdx.x; p.M && i < kPnSlots * DV; i += 256) {
    const int r = i / DV, k = i - r * DV;
    __nv_bfloat16 hi, mi;
    split2(Mb[i], hi, mi);
    const uint32_t o = kmajor_off(r, k, DV);
    *(__nv_bfloat16*)(im + kImM + o) = hi;
    *(__nv_bfloat16*)(im + kImM + mp + o) = mi;
  }
  if (threadIdx.x < kPnSlots) {
    const float inv_tau = __frcp_rn(p.tau[h]);
    const int g = g0 + threadIdx.x;
    ((float*)(im + kImBias))[threadIdx.x] =
        p.bias[(int64_t)b * p.sbb + (int64_t)h * p.sbh + g] * inv_tau * kLog2e;
    ((float*)(im + kImDs))[threadIdx.x] = p.ds ? p.ds[(int64_t)bh * p.G + g] : 0.f;
  }
}

// The point-owning kernels of the blocked family for bf16 point tensors in
// the bf16 dot mode, D = 32, DV in {32, 64}, G a multiple of 128, given the
// statistics (m, l), or forming them. A CTA owns a 128-point tile at a time
// and walks the blocks of 64 slots, their operand images double-buffered:
//  MODE 3, the statistics, two passes (blocked.py:350-400): m = max_g logit,
//  then l = sum_g exp(logit - m) with m as its consumers read it;
//  MODE 4, the statistics online, one pass (blocked.py:293-346): a running
//  max per thread, its sum rescaled by exp(m_old - m_new) when it moves;
//  MODE 2, deslice forward (blocked.py:466-510): out = sum_g e tok / l;
//  MODE 1, slice backward (blocked.py:577-673), and MODE 0, deslice backward
//  (blocked.py:745-815): pass 1 forms the row sum l = sum_g e, delta =
//  sum_g e dw / l (and, slice, dfx = sum_g e dz / l); pass 2 forms dl =
//  (e dw - e delta) / l, dx = sum_g dl W / tau and the row's temperature
//  term sum_g dl (logit - m), over all of G before it meets other rows.
// logits = x W^T and dw = v M^T (+ ds) on the tensor cores with W and M in
// two bf16 parts (x and v are bf16): within 2^-17 of the fp32 products, and
// the very products the slot-owning kernels form; the value dots round e,
// dl, tok, dz and W to bf16 (the bf16 dot mode, blocked.py). delta and l go
// to the slot-owning kernels through p.delta.
// Two threads per point row (32 slots each). Two CTAs per SM, so that one's
// MMAs run while the other forms its rows.
// smem: [image x 2][x tile][v tile][e / dl tile][row exchange][bars]
// TMEM: logits 0, dw 64, the value accumulator (dfx or out, then dx) 128.
constexpr int kPnIm = 25 * 1024;  // one image buffer (im_bytes(64) rounded up)
constexpr int kPnX = 2 * kPnIm, kPnV = kPnX + 8192, kPnE = kPnV + 16384,
              kPnRed = kPnE + 16384, kPnBar = kPnRed + 2048, kPnBytes = kPnBar + kBarBytes;
static_assert(im_bytes(64) <= kPnIm && kPnX % 1024 == 0 && kPnE % 1024 == 0,
              "point-owning layout");

template <int MODE>
__global__ void __launch_bounds__(256, 2) k_tc_blk_pown_bf16(const __grid_constant__ TcParams p) {
  constexpr bool BWD = MODE <= 1, SLICE = MODE == 1, STATS = MODE == 3, ONLINE = MODE == 4;
  constexpr int NPASS = MODE == 2 || ONLINE ? 1 : 2;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H, DV = p.dv, N = p.N;
  const int nblk = p.G / kPnSlots, mp = im_mpart(DV);
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kPnBar, p.wait_ns);
  prologue_end(c);
  const float inv_tau = __frcp_rn(p.tau[h]);
  const float scale = inv_tau * kLog2e;
  const uint32_t tL = c.tmem, tD = c.tmem + 64, tA = c.tmem + 128;
  const int warp = threadIdx.x >> 5, row = 32 * (warp & 3) + (threadIdx.x & 31), half = warp >> 2;
  const uint32_t tlane = (uint32_t)(32 * (warp & 3)) << 16;
  const uint8_t* img_bh = p.img + (int64_t)bh * nblk * im_bytes(DV);
  // the deslice forward reads W and M's hi part only, the statistics W only
  const uint32_t im_copy = BWD ? (uint32_t)im_bytes(DV)
                           : STATS || ONLINE ? (uint32_t)kImM : (uint32_t)(kImM + mp);
  const uint32_t stage_b = (uint32_t)(BWD ? 4 + DV / 8 : 4) * 2048;
  uint8_t* const xs = sm + kPnX;
  uint8_t* const vs = sm + kPnV;
  uint8_t* const et = sm + kPnE;
  float* const red = (float*)(sm + kPnRed);
  uint8_t* const etrow = et + (row >> 3) * 1024 + (row & 7) * 16;
  auto load_tile = [&](int tile) {  // x (4 boxes) and, backward, v (DV / 8 boxes)
    mbar_arrive_expect_tx(c.bar + kBarTma, stage_b);
    for (int i = 0; i < 4; ++i)
      tma_load_4d(xs + i * 2048, &p.mx, 8 * i, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    if (BWD)
      for (int i = 0; i < DV / 8; ++i)
        tma_load_4d(vs + i * 2048, &p.mv, 8 * i, h, sp.row(tile), sp.bc, c.bar + kBarTma);
  };
  auto load_image = [&](int q, int j) {  // block-pass q walks slot block j
    uint64_t* bar = c.bar + kG3 + (q & 1);
    mbar_arrive_expect_tx(bar, im_copy);
    bulk_load(sm + (q & 1) * kPnIm, img_bh + (int64_t)j * im_bytes(DV), im_copy, bar);
  };
  const uint32_t id_l = idesc_bf16(128, kPnSlots, 0, 0);
  const uint32_t id_a = idesc_bf16(128, DV == 64 ? 64 : 32, 0, 1), id_x = idesc_bf16(128, 32, 0, 1);
  const int n_my = sp.ntiles > (int)blockIdx.x ? (sp.ntiles - 1 - (int)blockIdx.x) / p.P + 1 : 0;
  const int nq = n_my * NPASS * nblk;
  if (c.issuer() && nq > 0) {
    load_tile(blockIdx.x);
    load_image(0, 0);
  }
  float dt_acc = 0.f;
  bool v_pending = false;  // value MMAs committed on kG2 and not yet waited for
  int q = 0;
  for (int k = 0; k < n_my; ++k) {
    const int tile = blockIdx.x + k * p.P;
    const int n = tile * kTile + row;
    const bool valid = n < sp.N;
    const int64_t ni = sp.n0 + n;
    const int64_t sbase = (int64_t)bh * 2 * N;
    float m2 = 0.f, inv_l = 0.f, delta = 0.f;
    if (valid && !STATS && !ONLINE) {
      m2 = p.stats_in[sbase + ni] * kLog2e;
      if (!BWD) inv_l = __frcp_rn(p.stats_in[sbase + N + ni]);
    }
    wait_bar(c, kBarTma, p.status);
    for (int pass = 0; pass < NPASS; ++pass) {
      // backward pass 0: row sum and sum e dw; pass 1: the temperature term;
      // statistics pass 0: row max (m2 = 0), pass 1: row sum
      // online statistics: running max acc_u (log2 units) and its sum acc_l
      float acc_l = STATS && pass == 0 ? -INFINITY : 0.f, acc_u = ONLINE ? -INFINITY : 0.f;
      const bool value_mma = MODE == 2 || SLICE || (BWD && pass == 1);
      for (int j = 0; j < nblk; ++j, ++q) {
        const uint8_t* im = sm + (q & 1) * kPnIm;
        // constant barrier indices keep the phase bits in registers
        if (q & 1)
          wait_bar(c, kG4, p.status);
        else
          wait_bar(c, kG3, p.status);
        if (c.issuer()) {
          // logits = x W^T and dw = v M^T, the small parts first
          for (int part = 0; part < 2; ++part)  // W mid, hi
            for (int ks = 0; ks < 2; ++ks)
              mma_bf16(tL, smem_desc(smem_u32(xs) + ks * 4096, 2048, 128),
                       smem_desc(smem_u32(im + kImW + part * 4096) + ks * 256, 128, 512), id_l,
                       (part | ks) != 0);
          if (BWD)
            for (int pi = 0; pi < 2; ++pi)  // M mid, hi
              for (int ks = 0; ks < DV / 16; ++ks)
                mma_bf16(tD, smem_desc(smem_u32(vs) + ks * 4096, 2048, 128),
                         smem_desc(smem_u32(im + kImM + (1 - pi) * mp) + ks * 256, 128, DV * 16),
                         id_l, (pi | ks) != 0);
          commit(c, kG1);
        }
        if (v_pending) {  // block-pass q - 1's value MMAs: the e tile and its image buffer free
          wait_bar(c, kG2, p.status);
          v_pending = false;
        }
        if (c.issuer() && q + 1 < nq) load_image(q + 1, j + 1 < nblk ? j + 1 : 0);
        wait_bar(c, kG1, p.status);
        // The tile's last products have read x and v: fetch the next tile's.
        // Every thread must have waited for this tile's phase of the TMA
        // barrier first (else a lagging thread would see it two phases on):
        // the barrier of the tile's first block-pass guarantees it (nblk >= 2).
        if (c.issuer() && j == nblk - 1 && pass == NPASS - 1 && k + 1 < n_my)
          load_tile(tile + p.P);
        const float* bias2 = (const float*)(im + kImBias);
        const float* dss = (const float*)(im + kImDs);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {  // this thread's 32 slots, 16 at a time
          const int c0 = half * 32 + ch * 16;
          uint32_t lr[16], dr[16];
          tld<16>(tL + tlane + c0, lr);
          if (BWD) tld<16>(tD + tlane + c0, dr);
          tld_wait();
          float va[16], vb[16];
          uint32_t e2[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            float ov[2];
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              const int i = 2 * jj + s2, g = c0 + i;
              const float t2 = __uint_as_float(lr[i]) * scale + bias2[g] - m2;
              const float e = valid ? ex2(t2) : 0.f;
              if (BWD) {
                float dwg = __uint_as_float(dr[i]);
                if (SLICE) dwg += dss[g];
                if (pass == 0) {
                  va[i] = e;
                  vb[i] = e * dwg;
                  ov[s2] = e;
                } else {
                  const float dl = (e * dwg - e * delta) * inv_l;
                  vb[i] = dl * t2;
                  ov[s2] = dl;
                }
              } else if (STATS) {
                va[i] = pass == 0 ? t2 : e;
              } else if (ONLINE) {
                va[i] = t2;
              } else {
                ov[s2] = e;
              }
            }
            e2[jj] = bf2_bits(__floats2bfloat162_rn(ov[0], ov[1]));
          }
          if (BWD) {
            if (pass == 0) acc_l += tree_sum2(va);
            acc_u += tree_sum2(vb);
          }
          if (ONLINE) {
            float bm = va[0];
#pragma unroll
            for (int i = 1; i < 16; ++i) bm = fmaxf(bm, va[i]);
            const float mn = fmaxf(acc_u, bm);
#pragma unroll
            for (int i = 0; i < 16; ++i) va[i] = ex2(va[i] - mn);
            acc_l = acc_l * ex2(acc_u - mn) + tree_sum2(va);
            acc_u = mn;
          }
          if (STATS) {
            if (pass == 0) {
#pragma unroll
              for (int i = 0; i < 16; ++i) acc_l = fmaxf(acc_l, va[i]);
            } else {
              acc_l += tree_sum2(va);
            }
          }
          if (value_mma) {
#pragma unroll
            for (int i4 = 0; i4 < 2; ++i4)  // slots c0 + 8 i4 .. + 7: one 16-byte chunk
              *(uint4*)(etrow + ((c0 >> 3) + i4) * 128) =
                  make_uint4(e2[4 * i4], e2[4 * i4 + 1], e2[4 * i4 + 2], e2[4 * i4 + 3]);
          }
        }
        to_async_barrier();
        if (value_mma) {
          if (c.issuer()) {
            if (BWD && pass == 1) {  // dx += dl W (W hi, MN-major)
              for (int ks = 0; ks < 4; ++ks)
                mma_bf16(tA, smem_desc(smem_u32(et) + ks * 256, 128, 1024),
                         smem_desc(smem_u32(im + kImW + 4096) + ks * 1024, 512, 128), id_x,
                         (j | ks) != 0);
            } else {  // dfx += e dz or out += e tok (M hi, MN-major)
              for (int ks = 0; ks < 4; ++ks)
                mma_bf16(tA, smem_desc(smem_u32(et) + ks * 256, 128, 1024),
                         smem_desc(smem_u32(im + kImM) + ks * 2 * DV * 16, DV * 16, 128), id_a,
                         (j | ks) != 0);
            }
            commit(c, kG2);
          }
          v_pending = true;
        }
      }
      // ---- end of a pass
      if (ONLINE) {
        red[half * 128 + row] = acc_u;
        red[256 + half * 128 + row] = acc_l;
        __syncthreads();
        if (half == 0 && valid) {
          const float ma = red[row], mb = red[128 + row], mx = fmaxf(ma, mb);
          // m in the logits' units; l taken to m on the log2 scale as its
          // readers form it (m log2(e), a rounding away from mx)
          const float m = mx * kLn2, mr = m * kLog2e;
          const float l = red[256 + row] * ex2(ma - mr) + red[384 + row] * ex2(mb - mr);
          p.stats_out[sbase + ni] = m;
          p.stats_out[sbase + N + ni] = l;
        }
      }
      if (STATS) {
        red[half * 128 + row] = acc_l;
        __syncthreads();
        if (pass == 0) {
          // m in the logits' units, and on the log2 scale as its readers form it
          const float m = fmaxf(red[row], red[128 + row]) * kLn2;
          m2 = m * kLog2e;
          if (half == 0 && valid) p.stats_out[sbase + ni] = m;
        } else if (half == 0 && valid) {
          p.stats_out[sbase + N + ni] = red[row] + red[128 + row];
        }
      }
      if (BWD) {
        red[(0 + half) * 128 + row] = acc_l;
        red[(2 + half) * 128 + row] = acc_u;
        __syncthreads();
        if (pass == 0) {
          const float lrow = red[row] + red[128 + row];
          const float sdw = red[256 + row] + red[384 + row];
          inv_l = valid ? __frcp_rn(lrow) : 0.f;
          delta = sdw * inv_l;
          if (half == 0 && valid) {
            p.delta[sbase + ni] = delta;
            p.delta[sbase + N + ni] = lrow;
          }
        } else if (half == 0 && valid) {
          dt_acc += red[256 + row] + red[384 + row];
        }
      }
      const bool store = MODE == 2 || (BWD && (SLICE || pass == 1));
      if (store) {
        if (v_pending) {
          wait_bar(c, kG2, p.status);
          v_pending = false;
        }
        // dx (16 columns a thread), dfx or out (DV / 2), 16 columns a read
        const bool dxo = BWD && pass == 1;
        const int w = dxo ? 16 : DV / 2, col = half * w;
        const float f = dxo ? inv_tau : inv_l;
        __nv_bfloat16* dst =
            dxo || !SLICE
                ? (__nv_bfloat16*)p.out + sp.bc * p.so[0] + ni * p.so[1] + h * p.so[2] + col
                : (__nv_bfloat16*)p.out2 + sp.bc * p.so2[0] + ni * p.so2[1] + h * p.so2[2] + col;
        for (int c16 = 0; c16 < w; c16 += 16) {
          uint32_t r[16];
          tld<16>(tA + tlane + col + c16, r);
          tld_wait();
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            o[i] = bf2_bits(__floats2bfloat162_rn(__uint_as_float(r[2 * i]) * f,
                                                  __uint_as_float(r[2 * i + 1]) * f));
          if (valid) {
            *(uint4*)(dst + c16) = make_uint4(o[0], o[1], o[2], o[3]);
            *(uint4*)(dst + c16 + 8) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        // the next MMAs into these columns follow a barrier after these reads
      }
    }
  }
  if (v_pending) wait_bar(c, kG2, p.status);
  if (BWD) {
    const float tot = cta_sum_nt<256>(dt_acc, red);
    if (threadIdx.x == 0) p.partDt[(int64_t)bh * p.P + blockIdx.x] = -inv_tau * tot * kLn2;
  }
  epilogue<256>(c);
}

// ------------------------------------------------------------ G = 64
// The single-tile family at G = 64 with D = DV = 32 (config 5's shape): the
// same exact three-part products as the G = 32 kernels above, with the 64
// slots of a row split over its two threads (thread cs owns slots
// [32 cs, 32 cs + 32)). Point tensors still have 32 values a row, so the
// point operands (x, fx, d_out) are split and staged exactly as at G = 32.
//  * logits = x W^T with W's three parts of 64 rows (K-major, +0, +4096,
//    +8192): the NW = 64 schedule with N = 128 ([x W_mid | x W_hi]), eight
//    MMAs;
//  * pools are formed transposed, D[point-operand parts][slot parts]: the
//    point operand's parts stacked along M ([lo; mid; hi; ones], the ones
//    row giving the plain sums s or db), the slot operand's three parts of
//    64 slots stacked along N (N = 192): one MMA per 16 points, all nine
//    partial products; the threads drain each tile's pool into fp32
//    registers, adding the slot parts small first, and the point operand's
//    parts are added once, at the end.
constexpr int kRS4 = 2048;               // point split with a ones part: 8-row group stride
constexpr int kSplit4 = 16 * kRS4;       // 32 KB
constexpr int kRSW = 3072;               // 64-slot split, N-stacked: 8-row group stride
constexpr int kSplitW = 16 * kRSW;       // 48 KB
constexpr int kSmall64 = 3 * 4096;       // a 64 x 32 matrix, three K-major parts
constexpr uint32_t kIdPool64 = idesc_bf16(128, 192, 1, 1);

// A 64 x 32 fp32 matrix M (row-major) split into three K-major parts (rows
// r, k = c) at +0 (lo), +4096 (mid), +8192 (hi).
template <int NT>
__device__ __forceinline__ void put_small64(uint8_t* dst, const float* M) {
  for (int i = threadIdx.x; i < 64 * 32; i += NT) {
    const int r = i >> 5, c = i & 31;
    __nv_bfloat16 h, m, l;
    split3(M[i], h, m, l);
    const uint32_t o = kmajor_off(r, c, 32);
    *(__nv_bfloat16*)(dst + o) = l;
    *(__nv_bfloat16*)(dst + 4096 + o) = m;
    *(__nv_bfloat16*)(dst + 8192 + o) = h;
  }
}

// Per-head row constants for 64 slots (bias2 holds 64 floats).
template <int NT>
__device__ __forceinline__ RowConst row_const64(float* bias_s, const float* bias, float tau) {
  const float scale = __frcp_rn(tau) * kLog2e;
  if (threadIdx.x < 64) bias_s[threadIdx.x] = bias[threadIdx.x] * scale;
  return RowConst{scale, bias_s};
}

// D (128 x 128) = [x W_mid | x W_hi], A = the point operand in TMEM at a
// (parts lo, mid, hi at +0, +16, +32 columns, K = 32), bd = the 64-row
// small operand: A lo and mid times [W_mid | W_hi], A hi times W_lo into
// the W_mid group, A hi times [W_mid | W_hi] -- seven of the nine partial
// products (the two left out are below 2^-26 of the result), small first.
// (AHI: the point operand has only a hi part, bf16 points: hi x [W_mid |
// W_hi] first, which sets all 128 columns, then hi x W_lo.)
template <bool AHI = false>
__device__ __forceinline__ void logits64(uint32_t d, uint32_t a, uint64_t bd) {
  constexpr uint32_t id128 = idesc_bf16(128, 128, 0, 0), id64 = idesc_bf16(128, 64, 0, 0);
  if constexpr (AHI) {
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_ts(d, a + 32 + ks * 8, bd + ((4096 + ks * 256) >> 4), id128, ks != 0);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_ts(d, a + 32 + ks * 8, bd + ((ks * 256) >> 4), id64, true);
  } else {
#pragma unroll
    for (int pa = 0; pa < 2; ++pa)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a + pa * 16 + ks * 8, bd + ((4096 + ks * 256) >> 4), id128, (pa | ks) != 0);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_ts(d, a + 32 + ks * 8, bd + ((ks * 256) >> 4), id64, true);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_ts(d, a + 32 + ks * 8, bd + ((4096 + ks * 256) >> 4), id128, true);
  }
}

// This thread's CG logits (slots CG cs ..) from the [W_mid | W_hi] groups.
template <int CG>
__device__ __forceinline__ void ld_logits64(uint32_t taddr, int cs, float (&v)[CG]) {
#pragma unroll
  for (int hf = 0; hf < CG / 16; ++hf) {
    uint32_t a[16], b[16];
    tld<16>(taddr + CG * cs + 16 * hf, a);
    tld<16>(taddr + 64 + CG * cs + 16 * hf, b);
    tld_wait();
#pragma unroll
    for (int k = 0; k < 8; ++k)
      put2(v, 8 * hf + k,
           __fadd2_rn(make_float2(__uint_as_float(a[2 * k]), __uint_as_float(a[2 * k + 1])),
                      make_float2(__uint_as_float(b[2 * k]), __uint_as_float(b[2 * k + 1]))));
  }
}

// A point row's C values (columns C cs ..) split into a stacked buffer
// with a ones part: per 8-row group lo, mid, hi, ones at +0, +512, +1024,
// +1536 (the M-stacked operand [lo; mid; hi; ones] of a transposed pool).
template <int C>
__device__ __forceinline__ void split_to_smem4(const Split<C>& sp, uint8_t* buf, int row, int cs) {
  uint8_t* base = buf + (row >> 3) * kRS4 + (row & 7) * 16;
  const uint4 ones = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
#pragma unroll
  for (int i = 0; i < C / 8; ++i) {
    const int j = (C / 8) * cs + i;
    *(uint4*)(base + j * 128) = make_uint4(sp.lw[4 * i], sp.lw[4 * i + 1], sp.lw[4 * i + 2], sp.lw[4 * i + 3]);
    *(uint4*)(base + 512 + j * 128) = make_uint4(sp.mw[4 * i], sp.mw[4 * i + 1], sp.mw[4 * i + 2], sp.mw[4 * i + 3]);
    *(uint4*)(base + 1024 + j * 128) = make_uint4(sp.hw[4 * i], sp.hw[4 * i + 1], sp.hw[4 * i + 2], sp.hw[4 * i + 3]);
    *(uint4*)(base + 1536 + j * 128) = ones;
  }
}

// A row's CG slot values (slots CG cs ..) split into the N-stacked 64-slot
// buffer: per 8-row group the lo, mid, hi parts of the 64 slots (128 bytes
// each, 8 core matrices) at +0, +1024, +2048.
template <int CG>
__device__ __forceinline__ void split_to_smemw(const Split<CG>& sp, uint8_t* buf, int row, int cs) {
  uint8_t* base = buf + (row >> 3) * kRSW + (row & 7) * 16;
#pragma unroll
  for (int i = 0; i < CG / 8; ++i) {
    const int j = (CG / 8) * cs + i;
    *(uint4*)(base + j * 128) = make_uint4(sp.lw[4 * i], sp.lw[4 * i + 1], sp.lw[4 * i + 2], sp.lw[4 * i + 3]);
    *(uint4*)(base + 1024 + j * 128) = make_uint4(sp.mw[4 * i], sp.mw[4 * i + 1], sp.mw[4 * i + 2], sp.mw[4 * i + 3]);
    *(uint4*)(base + 2048 + j * 128) = make_uint4(sp.hw[4 * i], sp.hw[4 * i + 1], sp.hw[4 * i + 2], sp.hw[4 * i + 3]);
  }
}

// D (128 x 192) = transposed pool over the tile's points: A = the stacked
// point buffer with a ones part (M-stacked), B = the N-stacked 64-slot
// buffer; eight K steps of 16 points.
__device__ __forceinline__ void mma_pool64(uint32_t d, const uint8_t* a, const uint8_t* b) {
  const uint64_t ad = smem_desc(smem_u32(a), kRS4, 128), bd = smem_desc(smem_u32(b), kRSW, 128);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
    mma_bf16(d, ad + ((ks * 2 * kRS4) >> 4), bd + ((ks * 2 * kRSW) >> 4), kIdPool64, ks > 0);
}

// Add this thread's CG columns of its pool row (slots CG cs .. of the slot
// parts lo, mid, hi, small first) into acc.
template <int CG>
__device__ __forceinline__ void drain_pool64(uint32_t taddr, int cs, float (&acc)[CG]) {
#pragma unroll
  for (int hf = 0; hf < CG / 16; ++hf) {
    uint32_t a[16], b[16], c[16];
    tld<16>(taddr + CG * cs + 16 * hf, a);
    tld<16>(taddr + 64 + CG * cs + 16 * hf, b);
    tld<16>(taddr + 128 + CG * cs + 16 * hf, c);
    tld_wait();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 s = __fadd2_rn(
          __fadd2_rn(make_float2(__uint_as_float(a[2 * k]), __uint_as_float(a[2 * k + 1])),
                     make_float2(__uint_as_float(b[2 * k]), __uint_as_float(b[2 * k + 1]))),
          make_float2(__uint_as_float(c[2 * k]), __uint_as_float(c[2 * k + 1])));
      put2(acc, 8 * hf + k, __fadd2_rn(f2(acc, 8 * hf + k), s));
    }
  }
}

// Transposed pool partials: thread (q, cs) with TMEM lane 32 q + t holds,
// for point-operand part q (q = 3: the ones row) and value t, its sums over
// slots CG cs + i. Writes part[g][c] = (lo + mid) + hi for the 64 x 32
// partial, and the plain sums (ones row) into sums[g] when sums is given;
// xch holds 3 x 32 x 65 floats.
template <int T>
__device__ __forceinline__ void pool64_write(float* xch, const float (&acc)[64 / T], float* part,
                                             float* sums, const Th<T>& th) {
  constexpr int CG = 64 / T;
  const int t = threadIdx.x & 31;
  __syncthreads();
  if (th.q < 3) {
#pragma unroll
    for (int i = 0; i < CG; ++i) xch[(th.q * 32 + t) * 65 + CG * th.cs + i] = acc[i];
  } else if (sums && t == 0) {
#pragma unroll
    for (int i = 0; i < CG; ++i) sums[CG * th.cs + i] = acc[i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 32; i += Th<T>::NT) {
    const int g = i >> 5, c = i & 31;
    part[i] = (xch[c * 65 + g] + xch[(32 + c) * 65 + g]) + xch[(64 + c) * 65 + g];
  }
}

// ------------------------------------------------------------ slice forward, G = 64
// One CTA of 256 threads (two per point row), two CTAs per SM.
// smem: [stage x][F: fx staged, then its split with a ones part][WS: w, 64
//       slots][W][bias][red][bars]
// TMEM (256 columns): logits at 0 (128), the z pool at 0 (192, once the
// logits are read), the x point operand at 192.
// x and fx arrive on barriers of their own (kBarTma, kG3). A tile's x is
// split and its logits issued at the end of the previous tile (once that
// tile's pool is drained out of the columns the logits take), so the fx
// split runs under the logits MMAs, and the next fx -- which can load only
// once the pool is done with F -- has the drain and the x split to land.
constexpr int kS6StageX = 0, kS6F = kStage, kS6WS = kS6F + kSplit4, kS6Ws = kS6WS + kSplitW,
              kS6Bias = kS6Ws + kSmall64, kS6Red = kS6Bias + 256,
              kS6Bar = kS6Red + red_bytes(2, 2), kS6Bytes = kS6Bar + kBarBytes;
static_assert(kS6F % 1024 == 0, "fx staging tile needs 1 KB alignment");

template <typename PT>
__global__ void __launch_bounds__(256, 2) k_tc_slice_fwd64(const __grid_constant__ TcParams p) {
  constexpr int T = 2, NT = 256;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kS6Bar, p.wait_ns);
  float* red = (float*)(sm + kS6Red);
  put_small64<NT>(sm + kS6Ws, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  const RowConst rc = row_const64<NT>((float*)(sm + kS6Bias),
                                      p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tP = c.tmem, tX = c.tmem + 192;
  const uint64_t dWs = desc_smallK(sm + kS6Ws);
  uint8_t* stX = sm + kS6StageX;
  uint8_t* F = sm + kS6F;
  uint8_t* WS = sm + kS6WS;
  float acc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.f;
  auto load_x = [&](int t) {  // one thread
    mbar_arrive_expect_tx(c.bar + kBarTma, stage_bytes<PT>());
    tma_load_4d(stX, &p.mx, 0, h, sp.row(t), sp.bc, c.bar + kBarTma);
  };
  auto load_f = [&](int t) {  // one thread
    mbar_arrive_expect_tx(c.bar + kG3, stage_bytes<PT>());
    tma_load_4d(F, &p.mv, 0, h, sp.row(t), sp.bc, c.bar + kG3);
  };
  // tile t's x into the TMEM operand and its logits issued; the barrier
  // also orders the last drain of the pool before the logits overwrite it,
  // and every read of the x stage before the next x loads into it
  auto x_phase = [&](int t) {
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<16, PT> x;
      x.load(stX, th.row, th.cs);
      x.split().to_tmem(tX + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      if (t + p.P < sp.ntiles) load_x(t + p.P);
      logits64<kHi<PT>>(tL, tX, dWs);
      commit(c, kG1);
    }
  };
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles) {
    load_x(tile);
    load_f(tile);
  }
  if (tile < sp.ntiles) x_phase(tile);
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool more = tile + p.P < sp.ntiles;
    wait_bar(c, kG3, p.status);
    {
      RowVals<16, PT> f;
      f.load(F, th.row, th.cs);
      __syncthreads();  // every staged fx row is in registers before F is overwritten
      split_to_smem4(f.split(), F, th.row, th.cs);
    }
    wait_bar(c, kG1, p.status);
    {
      float lg[32];
      ld_logits64(tL + th.lane_off, th.cs, lg);
      softmax_fwd<T, 32>(lg, rc, n0 + th.row < sp.N, red, th);
      split_to_smemw(Split<32>(lg), WS, th.row, th.cs);
    }
    to_async_barrier();  // the F and WS splits, and the logits read out
    if (c.issuer()) {
      mma_pool64(tP, F, WS);  // [fx; 1]^T w
      commit(c, kG2);
    }
    wait_bar(c, kG2, p.status);
    if (c.issuer() && more) load_f(tile + p.P);  // F is free once the pool is done
    drain_pool64(tP + th.lane_off, th.cs, acc);
    if (more) x_phase(tile + p.P);
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  tc_fence_before();
  pool64_write((float*)WS, acc, p.partA + slot * 64 * 32, p.partS + slot * 64, th);
  epilogue<256>(c);
}

// ------------------------------------------------------------ deslice forward, G = 64
// The 64-slot tokens as the N-stacked MN-major operand of out = w tokens
// (K = 64 slots, in 8-row groups of 1536 bytes, parts at +0, +512, +1024).
template <int NT>
__device__ __forceinline__ void put_small_stacked64(uint8_t* dst, const float* M) {
  for (int i = threadIdx.x; i < 64 * 32; i += NT) {
    const int r = i >> 5, c = i & 31;
    __nv_bfloat16 h, m, l;
    split3(M[i], h, m, l);
    const uint32_t o = (r >> 3) * kRS + (r & 7) * 16 + (c >> 3) * 128 + (c & 7) * 2;
    *(__nv_bfloat16*)(dst + o) = l;
    *(__nv_bfloat16*)(dst + 512 + o) = m;
    *(__nv_bfloat16*)(dst + 1024 + o) = h;
  }
}

// A row's CG slot values (slots CG cs ..) as this thread's part of a K = 64
// point operand in TMEM: parts lo, mid, hi at +0, +32, +64 columns, two bf16
// per column (even slot low), the thread's CG / 2 columns at (CG / 2) cs.
template <int CG>
__device__ __forceinline__ void split_to_tmem64(const Split<CG>& sp, uint32_t taddr, int cs) {
  const uint32_t a = taddr + (CG / 2) * cs;
  tst<CG / 2>(a, sp.lw);
  tst<CG / 2>(a + 32, sp.mw);
  tst<CG / 2>(a + 64, sp.hw);
}

// D (128 x 96) = A B^T with A = a K = 64 point operand in TMEM (parts at
// +0, +32, +64) and B = an N-stacked MN-major 64-row operand at bd: twelve
// MMAs, A parts lo, mid, hi one after the other (all nine partial products).
__device__ __forceinline__ void wide64_mn96(uint32_t d, uint32_t a, uint64_t bd) {
  constexpr uint32_t id = idesc_bf16(128, 96, 0, 1);
#pragma unroll
  for (int pa = 0; pa < 3; ++pa)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      mma_ts(d, a + pa * 32 + ks * 8, bd + ((ks * 2 * kRS) >> 4), id, (pa | ks) != 0);
}

// smem: [stage x, two tiles][W][tokens][bias][red][bars]
// TMEM (256 columns): logits at 0 (128), out at 0 (96, once the logits are
// read), the x operand at 128 (48) and then the w operand at 128 (96).
// Two x stages: the tile after next loads while this one is worked on.
constexpr int kD6Stage = 0, kD6Ws = 2 * kStage, kD6Ts = kD6Ws + kSmall64,
              kD6Bias = kD6Ts + 8 * kRS, kD6Red = kD6Bias + 256,
              kD6Bar = kD6Red + red_bytes(2, 2), kD6Bytes = kD6Bar + kBarBytes;

template <typename PT>
__global__ void __launch_bounds__(256, 2) k_tc_deslice_fwd64(const __grid_constant__ TcParams p) {
  constexpr int T = 2, NT = 256;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<256>(sm, kD6Bar, p.wait_ns);
  float* red = (float*)(sm + kD6Red);
  put_small64<NT>(sm + kD6Ws, p.W + (int64_t)b * p.swb + (int64_t)h * p.swh);
  put_small_stacked64<NT>(sm + kD6Ts, p.M + (int64_t)bh * 64 * 32);
  const RowConst rc = row_const64<NT>((float*)(sm + kD6Bias),
                                      p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tO = c.tmem, tX = c.tmem + 128, tA = c.tmem + 128;
  const uint64_t dWs = desc_smallK(sm + kD6Ws), dTs = desc_stacked(sm + kD6Ts);
  auto stage = [&](int k) { return sm + kD6Stage + (k & 1) * kStage; };
  // stage k & 1 completes on barrier kBarTma (even) or kG3 (odd)
  auto sbar = [&](int k) { return (k & 1) ? kG3 : kBarTma; };
  const int n_my = sp.ntiles > (int)blockIdx.x ? (sp.ntiles - 1 - (int)blockIdx.x) / p.P + 1 : 0;
  if (c.issuer()) {
    for (int k = 0; k < 2 && k < n_my; ++k)
      tma_tile<PT>(p, stage(k), nullptr, h, sp, blockIdx.x + k * p.P, c.bar + sbar(k));
  }
  for (int k = 0; k < n_my; ++k) {
    const int tile = blockIdx.x + k * p.P, n0 = tile * kTile;
    wait_bar(c, sbar(k), p.status);
    RowVals<16, PT> x;
    x.load(stage(k), th.row, th.cs);
    // the last tile's out is read out of TMEM before the logits overwrite it
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    x.split().to_tmem(tX + th.lane_off, th.cs);
    tst_wait();
    to_async_barrier();
    if (c.issuer()) {
      if (k + 2 < n_my)  // stage k & 1 is consumed: the tile after next
        tma_tile<PT>(p, stage(k), nullptr, h, sp, tile + 2 * p.P, c.bar + sbar(k));
      logits64<kHi<PT>>(tL, tX, dWs);
      commit(c, kG1);
    }
    wait_bar(c, kG1, p.status);
    {
      float lg[32];
      ld_logits64(tL + th.lane_off, th.cs, lg);
      softmax_fwd<T, 32>(lg, rc, true, red, th);
      split_to_tmem64(Split<32>(lg), tA + th.lane_off, th.cs);  // over the consumed x operand
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide64_mn96(tO, tA, dTs);  // out = w tokens, over the consumed logits
      commit(c, kG2);
    }
    wait_bar(c, kG2, p.status);
    store_result<96, 16>(tO, th.q, th.cs,
                         (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                             (int64_t)h * p.so[2],
                         p.so[1], sp.N - n0);
  }
  epilogue<256>(c);
}

// ------------------------------------------------------------ coupled backward, G = 64
// The tied backward of a round (as k_tc_coupled_bwd) at 64 slots: one CTA
// of 256 threads per SM with all 512 TMEM columns; the phases of a tile run
// in turn, the next tile's point tiles loading meanwhile.
//  A: logits = x W^T (x split in shared memory, K-major view), dw = d_out
//     tok^T + fx dz_num^T (point operands in TMEM), each N = 128;
//  threads: softmax Jacobian -> w, dl/tau;
//  B1: dfx = w dz_num and dx = (dl/tau) W (K = 64 slots, w and dl/tau in
//      TMEM, dz_num and W as N-stacked MN-major operands), N = 96 each;
//  B2: the transposed pool [x; 1]^T (dl/tau) -> dW and db (N = 192), formed
//      while the threads store dfx and dx.
// smem: [stage x][stage fx][stage d_out][XS: x split + ones][US: dl/tau,
//       64 slots][W K-major][W stacked][tokens K-major][dz K-major]
//       [dz stacked][bias][ds][red][bars]
// TMEM (512 columns): A: logits 0, dw 128, fx 256, d_out 304; B1: dfx 0,
// dx 96, dl/tau 256, w 352; B2: pool 192 (over the consumed B1 operands).
constexpr int kC6StX = 0, kC6StF = kStage, kC6StO = 2 * kStage, kC6XS = 3 * kStage,
              kC6US = kC6XS + kSplit4, kC6Wk = kC6US + kSplitW, kC6Wm = kC6Wk + kSmall64,
              kC6Tk = kC6Wm + 8 * kRS, kC6Zk = kC6Tk + kSmall64, kC6Zm = kC6Zk + kSmall64,
              kC6Bias = kC6Zm + 8 * kRS, kC6Ds = kC6Bias + 256, kC6Red = kC6Ds + 256;
#ifndef FS_TC_CB64_T
#define FS_TC_CB64_T 2
#endif
constexpr int kTCoupled64 = FS_TC_CB64_T;  // threads per point row
__host__ __device__ constexpr int c6_bar(int T) { return kC6Red + red_bytes(T, 3); }
__host__ __device__ constexpr int c6_bytes(int T) { return c6_bar(T) + kBarBytes; }
static_assert(kC6XS % 1024 == 0, "stage tiles need 1 KB alignment");

// logits64 with the point operand x in shared memory (the stacked buffer
// with a ones part, read K-major: part p at +512 p)
template <bool AHI = false>
__device__ __forceinline__ void logits64_ss(uint32_t d, const uint8_t* xs, uint64_t bd) {
  constexpr uint32_t id128 = idesc_bf16(128, 128, 0, 0), id64 = idesc_bf16(128, 64, 0, 0);
  auto ad = [&](int part, int ks) { return smem_desc(smem_u32(xs + 512 * part + 256 * ks), 128, kRS4); };
  if constexpr (AHI) {  // bf16 points: hi part only (as logits64)
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_bf16(d, ad(2, ks), bd + ((4096 + ks * 256) >> 4), id128, ks != 0);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_bf16(d, ad(2, ks), bd + ((ks * 256) >> 4), id64, true);
  } else {
#pragma unroll
    for (int pa = 0; pa < 2; ++pa)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_bf16(d, ad(pa, ks), bd + ((4096 + ks * 256) >> 4), id128, (pa | ks) != 0);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_bf16(d, ad(2, ks), bd + ((ks * 256) >> 4), id64, true);
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
      mma_bf16(d, ad(2, ks), bd + ((4096 + ks * 256) >> 4), id128, true);
  }
}

// D = A1 B1^T + A2 B2^T into one 128-column accumulator [. B_mid | . B_hi]
// (64-row small operands, point operands in TMEM, K = 32): the logits64
// schedule of both products, their partial products interleaved.
template <bool AHI = false>
__device__ __forceinline__ void wide64_pair(uint32_t d, uint32_t a1, uint64_t b1, uint32_t a2,
                                            uint64_t b2) {
  constexpr uint32_t id128 = idesc_bf16(128, 128, 0, 0), id64 = idesc_bf16(128, 64, 0, 0);
  const uint32_t a[2] = {a1, a2};
  const uint64_t b[2] = {b1, b2};
  if constexpr (AHI) {  // bf16 points: hi parts only (as logits64)
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((4096 + ks * 256) >> 4), id128, (s | ks) != 0);
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((ks * 256) >> 4), id64, true);
  } else {
#pragma unroll
    for (int pa = 0; pa < 2; ++pa)
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
          mma_ts(d, a[s] + pa * 16 + ks * 8, b[s] + ((4096 + ks * 256) >> 4), id128,
                 (pa | s | ks) != 0);
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((ks * 256) >> 4), id64, true);
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        mma_ts(d, a[s] + 32 + ks * 8, b[s] + ((4096 + ks * 256) >> 4), id128, true);
  }
}

template <typename PT, int T>
__global__ void __launch_bounds__(128 * T, 1) k_tc_coupled_bwd64(const __grid_constant__ TcParams p) {
  constexpr int NT = 128 * T, C = 32 / T, CG = 64 / T;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint8_t* sm = align_smem(sm_raw);
  const Th<T> th;
  const int bh = blockIdx.y, b = bh / p.H, h = bh - b * p.H;
  const Span sp = span_of(p, b);
  Ctl c = prologue_begin<512>(sm, c6_bar(T), p.wait_ns);
  float* ds_s = (float*)(sm + kC6Ds);
  float* red = (float*)(sm + kC6Red);
  const float* Wp = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;
  put_small64<NT>(sm + kC6Wk, Wp);
  put_small_stacked64<NT>(sm + kC6Wm, Wp);
  put_small64<NT>(sm + kC6Tk, p.M + (int64_t)bh * 64 * 32);
  put_small64<NT>(sm + kC6Zk, p.M2 + (int64_t)bh * 64 * 32);
  put_small_stacked64<NT>(sm + kC6Zm, p.M2 + (int64_t)bh * 64 * 32);
  const RowConst rc = row_const64<NT>((float*)(sm + kC6Bias),
                                      p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh, p.tau[h]);
  if (threadIdx.x < 64) ds_s[threadIdx.x] = p.ds[(int64_t)bh * 64 + threadIdx.x];
  const float inv_tau = __frcp_rn(p.tau[h]);
  prologue_end(c);
  const uint32_t tL = c.tmem, tD = c.tmem + 128, tF = c.tmem + 256, tO = c.tmem + 304;
  const uint32_t tDfx = c.tmem, tDx = c.tmem + 96, tU = c.tmem + 256, tW = c.tmem + 352,
                 tP = c.tmem + 192;
  const uint64_t dWk = desc_smallK(sm + kC6Wk), dWm = desc_stacked(sm + kC6Wm);
  const uint64_t dTk = desc_smallK(sm + kC6Tk), dZk = desc_smallK(sm + kC6Zk),
                 dZm = desc_stacked(sm + kC6Zm);
  uint8_t* XS = sm + kC6XS;
  uint8_t* US = sm + kC6US;
  auto load3 = [&](int tile) {  // one thread: x, fx, d_out of a tile
    mbar_arrive_expect_tx(c.bar + kBarTma, 3 * stage_bytes<PT>());
    tma_load_4d(sm + kC6StX, &p.mx, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    tma_load_4d(sm + kC6StF, &p.mv, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
    tma_load_4d(sm + kC6StO, &p.mo, 0, h, sp.row(tile), sp.bc, c.bar + kBarTma);
  };
  float acc[CG], dt_acc = 0.f;
#pragma unroll
  for (int i = 0; i < CG; ++i) acc[i] = 0.f;
  int tile = blockIdx.x;
  if (c.issuer() && tile < sp.ntiles) load3(tile);
  for (; tile < sp.ntiles; tile += p.P) {
    const int n0 = tile * kTile;
    const bool valid = n0 + th.row < sp.N;
    wait_bar(c, kBarTma, p.status);
    {
      RowVals<C, PT> x, f, o;
      x.load(sm + kC6StX, th.row, th.cs);
      f.load(sm + kC6StF, th.row, th.cs);
      o.load(sm + kC6StO, th.row, th.cs);
      // (the last tile's pool is read out of TMEM, and its reads of XS and
      // US are done, before anything here overwrites them)
      split_to_smem4(x.split(), XS, th.row, th.cs);
      f.split().to_tmem(tF + th.lane_off, th.cs);
      o.split().to_tmem(tO + th.lane_off, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      if (tile + p.P < sp.ntiles) load3(tile + p.P);  // the stages are consumed
      logits64_ss<kHi<PT>>(tL, XS, dWk);
      commit(c, kG1);
      wide64_pair<kHi<PT>>(tD, tO, dTk, tF, dZk);  // d_out tok^T + fx dz_num^T
      commit(c, kG2);
    }
    {
      float w[CG], dw[CG];
      wait_bar(c, kG1, p.status);
      ld_logits64(tL + th.lane_off, th.cs, w);
      wait_bar(c, kG2, p.status);
      ld_logits64(tD + th.lane_off, th.cs, dw);
      const float2* ds2 = (const float2*)(ds_s + CG * th.cs);
#pragma unroll
      for (int k = 0; k < CG / 2; ++k) put2(dw, k, __fadd2_rn(f2(dw, k), ds2[k]));
      const float rdt = softmax_bwd<T, CG>(w, dw, rc, inv_tau, valid, red, th);
      if (valid) dt_acc += rdt;
      split_to_tmem64(Split<CG>(w), tW + th.lane_off, th.cs);
      const Split<CG> us(dw);  // dl / tau
      split_to_tmem64(us, tU + th.lane_off, th.cs);
      split_to_smemw(us, US, th.row, th.cs);
      tst_wait();
    }
    to_async_barrier();
    if (c.issuer()) {
      wide64_mn96(tDfx, tW, dZm);  // dfx = w dz_num
      wide64_mn96(tDx, tU, dWm);   // dx = (dl/tau) W
      commit(c, kG3);
    }
    wait_bar(c, kG3, p.status);
    if (c.issuer()) {
      mma_pool64(tP, XS, US);  // [x; 1]^T (dl/tau): dW and db, over the consumed operands
      commit(c, kG4);
    }
    store_result<96, C>(tDfx, th.q, th.cs,
                        (PT*)p.out2 + (int64_t)sp.bc * p.so2[0] + (sp.n0 + n0) * p.so2[1] +
                            (int64_t)h * p.so2[2],
                        p.so2[1], sp.N - n0);
    store_result<96, C>(tDx, th.q, th.cs,
                        (PT*)p.out + (int64_t)sp.bc * p.so[0] + (sp.n0 + n0) * p.so[1] +
                            (int64_t)h * p.so[2],
                        p.so[1], sp.N - n0);
    wait_bar(c, kG4, p.status);
    drain_pool64(tP + th.lane_off, th.cs, acc);
    tc_fence_before();
    __syncthreads();  // the pool is read out; XS and US are free
    tc_fence_after();
  }
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  tc_fence_before();
  pool64_write((float*)US, acc, p.partA + slot * 64 * 32, p.partS + slot * 64, th);
  const float tot = cta_sum_nt<NT>(dt_acc, (float*)XS);
  if (threadIdx.x == 0) p.partDt[slot] = -inv_tau * kLn2 * tot;
  epilogue<512>(c);
}

// ------------------------------------------------------------ wait self-test
// One thread waits, with a limit of limit_ns, on an mbarrier that nothing
// arrives at: the bounded-wait path of the kernels (status word set, the
// kernel returns, the context stays usable), exercised without a fault.
__global__ void k_tc_wait_selftest(int* status, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait(&bar, 0, status, limit_ns);
  }
}

// ------------------------------------------------------------ host side

static __device__ int fs_tc_status_word;

// The status word's device address in the current context, looked up on
// every call (a host-only query): the address belongs to one context, so a
// cached one would go stale for a caller in another context or after a
// device reset, and nothing shared is written.
int* device_status() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, fs_tc_status_word) != cudaSuccess) return nullptr;
  return (int*)p;
}

bool make_point_map(CUtensorMap* map, const void* data, int64_t B, int64_t N, int64_t H,
                    const int64_t stride[4], int pdt, int width) {
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
  const int64_t es = pdt == 0 ? 4 : 2;
  if (stride[3] != 1 || ((uintptr_t)data & 15)) return false;
  for (int i = 0; i < 3; ++i)
    if (stride[i] <= 0 || (stride[i] * es) % 16 || stride[i] * es >= ((int64_t)1 << 40))
      return false;
  // The encoder is a driver call and needs a current context on this thread;
  // a thread that has made no runtime call yet (an autograd worker on its
  // first backward op) has none until the runtime binds the device's primary
  // context, which cudaSetDevice does.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return false;
  cuuint64_t dims[4] = {(cuuint64_t)width, (cuuint64_t)H, (cuuint64_t)N, (cuuint64_t)B};
  cuuint64_t gstr[3] = {(cuuint64_t)(stride[2] * es), (cuuint64_t)(stride[1] * es),
                        (cuuint64_t)(stride[0] * es)};
  cuuint32_t box[4] = {pdt == 2 ? 8u : 32u, 1, kTile, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // the encoder wants a 64-byte aligned map; do not rely on the caller's stack
  unsigned char raw[sizeof(CUtensorMap) + 64];
  CUtensorMap* aligned = (CUtensorMap*)(((uintptr_t)raw + 63) & ~(uintptr_t)63);
  // fp32 rows are 128 bytes (128B swizzle), bf16 rows 64 bytes (64B swizzle);
  // mode 2: bf16, 16-byte column boxes of 128 rows, no swizzle (one box lands
  // as 16 contiguous 8 x 16-byte core matrices)
  const CUresult r = encode(aligned,
                            pdt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            4, const_cast<void*>(data), dims, gstr, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE,
                            pdt == 0   ? CU_TENSOR_MAP_SWIZZLE_128B
                            : pdt == 1 ? CU_TENSOR_MAP_SWIZZLE_64B
                                       : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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
std::atomic<uint64_t> g_wait_limit_ns{0};

template <typename K>
static cudaError_t launch_tc(K kernel, int T, int bytes, const TcParams& p, cudaStream_t s) {
  const cudaError_t e = set_smem((const void*)kernel, bytes + kSmemPad);
  if (e != cudaSuccess) return e;
  kernel<<<dim3(p.P, p.B * p.H), 128 * T, bytes + kSmemPad, s>>>(p);
  return cudaSuccess;
}

template <typename PT>
static cudaError_t run_tc_t(TcKind k, const TcParams& p, cudaStream_t s) {
  switch (k) {
    case TcKind::SliceFwd: return launch_tc(k_tc_slice_fwd<PT>, kTSliceFwd, kSfBytes, p, s);
    case TcKind::DesliceFwd:
      return launch_tc(k_tc_deslice_fwd<PT>, kTDesliceFwd, kDfBytes, p, s);
    case TcKind::SliceBwd: return launch_tc(k_tc_slice_bwd<PT>, kTSliceBwd, kSbBytes, p, s);
    case TcKind::DesliceBwd:
      return launch_tc(k_tc_deslice_bwd<PT>, kTDesliceBwd, kDbBytes, p, s);
    case TcKind::CoupledBwd:
      return launch_tc(k_tc_coupled_bwd<PT>, kTCoupledBwd, kCbBytes, p, s);
    case TcKind::SliceFwd64: return launch_tc(k_tc_slice_fwd64<PT>, 2, kS6Bytes, p, s);
    case TcKind::DesliceFwd64: return launch_tc(k_tc_deslice_fwd64<PT>, 2, kD6Bytes, p, s);
    case TcKind::CoupledBwd64:
      return launch_tc(k_tc_coupled_bwd64<PT, kTCoupled64>, kTCoupled64, c6_bytes(kTCoupled64),
                       p, s);
    default: break;
  }
  return cudaErrorInvalidValue;
}

cudaError_t run_tc(TcKind k, const TcParams& p, cudaStream_t s) {
  cudaError_t e;
  if (k == TcKind::BlkSliceBwdG || k == TcKind::BlkDesliceBwdG) {
    const bool sl = k == TcKind::BlkSliceBwdG;
    const void* fn = sl ? (const void*)k_tc_blk_bwd_g_bf16<true> : (const void*)k_tc_blk_bwd_g_bf16<false>;
    e = set_smem(fn, kBbBytes + kSmemPad);
    if (e == cudaSuccess) {
      const dim3 grid(p.P, p.G / kBgSlots, p.B * p.H);
      if (sl)
        k_tc_blk_bwd_g_bf16<true><<<grid, 512, kBbBytes + kSmemPad, s>>>(p);
      else
        k_tc_blk_bwd_g_bf16<false><<<grid, 512, kBbBytes + kSmemPad, s>>>(p);
    }
  } else if (k == TcKind::BlkImage) {
    k_tc_blk_image<<<dim3(p.G / kPnSlots, p.B * p.H), 256, 0, s>>>(p);
    e = cudaSuccess;
  } else if (k == TcKind::BlkSliceBwdN || k == TcKind::BlkDesliceBwdN ||
             k == TcKind::BlkDesliceFwd || k == TcKind::BlkStats ||
             k == TcKind::BlkStatsOnline) {
    const int mode = k == TcKind::BlkDesliceBwdN ? 0
                     : k == TcKind::BlkSliceBwdN ? 1
                     : k == TcKind::BlkDesliceFwd ? 2
                     : k == TcKind::BlkStats      ? 3
                                                  : 4;
    const void* fns[5] = {(const void*)k_tc_blk_pown_bf16<0>, (const void*)k_tc_blk_pown_bf16<1>,
                          (const void*)k_tc_blk_pown_bf16<2>, (const void*)k_tc_blk_pown_bf16<3>,
                          (const void*)k_tc_blk_pown_bf16<4>};
    e = set_smem(fns[mode], kPnBytes + kSmemPad);
    if (e == cudaSuccess) {
      const dim3 grid(p.P, p.B * p.H);
      if (mode == 0)
        k_tc_blk_pown_bf16<0><<<grid, 256, kPnBytes + kSmemPad, s>>>(p);
      else if (mode == 1)
        k_tc_blk_pown_bf16<1><<<grid, 256, kPnBytes + kSmemPad, s>>>(p);
      else if (mode == 2)
        k_tc_blk_pown_bf16<2><<<grid, 256, kPnBytes + kSmemPad, s>>>(p);
      else if (mode == 3)
        k_tc_blk_pown_bf16<3><<<grid, 256, kPnBytes + kSmemPad, s>>>(p);
      else
        k_tc_blk_pown_bf16<4><<<grid, 256, kPnBytes + kSmemPad, s>>>(p);
    }
  } else if (k == TcKind::BlkSliceFwd) {
    e = set_smem((const void*)k_tc_blk_slice_fwd_bf16, kBgBytes + kSmemPad);
    if (e == cudaSuccess)
      k_tc_blk_slice_fwd_bf16<<<dim3(p.P, p.G / kBgSlots, p.B * p.H), 256, kBgBytes + kSmemPad,
                                s>>>(p);
  } else {
    e = p.pdt == 1 ? run_tc_t<__nv_bfloat16>(k, p, s) : run_tc_t<float>(k, p, s);
  }
  if (e != cudaSuccess) return e;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

cudaError_t run_wait_selftest(uint64_t limit_ns, cudaStream_t s) {
  int* word = device_status();
  if (!word) return cudaErrorInvalidValue;
  k_tc_wait_selftest<<<1, 32, 0, s>>>(word, limit_ns);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

// Co-resident CTAs per SM each kernel is sized for (shared memory, TMEM and
// registers): the grid holds this many CTAs per SM.
int tc_ctas_per_sm(TcKind k) {
  switch (k) {
    case TcKind::SliceFwd: return kCtasSliceFwd;
    case TcKind::DesliceFwd: return kCtasDesliceFwd;
    case TcKind::SliceBwd: return kCtasSliceBwd;
    case TcKind::DesliceBwd: return kCtasDesliceBwd;
    case TcKind::CoupledBwd: return kCtasCoupledBwd;
    case TcKind::BlkSliceFwd: return 2;
    case TcKind::BlkSliceBwdG:
    case TcKind::BlkDesliceBwdG:
    case TcKind::BlkImage: return 1;
    case TcKind::BlkSliceBwdN:
    case TcKind::BlkDesliceBwdN:
    case TcKind::BlkDesliceFwd:
    case TcKind::BlkStats:
    case TcKind::BlkStatsOnline: return 2;
    case TcKind::SliceFwd64: return 2;
    case TcKind::DesliceFwd64: return 2;
    case TcKind::CoupledBwd64: return 1;
  }
  return 1;
}

// shared memory per SM (228 KB) holds the co-resident CTAs, each with its
// alignment pad and the 1 KB the runtime reserves per CTA
static_assert((kSfBytes + kSmemPad + 1024) * kCtasSliceFwd <= 228 * 1024, "slice fwd smem");
static_assert((kBgBytes + kSmemPad + 1024) * 2 <= 228 * 1024, "blocked slice fwd smem");
static_assert(kBbBytes + kSmemPad + 1024 <= 228 * 1024, "blocked backward smem");
static_assert((kPnBytes + kSmemPad + 1024) * 2 <= 228 * 1024, "blocked point-owning smem");
static_assert(im_bytes(32) == blk_image_bytes(32) && im_bytes(64) == blk_image_bytes(64),
              "operand image size");
static_assert((kDfBytes + kSmemPad + 1024) * kCtasDesliceFwd <= 228 * 1024, "deslice fwd smem");
static_assert((kSbBytes + kSmemPad + 1024) * kCtasSliceBwd <= 228 * 1024, "slice bwd smem");
static_assert((kDbBytes + kSmemPad + 1024) * kCtasDesliceBwd <= 228 * 1024, "deslice bwd smem");
static_assert((kCbBytes + kSmemPad + 1024) * kCtasCoupledBwd <= 228 * 1024, "coupled bwd smem");
static_assert((kS6Bytes + kSmemPad + 1024) * 2 <= 228 * 1024, "slice fwd G=64 smem");
static_assert((kD6Bytes + kSmemPad + 1024) * 2 <= 228 * 1024, "deslice fwd G=64 smem");
static_assert(kD6Ts % 16 == 0 && kD6Ws % 16 == 0, "G=64 operand alignment");
static_assert(c6_bytes(kTCoupled64) + kSmemPad + 1024 <= 228 * 1024, "coupled bwd G=64 smem");
// TMEM per SM (512 columns) holds the co-resident CTAs' allocations
static_assert(256 * kCtasSliceFwd <= 512 && kDfCols * kCtasDesliceFwd <= 512 &&
                  256 * kCtasSliceBwd <= 512 && 256 * kCtasDesliceBwd <= 512,
              "TMEM columns");
static_assert(kSfWS % 16 == 0 && kSfF % 16 == 0 && kSbUp % 16 == 0 && kDbUp % 16 == 0 &&
                  kDfTs % 16 == 0,
              "operand alignment");

}  // namespace tcx
}  // namespace fs
