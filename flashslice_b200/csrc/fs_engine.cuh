// flashslice_b200 -- shared definitions of the exact-fp32 point engine.
//
// One CTA of NT threads works on tiles of NT points of one (b, h); thread t
// owns point row t of the tile. A point's vectors (x_mid, fx_mid, d_out and
// the rows it produces) live in shared-memory rows, staged with coalesced
// 16-byte loads; its per-slot scalars (logits, weights, dw, dl) live in
// registers, GB = 32 slots at a time. Sums over points (z_num, s, dtokens,
// dW, db) are accumulated per CTA in shared memory in a fixed order and
// written as per-CTA partials, which fs_reduce sums in a fixed order: no
// atomics anywhere, so every result is bitwise reproducible for a shape.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace fs {

constexpr int GB = 32;  // slots held in registers per point at a time
constexpr float kLog2e = 1.4426950408889634f;

// A strided (B, N, H, width) point tensor.
struct Pt {
  void* data;
  int64_t sb, sn, sh, sw;
};

// Shared-memory plan of one launch; offsets in floats (-1: unused).
struct Plan {
  int dt, dvt;                  // D and DV padded to a multiple of 4
  int xrs, vrs, ors, prs, ars;  // row strides of the point rows / slot rows
  int oW, oBias, oM, oDs;       // slot-block operands: W, bias, tokens|dz_num, ds
  int oX, oV, oO, oP;           // point rows: x_mid, fx_mid|d_out, out rows
  int oA, oU;                   // per-point slot rows (weights, dl/tau)
  int oAccA, oAccB, oAccS, oAccT;  // per-CTA accumulators
  int oRed;                     // scratch for the CTA's dtau reduction
  int total;
};

struct Params {
  int B, N, H, D, DV, G;
  int P;       // programs per (b, h) (per G-block for the slot-owning kernels)
  int ntiles;  // ceil(N / NT)
  Pt x, v, o1, o2;
  const float* W;
  const float* bias;
  const float* tau;
  int64_t swb, swh, sbb, sbh;  // element strides of W / bias along b, h (0 = shared)
  const float* M;              // tokens or dz_num, (B, H, G, DV) fp32
  const float* ds;             // (B, H, G) fp32
  const float* stats_in;       // (B, H, 2, N)
  float* stats_out;
  float* delta;                // (B, H, 2, N): delta and row sum, point- to slot-owning
  float* partA;                // [bh][P][G][W] partials
  float* partB;
  float* partS;                // [bh][P][G]
  float* partDt;               // [bh][P]
  Plan pl;
};

// ---------------------------------------------------------------- dtypes
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float in(float v) { return v; }
  static __device__ __forceinline__ float out(float v) { return v; }
  static __device__ __forceinline__ void unpack(uint4 r, float* f) {
    f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                      __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float in(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 out(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ void unpack(uint4 r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]));
      const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]));
      w[i] = lo | (hi << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float in(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half out(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ void unpack(uint4 r, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
      f[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
  }
  static __device__ __forceinline__ uint4 pack(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = __half_as_ushort(__float2half_rn(f[2 * i]));
      const uint32_t hi = __half_as_ushort(__float2half_rn(f[2 * i + 1]));
      w[i] = lo | (hi << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

// ---------------------------------------------------------------- staging
// Rows [n0, n0 + NT) of the (b, h) slice of a point tensor into shared rows
// of stride rs (floats), columns [0, w) converted to fp32; columns [w, wt)
// and rows past N are zero. 16-byte vector loads when the layout allows.
template <typename T, int NT>
__device__ __forceinline__ void stage_rows(float* dst, int rs, int wt, const Pt& t,
                                           int b, int h, int n0, int N, int w) {
  const T* base = (const T*)t.data + (int64_t)b * t.sb + (int64_t)h * t.sh;
  constexpr int VEC = 16 / (int)sizeof(T);
  const bool vec = t.sw == 1 && (w % VEC) == 0 && (t.sn % VEC) == 0 &&
                   ((uintptr_t)base % 16) == 0;
  if (vec) {
    const int q = w / VEC;
    // thread -> (row, chunk) once; rows advance by NT / q when q divides NT
    const bool even = q <= NT && (NT % q) == 0;
    const int step = even ? NT / q : 0;
    const int c0 = even ? (threadIdx.x % q) * VEC : 0;
    const int i_end = NT * q;
    for (int i = threadIdx.x, r = even ? threadIdx.x / q : 0; i < i_end; i += NT) {
      int c = c0;
      if (even) {
        if (i != (int)threadIdx.x) r += step;
      } else {
        r = i / q;
        c = (i - r * q) * VEC;
      }
      const int n = n0 + r;
      float f[VEC];
      if (n < N) {
        const uint4 raw = __ldg((const uint4*)(base + (int64_t)n * t.sn + c));
        Cvt<T>::unpack(raw, f);
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) f[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < VEC; k += 4)
        *(float4*)(dst + r * rs + c + k) = make_float4(f[k], f[k + 1], f[k + 2], f[k + 3]);
    }
    for (int i = threadIdx.x; i < NT * (wt - w); i += NT) {
      const int r = i / (wt - w);
      dst[r * rs + w + (i - r * (wt - w))] = 0.f;
    }
  } else {
    for (int i = threadIdx.x; i < NT * wt; i += NT) {
      const int r = i / wt;
      const int c = i - r * wt;
      const int n = n0 + r;
      float f = 0.f;
      if (n < N && c < w) f = Cvt<T>::in(base[(int64_t)n * t.sn + (int64_t)c * t.sw]);
      dst[r * rs + c] = f;
    }
  }
}

// Shared rows back to the (b, h) slice of a point tensor, columns [0, w).
template <typename T, int NT>
__device__ __forceinline__ void store_rows(const float* src, int rs, const Pt& t, int b,
                                           int h, int n0, int N, int w) {
  T* base = (T*)t.data + (int64_t)b * t.sb + (int64_t)h * t.sh;
  constexpr int VEC = 16 / (int)sizeof(T);
  const bool vec = t.sw == 1 && (w % VEC) == 0 && (t.sn % VEC) == 0 &&
                   ((uintptr_t)base % 16) == 0;
  if (vec) {
    const int q = w / VEC;
    const bool even = q <= NT && (NT % q) == 0;
    const int step = even ? NT / q : 0;
    const int c0 = even ? (threadIdx.x % q) * VEC : 0;
    const int i_end = NT * q;
    for (int i = threadIdx.x, r = even ? threadIdx.x / q : 0; i < i_end; i += NT) {
      int c = c0;
      if (even) {
        if (i != (int)threadIdx.x) r += step;
      } else {
        r = i / q;
        c = (i - r * q) * VEC;
      }
      const int n = n0 + r;
      if (n >= N) continue;
      float f[VEC];
#pragma unroll
      for (int k = 0; k < VEC; k += 4) {
        const float4 a = *(const float4*)(src + r * rs + c + k);
        f[k] = a.x; f[k + 1] = a.y; f[k + 2] = a.z; f[k + 3] = a.w;
      }
      *(uint4*)(base + (int64_t)n * t.sn + c) = Cvt<T>::pack(f);
    }
  } else {
    for (int i = threadIdx.x; i < NT * w; i += NT) {
      const int r = i / w;
      const int c = i - r * w;
      const int n = n0 + r;
      if (n < N) base[(int64_t)n * t.sn + (int64_t)c * t.sw] = Cvt<T>::out(src[r * rs + c]);
    }
  }
}

// Rows [g0, g0 + GB) x [0, w) of a row-major (G, w) fp32 block into shared
// rows of stride wt, zero outside [0, G) x [0, w).
template <int NT>
__device__ __forceinline__ void stage_block(float* dst, int wt, const float* src, int g0,
                                            int G, int w) {
  for (int i = threadIdx.x; i < GB * wt; i += NT) {
    const int g = i / wt;
    const int c = i - g * wt;
    dst[i] = (g0 + g < G && c < w) ? src[(int64_t)(g0 + g) * w + c] : 0.f;
  }
}

template <int NT>
__device__ __forceinline__ void stage_vec(float* dst, const float* src, int g0, int G) {
  for (int g = threadIdx.x; g < GB; g += NT) dst[g] = (g0 + g < G) ? src[g0 + g] : 0.f;
}

// ---------------------------------------------------------------- per-point math
// lg[g] = x_row . W_s[g]  over the padded width dt (sequential in d).
__device__ __forceinline__ void row_dots(float (&lg)[GB], const float* row, const float* Ms,
                                         int mrs, int dt) {
#pragma unroll
  for (int g = 0; g < GB; ++g) lg[g] = 0.f;
  for (int d = 0; d < dt; d += 4) {
    const float4 xv = *(const float4*)(row + d);
#pragma unroll
    for (int g = 0; g < GB; ++g) {
      const float4 wv = *(const float4*)(Ms + g * mrs + d);
      lg[g] = fmaf(xv.x, wv.x, lg[g]);
      lg[g] = fmaf(xv.y, wv.y, lg[g]);
      lg[g] = fmaf(xv.z, wv.z, lg[g]);
      lg[g] = fmaf(xv.w, wv.w, lg[g]);
    }
  }
}

// Logits of one block: (x . W + b) / tau as (dot + b) * (1/tau), the
// reciprocal correctly rounded; slots >= G are -inf.
__device__ __forceinline__ void block_logits(float (&lg)[GB], const float* xrow, const float* Ws,
                                             const float* bs, int dt, float inv_tau, int g0,
                                             int G) {
  row_dots(lg, xrow, Ws, dt, dt);
#pragma unroll
  for (int g = 0; g < GB; ++g)
    lg[g] = (g0 + g < G) ? (lg[g] + bs[g]) * inv_tau : -INFINITY;
}

// exp(d) for d = logit - max <= 0, as exp2 of d*log2(e).
__device__ __forceinline__ float expd(float d) { return exp2f(d * kLog2e); }

// Pairwise (tree) sum of a register array, in a fixed order: v[i] += v[i+s]
// for s = N/2, N/4, ..., 1. The rounding error grows with log2(N) rather
// than N, which the temperature gradient -- a row sum that cancels to zero
// in exact arithmetic -- needs at large G. Destroys v.
template <int N>
__device__ __forceinline__ float tree_sum(float (&v)[N]) {
#pragma unroll
  for (int s = N / 2; s > 0; s >>= 1) {
#pragma unroll
    for (int i = 0; i < s; ++i) v[i] += v[i + s];
  }
  return v[0];
}

// row[c] = scale * row[c] + sum_g coef[g] * Ms[g][c]  over the padded width.
__device__ __forceinline__ void row_axpy(float* row, const float (&coef)[GB], const float* Ms,
                                         int mrs, int wt, float scale, bool init) {
  for (int c = 0; c < wt; c += 4) {
    float4 a = init ? make_float4(0.f, 0.f, 0.f, 0.f) : *(float4*)(row + c);
    if (!init) { a.x *= scale; a.y *= scale; a.z *= scale; a.w *= scale; }
#pragma unroll
    for (int g = 0; g < GB; ++g) {
      const float4 m = *(const float4*)(Ms + g * mrs + c);
      a.x = fmaf(coef[g], m.x, a.x);
      a.y = fmaf(coef[g], m.y, a.y);
      a.z = fmaf(coef[g], m.z, a.z);
      a.w = fmaf(coef[g], m.w, a.w);
    }
    *(float4*)(row + c) = a;
  }
}

__device__ __forceinline__ void row_scale(float* row, int wt, float s) {
  for (int c = 0; c < wt; c += 4) {
    float4 a = *(float4*)(row + c);
    a.x *= s; a.y *= s; a.z *= s; a.w *= s;
    *(float4*)(row + c) = a;
  }
}

__device__ __forceinline__ void row_put(float* row, const float (&v)[GB]) {
#pragma unroll
  for (int g = 0; g < GB; g += 4) *(float4*)(row + g) = make_float4(v[g], v[g + 1], v[g + 2], v[g + 3]);
}

// acc[g][c] += sum_r A[r][g] * V[r][c] for the GB slots and padded width wt
// (and accs[g] += sum_r A[r][g] when accs is given): each thread owns chunks
// of 2 slots x 4 columns; rows are summed in order r = 0, 1, ... per tile.
template <int NT>
__device__ __forceinline__ void pool_tile(float* acc, float* accs, const float* A, int ars,
                                          const float* V, int vrs, int wt, int nrows) {
  const int q = wt >> 2;
  const int nch = (GB / 2) * q;
  for (int ch = threadIdx.x; ch < nch; ch += NT) {
    const int gp = ch / q;
    const int c = (ch - gp * q) * 4;
    const int g = 2 * gp;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    float s0 = 0.f, s1 = 0.f;
    const bool own_s = accs != nullptr && c == 0;
    for (int r = 0; r < nrows; ++r) {
      const float2 av = *(const float2*)(A + r * ars + g);
      const float4 v = *(const float4*)(V + r * vrs + c);
      a0.x = fmaf(av.x, v.x, a0.x); a0.y = fmaf(av.x, v.y, a0.y);
      a0.z = fmaf(av.x, v.z, a0.z); a0.w = fmaf(av.x, v.w, a0.w);
      a1.x = fmaf(av.y, v.x, a1.x); a1.y = fmaf(av.y, v.y, a1.y);
      a1.z = fmaf(av.y, v.z, a1.z); a1.w = fmaf(av.y, v.w, a1.w);
      if (own_s) { s0 += av.x; s1 += av.y; }
    }
    float4* p0 = (float4*)(acc + g * wt + c);
    float4* p1 = (float4*)(acc + (g + 1) * wt + c);
    float4 o0 = *p0, o1 = *p1;
    o0.x += a0.x; o0.y += a0.y; o0.z += a0.z; o0.w += a0.w;
    o1.x += a1.x; o1.y += a1.y; o1.z += a1.z; o1.w += a1.w;
    *p0 = o0; *p1 = o1;
    if (own_s) { accs[g] += s0; accs[g + 1] += s1; }
  }
}

// Fixed-order CTA sum of one float per thread (tree over a shared scratch).
template <int NT>
__device__ __forceinline__ float cta_sum(float v, float* red) {
  red[threadIdx.x] = v;
  __syncthreads();
#pragma unroll
  for (int s = NT / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  const float r = red[0];
  __syncthreads();
  return r;
}

}  // namespace fs
