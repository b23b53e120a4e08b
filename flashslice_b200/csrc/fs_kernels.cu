// flashslice_b200 -- kernels of the exact-fp32 point engine (sm_100a).
//
// Two kernel families, the two contracts of the reference:
//   fused (G <= 32): one pass per op, the softmax formed whole per point in
//     registers (the reference's single-tile family, slice_ops.py:555-776);
//   blocked (any G): the per-point statistics (m, l) formed once, weights
//     recomputed one block of 32 slots at a time; point-owning kernels make
//     the per-point outputs, slot-owning kernels the sums over points
//     (the reference's G-blocked family, blocked.py:293-888).
// Every product is an fp32 FMA, every accumulator fp32: the precision of the
// reference's ieee dot level, served for every level.
#include <atomic>

#include "fs_engine.cuh"
#include "fs_launch.h"

namespace fs {

#define FS_PROLOGUE(BH)                                                   \
  extern __shared__ float4 fs_smem4[];                                    \
  float* sm = reinterpret_cast<float*>(fs_smem4);                         \
  const Plan& L = p.pl;                                                   \
  const int bh = (BH);                                                    \
  const int b = bh / p.H;                                                 \
  const int h = bh - b * p.H;                                             \
  const int N = p.N, G = p.G, D = p.D, DV = p.DV;                         \
  const int t = threadIdx.x;                                              \
  const float* Wb = p.W + (int64_t)b * p.swb + (int64_t)h * p.swh;        \
  const float* bb = p.bias + (int64_t)b * p.sbb + (int64_t)h * p.sbh;     \
  const float inv_tau = __frcp_rn(p.tau[h]);                              \
  (void)D; (void)DV; (void)Wb; (void)bb; (void)inv_tau; (void)G; (void)t;

// whole-row softmax of one block (G <= 32): w = exp(lg - m) * (1 / sum);
// returns the row max m
__device__ __forceinline__ float row_softmax(const float (&lg)[GB], float (&w)[GB], bool valid) {
  float m = lg[0];
#pragma unroll
  for (int g = 1; g < GB; ++g) m = fmaxf(m, lg[g]);
  float tmp[GB];
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    w[g] = expd(lg[g] - m);
    tmp[g] = w[g];
  }
  const float s = tree_sum(tmp);
  const float r = valid ? __frcp_rn(s) : 0.f;
#pragma unroll
  for (int g = 0; g < GB; ++g) w[g] *= r;
  return m;
}

// dl = w * (dw - sum_g w dw) (the softmax Jacobian, pre-division); returns
// sum_g dl * (lg - m) over the valid slots and leaves dl / tau in dw.
// sum_g dl vanishes exactly, so sum_g dl * lg = sum_g dl * (lg - m); centring
// on the row max m keeps a common offset of the logits from multiplying the
// rounding residue of sum_g dl into the temperature gradient.
__device__ __forceinline__ float row_jacobian(const float (&w)[GB], float (&dw)[GB],
                                              const float (&lg)[GB], float m, float inv_tau,
                                              int G) {
  float tmp[GB];
#pragma unroll
  for (int g = 0; g < GB; ++g) tmp[g] = w[g] * dw[g];
  const float gs = tree_sum(tmp);
#pragma unroll
  for (int g = 0; g < GB; ++g) {
    const float dl = w[g] * (dw[g] - gs);
    tmp[g] = g < G ? dl * (lg[g] - m) : 0.f;
    dw[g] = dl * inv_tau;
  }
  return tree_sum(tmp);
}

template <int NT>
__device__ __forceinline__ void zero_region(float* a, int n) {
  for (int i = threadIdx.x; i < n; i += NT) a[i] = 0.f;
}

// (GB x wt) shared accumulator rows [0, gcount) -> part (gcount x w) slice
template <int NT>
__device__ __forceinline__ void write_part(float* part, const float* acc, int wt, int gcount,
                                           int w) {
  for (int i = threadIdx.x; i < gcount * w; i += NT) {
    const int g = i / w;
    part[i] = acc[g * wt + (i - g * w)];
  }
}

// ============================================================== fused family

template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_fused_slice_fwd(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *xs = sm + L.oX, *vs = sm + L.oV;
  float *as = sm + L.oA, *accz = sm + L.oAccA, *accs = sm + L.oAccS;
  stage_block<NT>(Ws, L.dt, Wb, 0, G, D);
  stage_vec<NT>(bs, bb, 0, G);
  zero_region<NT>(accz, GB * L.dvt);
  zero_region<NT>(accs, GB);
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    __syncthreads();
    float lg[GB], w[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, 0, G);
    row_softmax(lg, w, n0 + t < N);
    row_put(as + t * L.ars, w);
    __syncthreads();
    pool_tile<NT>(accz, accs, as, L.ars, vs, L.vrs, L.dvt, min(NT, N - n0));
  }
  __syncthreads();
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  write_part<NT>(p.partA + slot * G * DV, accz, L.dvt, G, DV);
  for (int g = t; g < G; g += NT) p.partS[slot * G + g] = accs[g];
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_fused_deslice_fwd(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM, *xs = sm + L.oX, *os = sm + L.oO;
  stage_block<NT>(Ws, L.dt, Wb, 0, G, D);
  stage_vec<NT>(bs, bb, 0, G);
  stage_block<NT>(Ms, L.dvt, p.M + (int64_t)bh * G * DV, 0, G, DV);
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    __syncthreads();
    float lg[GB], w[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, 0, G);
    row_softmax(lg, w, true);
    row_axpy(os + t * L.ors, w, Ms, L.dvt, L.dvt, 1.f, true);
    __syncthreads();
    store_rows<T, NT>(os, L.ors, p.o1, b, h, n0, N, DV);
  }
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_fused_slice_bwd(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM, *dss = sm + L.oDs;
  float *xs = sm + L.oX, *vs = sm + L.oV, *us = sm + L.oU;
  float *accw = sm + L.oAccA, *accb = sm + L.oAccS, *red = sm + L.oRed;
  stage_block<NT>(Ws, L.dt, Wb, 0, G, D);
  stage_vec<NT>(bs, bb, 0, G);
  stage_block<NT>(Ms, L.dvt, p.M + (int64_t)bh * G * DV, 0, G, DV);
  stage_vec<NT>(dss, p.ds + (int64_t)bh * G, 0, G);
  zero_region<NT>(accw, GB * L.dt);
  zero_region<NT>(accb, GB);
  float dt_acc = 0.f;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    __syncthreads();
    float lg[GB], w[GB], dw[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, 0, G);
    const float mrow = row_softmax(lg, w, n0 + t < N);
    // dw = fx . dz_num^T + ds  (slice_ops.py:695)
    row_dots(dw, vs + t * L.vrs, Ms, L.dvt, L.dvt);
#pragma unroll
    for (int g = 0; g < GB; ++g) dw[g] += dss[g];
    dt_acc += row_jacobian(w, dw, lg, mrow, inv_tau, G);
    // dfx = w @ dz_num, written over this point's fx row (slice_ops.py:690)
    row_axpy(vs + t * L.vrs, w, Ms, L.dvt, L.dvt, 1.f, true);
    row_put(us + t * L.ars, dw);
    __syncthreads();
    pool_tile<NT>(accw, accb, us, L.ars, xs, L.xrs, L.dt, min(NT, N - n0));
    __syncthreads();
    // dx = (dl / tau) @ W, written over this point's x row (slice_ops.py:699)
    row_axpy(xs + t * L.xrs, dw, Ws, L.dt, L.dt, 1.f, true);
    __syncthreads();
    store_rows<T, NT>(vs, L.vrs, p.o2, b, h, n0, N, DV);
    store_rows<T, NT>(xs, L.xrs, p.o1, b, h, n0, N, D);
  }
  __syncthreads();
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  write_part<NT>(p.partA + slot * G * D, accw, L.dt, G, D);
  for (int g = t; g < G; g += NT) p.partS[slot * G + g] = accb[g];
  const float tot = cta_sum<NT>(dt_acc, red);
  if (t == 0) p.partDt[slot] = -inv_tau * tot;
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_fused_deslice_bwd(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM;
  float *xs = sm + L.oX, *vs = sm + L.oV, *as = sm + L.oA, *us = sm + L.oU;
  float *accw = sm + L.oAccA, *acct = sm + L.oAccB, *accb = sm + L.oAccS, *red = sm + L.oRed;
  stage_block<NT>(Ws, L.dt, Wb, 0, G, D);
  stage_vec<NT>(bs, bb, 0, G);
  stage_block<NT>(Ms, L.dvt, p.M + (int64_t)bh * G * DV, 0, G, DV);
  zero_region<NT>(accw, GB * L.dt);
  zero_region<NT>(acct, GB * L.dvt);
  zero_region<NT>(accb, GB);
  float dt_acc = 0.f;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    __syncthreads();
    float lg[GB], w[GB], dw[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, 0, G);
    const float mrow = row_softmax(lg, w, n0 + t < N);
    // dw = d_out . tokens^T  (slice_ops.py:760)
    row_dots(dw, vs + t * L.vrs, Ms, L.dvt, L.dvt);
    dt_acc += row_jacobian(w, dw, lg, mrow, inv_tau, G);
    row_put(as + t * L.ars, w);
    row_put(us + t * L.ars, dw);
    __syncthreads();
    const int nr = min(NT, N - n0);
    pool_tile<NT>(acct, nullptr, as, L.ars, vs, L.vrs, L.dvt, nr);  // dtokens += w^T d_out
    pool_tile<NT>(accw, accb, us, L.ars, xs, L.xrs, L.dt, nr);      // dW += (dl/tau)^T x
    __syncthreads();
    row_axpy(xs + t * L.xrs, dw, Ws, L.dt, L.dt, 1.f, true);
    __syncthreads();
    store_rows<T, NT>(xs, L.xrs, p.o1, b, h, n0, N, D);
  }
  __syncthreads();
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  write_part<NT>(p.partA + slot * G * D, accw, L.dt, G, D);
  write_part<NT>(p.partB + slot * G * DV, acct, L.dvt, G, DV);
  for (int g = t; g < G; g += NT) p.partS[slot * G + g] = accb[g];
  const float tot = cta_sum<NT>(dt_acc, red);
  if (t == 0) p.partDt[slot] = -inv_tau * tot;
}

// ============================================================== blocked family

__device__ __forceinline__ void load_stats(const Params& p, int bh, int n, float& m, float& l) {
  if (n < p.N) {
    const float* st = p.stats_in + (int64_t)bh * 2 * p.N;
    m = st[n];
    l = st[p.N + n];
  } else {
    m = 0.f;
    l = 1.f;
  }
}

// Per-point statistics: online (l rescaled by exp(m_old - m_new) when the
// max moves, blocked.py:331-343) or two-pass (max, then sum, :350-400).
template <typename T, int NT, bool TWOPASS>
__global__ void __launch_bounds__(NT) k_blk_stats(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *xs = sm + L.oX;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    float m = -INFINITY, l = 0.f;
    for (int g0 = 0; g0 < G; g0 += GB) {
      __syncthreads();
      stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
      stage_vec<NT>(bs, bb, g0, G);
      __syncthreads();
      float lg[GB];
      block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
      float bm = lg[0];
#pragma unroll
      for (int g = 1; g < GB; ++g) bm = fmaxf(bm, lg[g]);
      if (TWOPASS) {
        m = fmaxf(m, bm);
      } else {
        const float mn = fmaxf(m, bm);
#pragma unroll
        for (int g = 0; g < GB; ++g) lg[g] = expd(lg[g] - mn);
        l = l * expd(m - mn) + tree_sum(lg);
        m = mn;
      }
    }
    if (TWOPASS) {
      for (int g0 = 0; g0 < G; g0 += GB) {
        __syncthreads();
        stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
        stage_vec<NT>(bs, bb, g0, G);
        __syncthreads();
        float lg[GB];
        block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
#pragma unroll
        for (int g = 0; g < GB; ++g) lg[g] = expd(lg[g] - m);
        l += tree_sum(lg);
      }
    }
    const int n = n0 + t;
    if (n < N) {
      float* st = p.stats_out + (int64_t)bh * 2 * N;
      st[n] = m;
      st[N + n] = l;
    }
  }
}

// Deslice forward, point-owning: with the statistics in hand (out = sum_g e
// tok / l, blocked.py:466-510) or online, forming out and (m, l) in one pass
// (FlashAttention-forward rescaling, blocked.py:514-573).
template <typename T, int NT, bool ONLINE>
__global__ void __launch_bounds__(NT) k_blk_deslice_fwd(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM, *xs = sm + L.oX, *os = sm + L.oO;
  const float* tokb = p.M + (int64_t)bh * G * DV;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    const int n = n0 + t;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    float m = -INFINITY, l = 0.f;
    if (!ONLINE) load_stats(p, bh, n, m, l);
    bool first = true;
    for (int g0 = 0; g0 < G; g0 += GB) {
      __syncthreads();
      stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
      stage_vec<NT>(bs, bb, g0, G);
      stage_block<NT>(Ms, L.dvt, tokb, g0, G, DV);
      __syncthreads();
      float lg[GB];
      block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
      if (ONLINE) {
        float bm = lg[0];
#pragma unroll
        for (int g = 1; g < GB; ++g) bm = fmaxf(bm, lg[g]);
        const float mn = fmaxf(m, bm);
        const float alpha = expd(m - mn);
        float tmp[GB];
#pragma unroll
        for (int g = 0; g < GB; ++g) {
          lg[g] = expd(lg[g] - mn);
          tmp[g] = lg[g];
        }
        l = l * alpha + tree_sum(tmp);
        m = mn;
        row_axpy(os + t * L.ors, lg, Ms, L.dvt, L.dvt, alpha, first);
      } else {
#pragma unroll
        for (int g = 0; g < GB; ++g) lg[g] = expd(lg[g] - m);
        row_axpy(os + t * L.ors, lg, Ms, L.dvt, L.dvt, 1.f, first);
      }
      first = false;
    }
    row_scale(os + t * L.ors, L.dvt, __frcp_rn(l));
    if (ONLINE && n < N) {
      float* st = p.stats_out + (int64_t)bh * 2 * N;
      st[n] = m;
      st[N + n] = l;
    }
    __syncthreads();
    store_rows<T, NT>(os, L.ors, p.o1, b, h, n0, N, DV);
  }
}

// Slot-owning slice forward: one block of 32 slots, streaming the points
// (blocked.py:404-462). Grid (P, blocks, B*H).
template <typename T, int NT>
__global__ void __launch_bounds__(NT) k_blk_slice_fwd_g(Params p) {
  FS_PROLOGUE(blockIdx.z)
  const int g0 = blockIdx.y * GB;
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *xs = sm + L.oX, *vs = sm + L.oV;
  float *as = sm + L.oA, *accz = sm + L.oAccA, *accs = sm + L.oAccS;
  stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
  stage_vec<NT>(bs, bb, g0, G);
  zero_region<NT>(accz, GB * L.dvt);
  zero_region<NT>(accs, GB);
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    const int n = n0 + t;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    float m, l;
    load_stats(p, bh, n, m, l);
    __syncthreads();
    float lg[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
    const float r = n < N ? __frcp_rn(l) : 0.f;
#pragma unroll
    for (int g = 0; g < GB; ++g) lg[g] = expd(lg[g] - m) * r;
    row_put(as + t * L.ars, lg);
    __syncthreads();
    pool_tile<NT>(accz, accs, as, L.ars, vs, L.vrs, L.dvt, min(NT, N - n0));
  }
  __syncthreads();
  const int gc = min(GB, G - g0);
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* pz = p.partA + slot * G * DV + (int64_t)g0 * DV;
  for (int i = t; i < gc * DV; i += NT) {
    const int g = i / DV;
    pz[i] = accz[g * L.dvt + (i - g * DV)];
  }
  for (int g = t; g < gc; g += NT) p.partS[slot * G + g0 + g] = accs[g];
}

// Point-owning backward (slice: dfx, delta, dx, dtau; blocked.py:577-673.
// deslice: delta, dx, dtau; blocked.py:745-815). Pass 1 over the slot
// blocks forms delta = sum_g e dw / l (and dfx for the slice); pass 2 forms
// dl = (e dw - e delta) / l from the same products, dx and the per-row
// temperature term, row by row over all of G.
template <typename T, int NT, bool SLICE>
__global__ void __launch_bounds__(NT) k_blk_bwd_n(Params p) {
  FS_PROLOGUE(blockIdx.y)
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM, *dss = sm + L.oDs;
  float *xs = sm + L.oX, *vs = sm + L.oV, *os = sm + L.oO, *ps = sm + L.oP, *red = sm + L.oRed;
  const float* mb = p.M + (int64_t)bh * G * DV;
  const float* dsb = p.ds + (int64_t)bh * G;
  float dt_acc = 0.f;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    const int n = n0 + t;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    float m, l_saved;
    load_stats(p, bh, n, m, l_saved);
    // The row sum is formed here from the very exponentials the Jacobian
    // uses, so that sum_g dl vanishes to one summation's rounding whatever
    // rounding the saved l carries (the temperature gradient, sum dl*logit,
    // turns any mismatch into a bias).
    float sdw = 0.f, lrow = 0.f;
    bool first = true;
    for (int g0 = 0; g0 < G; g0 += GB) {
      __syncthreads();
      stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
      stage_vec<NT>(bs, bb, g0, G);
      stage_block<NT>(Ms, L.dvt, mb, g0, G, DV);
      if (SLICE) stage_vec<NT>(dss, dsb, g0, G);
      __syncthreads();
      float lg[GB], dw[GB], tmp[GB];
      block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
#pragma unroll
      for (int g = 0; g < GB; ++g) {
        lg[g] = expd(lg[g] - m);
        tmp[g] = lg[g];
      }
      lrow += tree_sum(tmp);
      row_dots(dw, vs + t * L.vrs, Ms, L.dvt, L.dvt);
#pragma unroll
      for (int g = 0; g < GB; ++g) {
        if (SLICE) dw[g] += dss[g];
        dw[g] *= lg[g];
      }
      sdw += tree_sum(dw);
      if (SLICE) row_axpy(os + t * L.ors, lg, Ms, L.dvt, L.dvt, 1.f, first);
      first = false;
    }
    const float inv_l = __frcp_rn(lrow);
    const float delta = sdw * inv_l;
    if (n < N) {
      p.delta[(int64_t)bh * 2 * N + n] = delta;
      p.delta[(int64_t)bh * 2 * N + N + n] = lrow;
    }
    if (SLICE) {
      row_scale(os + t * L.ors, L.dvt, inv_l);
      // dfx is complete: store it now, its rows may hold dx next
      __syncthreads();
      store_rows<T, NT>(os, L.ors, p.o2, b, h, n0, N, DV);
    }
    float rdt = 0.f;
    first = true;
    for (int g0 = 0; g0 < G; g0 += GB) {
      __syncthreads();
      stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
      stage_vec<NT>(bs, bb, g0, G);
      stage_block<NT>(Ms, L.dvt, mb, g0, G, DV);
      if (SLICE) stage_vec<NT>(dss, dsb, g0, G);
      __syncthreads();
      float lg[GB], dw[GB];
      block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
      row_dots(dw, vs + t * L.vrs, Ms, L.dvt, L.dvt);
#pragma unroll
      for (int g = 0; g < GB; ++g) {
        const float e = expd(lg[g] - m);
        const float dwg = SLICE ? dw[g] + dss[g] : dw[g];
        const float dl = (e * dwg - e * delta) * inv_l;
        lg[g] = g0 + g < G ? dl * (lg[g] - m) : 0.f;  // centred, see row_jacobian
        dw[g] = dl;
      }
      rdt += tree_sum(lg);
      row_axpy(ps + t * L.prs, dw, Ws, L.dt, L.dt, 1.f, first);
      first = false;
    }
    row_scale(ps + t * L.prs, L.dt, inv_tau);
    if (n < N) dt_acc += rdt;
    __syncthreads();
    store_rows<T, NT>(ps, L.prs, p.o1, b, h, n0, N, D);
  }
  __syncthreads();
  const float tot = cta_sum<NT>(dt_acc, red);
  if (t == 0) p.partDt[(int64_t)bh * p.P + blockIdx.x] = -inv_tau * tot;
}

// Slot-owning backward: partial dW, db (slice, blocked.py:677-741) and
// dtokens (deslice, :819-888) for one block of 32 slots. Grid (P, blocks, B*H).
template <typename T, int NT, bool SLICE>
__global__ void __launch_bounds__(NT) k_blk_bwd_g(Params p) {
  FS_PROLOGUE(blockIdx.z)
  const int g0 = blockIdx.y * GB;
  float *Ws = sm + L.oW, *bs = sm + L.oBias, *Ms = sm + L.oM, *dss = sm + L.oDs;
  float *xs = sm + L.oX, *vs = sm + L.oV, *as = sm + L.oA, *us = sm + L.oU;
  float *accw = sm + L.oAccA, *acct = sm + L.oAccB, *accb = sm + L.oAccS;
  stage_block<NT>(Ws, L.dt, Wb, g0, G, D);
  stage_vec<NT>(bs, bb, g0, G);
  stage_block<NT>(Ms, L.dvt, p.M + (int64_t)bh * G * DV, g0, G, DV);
  if (SLICE) stage_vec<NT>(dss, p.ds + (int64_t)bh * G, g0, G);
  zero_region<NT>(accw, GB * L.dt);
  if (!SLICE) zero_region<NT>(acct, GB * L.dvt);
  zero_region<NT>(accb, GB);
  for (int tile = blockIdx.x; tile < p.ntiles; tile += p.P) {
    const int n0 = tile * NT;
    const int n = n0 + t;
    __syncthreads();
    stage_rows<T, NT>(xs, L.xrs, L.dt, p.x, b, h, n0, N, D);
    stage_rows<T, NT>(vs, L.vrs, L.dvt, p.v, b, h, n0, N, DV);
    float m, l;
    load_stats(p, bh, n, m, l);
    // delta and the row sum the point-owning kernel formed (see k_blk_bwd_n)
    const float delta = n < N ? p.delta[(int64_t)bh * 2 * N + n] : 0.f;
    if (n < N) l = p.delta[(int64_t)bh * 2 * N + N + n];
    __syncthreads();
    float lg[GB], dw[GB];
    block_logits(lg, xs + t * L.xrs, Ws, bs, L.dt, inv_tau, g0, G);
    const float r = n < N ? __frcp_rn(l) : 0.f;
#pragma unroll
    for (int g = 0; g < GB; ++g) lg[g] = expd(lg[g] - m) * r;
    row_dots(dw, vs + t * L.vrs, Ms, L.dvt, L.dvt);
#pragma unroll
    for (int g = 0; g < GB; ++g) {
      const float dwg = SLICE ? dw[g] + dss[g] : dw[g];
      dw[g] = lg[g] * (dwg - delta) * inv_tau;
    }
    if (!SLICE) row_put(as + t * L.ars, lg);
    row_put(us + t * L.ars, dw);
    __syncthreads();
    const int nr = min(NT, N - n0);
    if (!SLICE) pool_tile<NT>(acct, nullptr, as, L.ars, vs, L.vrs, L.dvt, nr);
    pool_tile<NT>(accw, accb, us, L.ars, xs, L.xrs, L.dt, nr);
  }
  __syncthreads();
  const int gc = min(GB, G - g0);
  const int64_t slot = (int64_t)bh * p.P + blockIdx.x;
  float* pw = p.partA + slot * G * D + (int64_t)g0 * D;
  for (int i = t; i < gc * D; i += NT) {
    const int g = i / D;
    pw[i] = accw[g * L.dt + (i - g * D)];
  }
  if (!SLICE) {
    float* pt = p.partB + slot * G * DV + (int64_t)g0 * DV;
    for (int i = t; i < gc * DV; i += NT) {
      const int g = i / DV;
      pt[i] = acct[g * L.dvt + (i - g * DV)];
    }
  }
  for (int g = t; g < gc; g += NT) p.partS[slot * G + g0 + g] = accb[g];
}

// ============================================================== reduction
// out[ob][oh][e] = sum_b sum_h sum_p part[(b*H + h)*P + p][e], b over all of
// B when the output has no batch axis (ob_ext == 1) and h likewise: the
// per-program partials and the broadcast-axis sums of slice_ops.py:481-500,
// in one fixed order.
__global__ void k_reduce(const float* __restrict__ part, float* __restrict__ out, int B, int H,
                         int P, int64_t E, int ob_ext, int oh_ext) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const int o = blockIdx.y;
  const int ob = o / oh_ext, oh = o - ob * oh_ext;
  const int b0 = ob_ext == 1 ? 0 : ob, b1 = ob_ext == 1 ? B : ob + 1;
  const int h0 = oh_ext == 1 ? 0 : oh, h1 = oh_ext == 1 ? H : oh + 1;
  float acc = 0.f;
  for (int bb = b0; bb < b1; ++bb)
    for (int hh = h0; hh < h1; ++hh) {
      const float* src = part + ((int64_t)(bb * H + hh) * P) * E + e;
      for (int q = 0; q < P; ++q) acc += src[(int64_t)q * E];
    }
  out[(int64_t)o * E + e] = acc;
}

// ============================================================== launchers

std::atomic<uint64_t> g_launches{0};

constexpr size_t kMaxSmem = 227 * 1024;

template <typename K>
static cudaError_t launch(K kernel, dim3 grid, int nt, const Params& p, cudaStream_t s) {
  const size_t bytes = (size_t)p.pl.total * sizeof(float);
  if (bytes > kMaxSmem) return cudaErrorInvalidConfiguration;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)bytes);
  if (e != cudaSuccess) return e;
  // the full shared carveout, so that as many CTAs as fit are resident
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  kernel<<<grid, nt, bytes, s>>>(p);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

template <typename T, int NT>
static cudaError_t run_kind(Kind k, const Params& p, int nblk, cudaStream_t s) {
  const int bhn = p.B * p.H;
  const dim3 gn(p.P, bhn);
  const dim3 gg(p.P, nblk, bhn);
  switch (k) {
    case Kind::FusedSliceFwd: return launch(k_fused_slice_fwd<T, NT>, gn, NT, p, s);
    case Kind::FusedDesliceFwd: return launch(k_fused_deslice_fwd<T, NT>, gn, NT, p, s);
    case Kind::FusedSliceBwd: return launch(k_fused_slice_bwd<T, NT>, gn, NT, p, s);
    case Kind::FusedDesliceBwd: return launch(k_fused_deslice_bwd<T, NT>, gn, NT, p, s);
    case Kind::StatsOnline: return launch(k_blk_stats<T, NT, false>, gn, NT, p, s);
    case Kind::StatsTwoPass: return launch(k_blk_stats<T, NT, true>, gn, NT, p, s);
    case Kind::DesliceFwdStats: return launch(k_blk_deslice_fwd<T, NT, false>, gn, NT, p, s);
    case Kind::DesliceFwdOnline: return launch(k_blk_deslice_fwd<T, NT, true>, gn, NT, p, s);
    case Kind::SliceFwdG: return launch(k_blk_slice_fwd_g<T, NT>, gg, NT, p, s);
    case Kind::SliceBwdN: return launch(k_blk_bwd_n<T, NT, true>, gn, NT, p, s);
    case Kind::DesliceBwdN: return launch(k_blk_bwd_n<T, NT, false>, gn, NT, p, s);
    case Kind::SliceBwdG: return launch(k_blk_bwd_g<T, NT, true>, gg, NT, p, s);
    case Kind::DesliceBwdG: return launch(k_blk_bwd_g<T, NT, false>, gg, NT, p, s);
  }
  return cudaErrorInvalidValue;
}

// CTAs of kind k that fit one SM at once (its shared memory, registers and
// threads), 0 if the query fails.
template <typename K>
static int resident(K kernel, int nt, const Params& p) {
  const size_t bytes = (size_t)p.pl.total * sizeof(float);
  if (bytes > kMaxSmem ||
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return 0;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, nt, bytes) != cudaSuccess)
    return 0;
  return n;
}

template <typename T, int NT>
static int resident_kind(Kind k, const Params& p) {
  switch (k) {
    case Kind::FusedSliceFwd: return resident(k_fused_slice_fwd<T, NT>, NT, p);
    case Kind::FusedDesliceFwd: return resident(k_fused_deslice_fwd<T, NT>, NT, p);
    case Kind::FusedSliceBwd: return resident(k_fused_slice_bwd<T, NT>, NT, p);
    case Kind::FusedDesliceBwd: return resident(k_fused_deslice_bwd<T, NT>, NT, p);
    case Kind::StatsOnline: return resident(k_blk_stats<T, NT, false>, NT, p);
    case Kind::StatsTwoPass: return resident(k_blk_stats<T, NT, true>, NT, p);
    case Kind::DesliceFwdStats: return resident(k_blk_deslice_fwd<T, NT, false>, NT, p);
    case Kind::DesliceFwdOnline: return resident(k_blk_deslice_fwd<T, NT, true>, NT, p);
    case Kind::SliceFwdG: return resident(k_blk_slice_fwd_g<T, NT>, NT, p);
    case Kind::SliceBwdN: return resident(k_blk_bwd_n<T, NT, true>, NT, p);
    case Kind::DesliceBwdN: return resident(k_blk_bwd_n<T, NT, false>, NT, p);
    case Kind::SliceBwdG: return resident(k_blk_bwd_g<T, NT, true>, NT, p);
    case Kind::DesliceBwdG: return resident(k_blk_bwd_g<T, NT, false>, NT, p);
  }
  return 0;
}

int engine_resident(Kind k, int dtype, int nt, const Params& p) {
  if (nt == 128) {
    if (dtype == 0) return resident_kind<float, 128>(k, p);
    if (dtype == 1) return resident_kind<__nv_bfloat16, 128>(k, p);
    return resident_kind<__half, 128>(k, p);
  }
  if (dtype == 0) return resident_kind<float, 32>(k, p);
  if (dtype == 1) return resident_kind<__nv_bfloat16, 32>(k, p);
  return resident_kind<__half, 32>(k, p);
}

cudaError_t run_engine(Kind k, int dtype, int nt, const Params& p, int nblk, cudaStream_t s) {
  const bool fused = k == Kind::FusedSliceFwd || k == Kind::FusedDesliceFwd ||
                     k == Kind::FusedSliceBwd || k == Kind::FusedDesliceBwd;
  if (fused && nt != 128) return cudaErrorInvalidValue;
  if (nt == 128) {
    if (dtype == 0) return run_kind<float, 128>(k, p, nblk, s);
    if (dtype == 1) return run_kind<__nv_bfloat16, 128>(k, p, nblk, s);
    return run_kind<__half, 128>(k, p, nblk, s);
  }
  if (fused) return cudaErrorInvalidValue;
  if (dtype == 0) return run_kind<float, 32>(k, p, nblk, s);
  if (dtype == 1) return run_kind<__nv_bfloat16, 32>(k, p, nblk, s);
  return run_kind<__half, 32>(k, p, nblk, s);
}

cudaError_t run_reduce(const float* part, float* out, int B, int H, int P, int64_t E, int ob_ext,
                       int oh_ext, cudaStream_t s) {
  if (E <= 0) return cudaSuccess;
  const int nt = 256;
  const dim3 grid((unsigned)((E + nt - 1) / nt), ob_ext * oh_ext);
  k_reduce<<<grid, nt, 0, s>>>(part, out, B, H, P, E, ob_ext, oh_ext);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaGetLastError();
}

}  // namespace fs
