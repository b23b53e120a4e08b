// flashslice_b200 -- host-side view of the point engine: kernel kinds, the
// shared-memory plan and the launchers (fs_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <initializer_list>

#include "fs_engine.cuh"

namespace fs {

enum class Kind {
  FusedSliceFwd,
  FusedDesliceFwd,
  FusedSliceBwd,
  FusedDesliceBwd,
  StatsOnline,
  StatsTwoPass,
  DesliceFwdStats,
  DesliceFwdOnline,
  SliceFwdG,
  SliceBwdN,
  DesliceBwdN,
  SliceBwdG,
  DesliceBwdG,
};

constexpr int kTargetCtas = 4 * 148;  // one persistent wave at 4 CTAs per SM

inline int round4(int v) { return (v + 3) & ~3; }
// Shared row stride (floats) with an odd number of 16-byte units, so that
// the own-row 16-byte accesses of 8 consecutive threads hit 8 bank groups.
inline int row_stride(int w) { return ((w / 4) & 1) ? w : w + 4; }

inline Plan make_plan(Kind k, int D, int DV, int nt) {
  Plan pl = {};
  pl.dt = round4(D);
  pl.dvt = round4(DV);
  pl.xrs = row_stride(pl.dt);
  pl.vrs = row_stride(pl.dvt);
  pl.ors = pl.vrs;
  pl.prs = pl.xrs;
  pl.ars = row_stride(GB);
  int off = 0;
  auto take = [&](int n) { const int o = off; off += round4(n); return o; };
  auto any = [k](std::initializer_list<Kind> ks) {
    for (Kind q : ks) if (q == k) return true;
    return false;
  };
  using K = Kind;
  pl.oW = take(GB * pl.dt);
  pl.oBias = take(GB);
  if (any({K::FusedDesliceFwd, K::FusedSliceBwd, K::FusedDesliceBwd, K::DesliceFwdStats,
           K::DesliceFwdOnline, K::SliceBwdN, K::DesliceBwdN, K::SliceBwdG, K::DesliceBwdG}))
    pl.oM = take(GB * pl.dvt);
  if (any({K::FusedSliceBwd, K::SliceBwdN, K::SliceBwdG})) pl.oDs = take(GB);
  pl.oX = take(nt * pl.xrs);
  if (any({K::FusedSliceFwd, K::FusedSliceBwd, K::FusedDesliceBwd, K::SliceFwdG, K::SliceBwdN,
           K::DesliceBwdN, K::SliceBwdG, K::DesliceBwdG}))
    pl.oV = take(nt * pl.vrs);
  if (any({K::FusedDesliceFwd, K::DesliceFwdStats, K::DesliceFwdOnline, K::SliceBwdN}))
    pl.oO = take(nt * pl.ors);
  // slice's point-owning backward stores its dfx rows before it forms dx, so
  // the dx rows reuse them when they fit (a second resident CTA at DV = 64)
  if (k == K::SliceBwdN && pl.prs <= pl.ors)
    pl.oP = pl.oO;
  else if (any({K::SliceBwdN, K::DesliceBwdN}))
    pl.oP = take(nt * pl.prs);
  if (any({K::FusedSliceFwd, K::FusedDesliceBwd, K::SliceFwdG, K::DesliceBwdG}))
    pl.oA = take(nt * pl.ars);
  if (any({K::FusedSliceBwd, K::FusedDesliceBwd, K::SliceBwdG, K::DesliceBwdG}))
    pl.oU = take(nt * pl.ars);
  if (any({K::FusedSliceFwd, K::SliceFwdG})) pl.oAccA = take(GB * pl.dvt);
  if (any({K::FusedSliceBwd, K::FusedDesliceBwd, K::SliceBwdG, K::DesliceBwdG}))
    pl.oAccA = take(GB * pl.dt);
  if (any({K::FusedDesliceBwd, K::DesliceBwdG})) pl.oAccB = take(GB * pl.dvt);
  if (any({K::FusedSliceFwd, K::SliceFwdG, K::FusedSliceBwd, K::FusedDesliceBwd, K::SliceBwdG,
           K::DesliceBwdG}))
    pl.oAccS = take(GB);
  if (any({K::FusedSliceBwd, K::FusedDesliceBwd, K::SliceBwdN, K::DesliceBwdN}))
    pl.oRed = take(nt);
  pl.total = off;
  return pl;
}

// Kernels launched by this library (fs_launch_count).
extern std::atomic<uint64_t> g_launches;

// Launch one engine kernel: dtype 0 fp32, 1 bf16, 2 fp16; nt 128 or 32;
// nblk = slot blocks for the slot-owning kinds.
cudaError_t run_engine(Kind k, int dtype, int nt, const Params& p, int nblk, cudaStream_t s);

// CTAs of kind k (dtype, nt, p's shared-memory plan) resident per SM, 0 if
// unknown.
int engine_resident(Kind k, int dtype, int nt, const Params& p);

// Fixed-order sum of per-program partials (see k_reduce).
cudaError_t run_reduce(const float* part, float* out, int B, int H, int P, int64_t E, int ob_ext,
                       int oh_ext, cudaStream_t s);

}  // namespace fs
