// flashslice_b200 -- the C ABI (include/flashslice_b200.h): validation,
// engine choice, workspace carving and launch order of each op.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "flashslice_b200.h"
#include "fs_launch.h"
#include "fs_tc_launch.h"

using namespace fs;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define FS_TRY(call)                                                              \
  do {                                                                            \
    const cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess)                                                        \
      return fail(FS_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));   \
  } while (0)

int check_problem(const fs_problem* p) {
  if (!p) return fail(FS_ERR_ARGUMENT, "problem is NULL");
  if (p->B < 1 || p->H < 1 || p->N < 0 || p->G < 1)
    return fail(FS_ERR_SHAPE, "bad extents B=%lld N=%lld H=%lld G=%lld", (long long)p->B,
                (long long)p->N, (long long)p->H, (long long)p->G);
  if (p->D < 1 || p->D > 256)
    return fail(FS_ERR_UNSUPPORTED, "dim_head=%lld is outside the supported range [1, 256]",
                (long long)p->D);
  if (p->DV < 1 || p->DV > 256)
    return fail(FS_ERR_UNSUPPORTED, "value width %lld is outside the supported range [1, 256]",
                (long long)p->DV);
  if (p->N > (int64_t)1 << 30 || p->B * p->H > 65535 || (p->G + GB - 1) / GB > 65535 ||
      p->G > ((int64_t)1 << 24))
    return fail(FS_ERR_SHAPE, "extents beyond the engine's index range");
  if (p->act_dtype < 0 || p->act_dtype > 2) return fail(FS_ERR_ARGUMENT, "bad act_dtype");
  if (p->dot < 0 || p->dot > 4) return fail(FS_ERR_ARGUMENT, "bad dot level %d", p->dot);
  if (p->family != FS_FAMILY_SINGLE && p->family != FS_FAMILY_BLOCKED)
    return fail(FS_ERR_ARGUMENT, "bad family %d", p->family);
  if (p->stats_mode != 0 && p->stats_mode != 1)
    return fail(FS_ERR_ARGUMENT, "bad stats_mode %d", p->stats_mode);
  auto ext_ok = [](int32_t v, int64_t full) { return v == 1 || v == full; };
  if (!ext_ok(p->w_batch, p->B) || !ext_ok(p->w_heads, p->H))
    return fail(FS_ERR_SHAPE, "weight has (batch, heads) = (%d, %d), x_mid has (%lld, %lld)",
                p->w_batch, p->w_heads, (long long)p->B, (long long)p->H);
  if (!ext_ok(p->b_batch, p->B) || !ext_ok(p->b_heads, p->H))
    return fail(FS_ERR_SHAPE, "bias has (batch, heads) = (%d, %d), x_mid has (%lld, %lld)",
                p->b_batch, p->b_heads, (long long)p->B, (long long)p->H);
  if (p->flags < 0 || p->flags > 3) return fail(FS_ERR_ARGUMENT, "bad flags %d", p->flags);
  if (p->engine != FS_ENGINE_AUTO && p->engine != FS_ENGINE_FMA)
    return fail(FS_ERR_ARGUMENT, "bad engine %d", p->engine);
  if (p->row_splits) {
    const int64_t* r = p->row_splits;
    if (r[0] != 0 || r[p->B] != p->N)
      return fail(FS_ERR_SHAPE, "row_splits must run from 0 to N=%lld (got %lld .. %lld)",
                  (long long)p->N, (long long)r[0], (long long)r[p->B]);
    for (int64_t b = 0; b < p->B; ++b)
      if (r[b + 1] < r[b]) return fail(FS_ERR_SHAPE, "row_splits decrease at sample %lld",
                                       (long long)b);
  }
  return FS_OK;
}

// The calls below serve row splits on the tensor-core engine only.
int ragged_unsupported(const char* op) {
  return fail(FS_ERR_UNSUPPORTED,
              "%s with row_splits needs the tensor-core engine: single-tile problems with "
              "fp32 or bf16 point tensors, D = DV = 32 and G = 32 (every op) or G = 64 (slice "
              "forward, deslice forward, coupled backward), TMA-addressable point tensors, at "
              "most %d samples", op, FS_MAX_SPLITS);
}

// ---------------------------------------------------------------- tensor-core path
// The tcgen05 kernels serve the single-tile family for fp32 or bf16 point
// tensors with D = DV = 32 and G = 32 or 64 whose rows TMA can address, and
// the blocked family's bf16 shapes (blk_tc_shape). Their CTA count per
// (b, h) is a function of the shape only (148 SMs of a B200 as a constant),
// so results stay bitwise reproducible.
constexpr int kSmCount = 148;

bool tc_tensor_ok(const fs_tensor4* t) {
  if (!t || t->stride[3] != 1 || ((uintptr_t)t->data & 15)) return false;
  for (int i = 0; i < 3; ++i)
    if (t->stride[i] <= 0 || (t->stride[i] & 3)) return false;
  return true;
}

// FLASHSLICE_B200_DEBUG=1: report each op's engine choice on stderr
bool debug_routes() {
  static const int on = [] {
    const char* v = getenv("FLASHSLICE_B200_DEBUG");
    return v && v[0] == '1' ? 1 : 0;
  }();
  return on != 0;
}

void route_note(const char* op, const char* engine, const fs_problem& p, const fs_tensor4* a,
                const fs_tensor4* b2) {
  if (!debug_routes()) return;
  fprintf(stderr, "[flashslice_b200] %s -> %s (B=%lld N=%lld H=%lld D=%lld DV=%lld G=%lld "
          "dtype=%d family=%d engine=%d", op, engine, (long long)p.B, (long long)p.N,
          (long long)p.H, (long long)p.D, (long long)p.DV, (long long)p.G, p.act_dtype, p.family,
          p.engine);
  for (const fs_tensor4* t : {a, b2})
    if (t)
      fprintf(stderr, " [%p %lld %lld %lld %lld]", t->data, (long long)t->stride[0],
              (long long)t->stride[1], (long long)t->stride[2], (long long)t->stride[3]);
  fprintf(stderr, ")\n");
}

bool tc_shape(const fs_problem& p) {
  return p.engine == FS_ENGINE_AUTO && p.family == FS_FAMILY_SINGLE &&
         (p.act_dtype == FS_F32 || p.act_dtype == FS_BF16) &&
         p.D == 32 && p.DV == 32 && p.G == 32 && p.N >= 1;
}

// The G = 64 tensor-core kernels: the single-tile family with D = DV = 32
// and 64 slots (config 5's shape), fp32 or bf16 point tensors, no statistics.
bool tc64_shape(const fs_problem& p) {
  return p.engine == FS_ENGINE_AUTO && p.family == FS_FAMILY_SINGLE &&
         (p.act_dtype == FS_F32 || p.act_dtype == FS_BF16) && p.D == 32 && p.DV == 32 &&
         p.G == 64 && p.N >= 1 && !p.flags;
}

// The slot-owning slice forward on the tensor cores (shapes past the single
// tile, either family): bf16 point tensors in the bf16 dot mode (the value
// dot rounds the weights w to bf16, blocked.py), D = 32, DV = 32 or 64, G a
// multiple of 128, dense points.
bool blk_tc_shape(const fs_problem& p) {
  return p.engine == FS_ENGINE_AUTO && p.act_dtype == FS_BF16 &&
         p.dot == 3 && p.D == 32 && (p.DV == 32 || p.DV == 64) && p.G % 128 == 0 &&
         p.N >= 1 && !p.row_splits;
}

bool blk_tc_params(const fs_problem& p, const fs_tensor4* x, const fs_tensor4* v,
                   const float* W, const float* bias, const float* tau, const float* stats,
                   int max_p, tcx::TcParams& q, int ctas_per_sm = 2) {
  q = tcx::TcParams();
  q.pdt = 1;
  if (!tcx::make_point_map(&q.mx, x->data, p.B, p.N, p.H, x->stride, 2, (int)p.D) ||
      (v && !tcx::make_point_map(&q.mv, v->data, p.B, p.N, p.H, v->stride, 2, (int)p.DV)))
    return false;
  q.status = tcx::device_status();
  q.wait_ns = tcx::g_wait_limit_ns.load(std::memory_order_relaxed);
  if (!q.status) return false;
  q.B = (int)p.B;
  q.N = (int)p.N;
  q.H = (int)p.H;
  q.G = (int)p.G;
  q.dv = (int)p.DV;
  q.ntiles = (int)((p.N + 127) / 128);
  // Programs per (slot block, b, h): the fewest that fill whole waves of
  // ctas_per_sm CTAs per SM to 97% (one program per unit would leave SMs
  // idle: config 3's 128 slot blocks on 148 SMs), within the partial
  // buffers (max_p programs) and the tiles; a function of the shape only.
  const int64_t units = p.B * p.H * (p.G / 128), slots = (int64_t)ctas_per_sm * kSmCount;
  int64_t lim = max_p < q.ntiles ? max_p : q.ntiles;
  if (lim < 1) lim = 1;
  int64_t P = 1;
  double best = 0.0;
  for (int64_t c = 1; c <= lim; ++c) {
    const int64_t waves = (units * c + slots - 1) / slots;
    const double eff = (double)(units * c) / (double)(waves * slots);
    if (eff > best + 1e-9) {
      best = eff;
      P = c;
    }
    if (eff >= 0.97) break;
  }
  q.P = (int)P;
  q.W = W;
  q.bias = bias;
  q.tau = tau;
  q.stats_in = stats;
  q.swb = p.w_batch > 1 ? (int64_t)p.w_heads * p.G * p.D : 0;
  q.swh = p.w_heads > 1 ? p.G * p.D : 0;
  q.sbb = p.b_batch > 1 ? (int64_t)p.b_heads * p.G : 0;
  q.sbh = p.b_heads > 1 ? p.G : 0;
  return true;
}

// CTAs per (b, h) of the blocked point-owning tensor-core kernels: two per
// SM over all (b, h), within the dtau partial buffer (s.Pn per (b, h)).
struct Setup;
int pown_P(const fs_problem& p, const Setup& s);

// Fill the tensor-core parameters; false when a tensor map cannot be made
// (the FMA kernels then serve the call).
// TMA map of a point tensor of problem p: (B, N) rows, or with row splits
// one batch entry of N rows.
bool point_map(CUtensorMap* map, const fs_problem& p, const fs_tensor4* t) {
  return tcx::make_point_map(map, t->data, p.row_splits ? 1 : p.B, p.N, p.H, t->stride,
                             p.act_dtype == FS_BF16 ? 1 : 0);
}

bool tc_params(const fs_problem& p, tcx::TcKind k, const fs_tensor4* x, const fs_tensor4* v,
               const float* W, const float* bias, const float* tau, tcx::TcParams& q) {
  q = tcx::TcParams();
  q.pdt = p.act_dtype == FS_BF16 ? 1 : 0;
  if (p.row_splits) {
    if (p.B > tcx::kMaxSplits) return false;
    q.nsplit = (int)p.B;
    for (int64_t b = 0; b <= p.B; ++b) q.split[b] = p.row_splits[b];
  }
  if (!point_map(&q.mx, p, x)) {
    if (debug_routes()) fprintf(stderr, "[flashslice_b200] tensor map of x_mid refused\n");
    return false;
  }
  if (v && !point_map(&q.mv, p, v)) {
    if (debug_routes()) fprintf(stderr, "[flashslice_b200] tensor map of the value tensor refused\n");
    return false;
  }
  q.status = tcx::device_status();
  q.wait_ns = tcx::g_wait_limit_ns.load(std::memory_order_relaxed);
  if (!q.status) {
    if (debug_routes()) fprintf(stderr, "[flashslice_b200] no device status word\n");
    return false;
  }
  q.B = (int)p.B;
  q.N = (int)p.N;
  q.H = (int)p.H;
  q.ntiles = (int)((p.N + 127) / 128);
  const int64_t BH = p.B * p.H;
  // CTAs per (b, h): as many as fill the co-resident slots of all SMs without
  // going over (a CTA past them would run in a second wave after the others)
  int64_t P = tcx::tc_ctas_per_sm(k) * kSmCount / BH;
  if (P > q.ntiles) P = q.ntiles;
  q.P = (int)(P < 1 ? 1 : P);
  q.W = W;
  q.bias = bias;
  q.tau = tau;
  q.swb = p.w_batch > 1 ? (int64_t)p.w_heads * p.G * p.D : 0;
  q.swh = p.w_heads > 1 ? p.G * p.D : 0;
  q.sbb = p.b_batch > 1 ? (int64_t)p.b_heads * p.G : 0;
  q.sbh = p.b_heads > 1 ? p.G : 0;
  return true;
}

constexpr int kBlkTcMaxP = 16;

struct Setup {
  bool fused;
  int nt, ntiles, ngb, Pn, Pg, Pgb, BH;
  bool internal_stats;
  size_t stats, delta, partA, partB, partS, partDt, total;
  bool has_img;  // operand images of the blocked point-owning tensor-core kernels
  size_t img;
};

int pown_P(const fs_problem& p, const Setup& s) {
  int64_t P = 2 * kSmCount / ((int64_t)p.B * p.H);
  if (P > s.Pn) P = s.Pn;
  if (P > s.ntiles) P = s.ntiles;
  return (int)(P < 1 ? 1 : P);
}

Setup setup(int op, const fs_problem& p) {
  Setup s = {};
  const int D = (int)p.D, DV = (int)p.DV, G = (int)p.G;
  s.BH = (int)(p.B * p.H);
  s.nt = (round4(D) <= 64 && round4(DV) <= 64) ? 128 : 32;
  s.fused = p.family == FS_FAMILY_SINGLE && G <= GB && s.nt == 128;
  s.ntiles = (int)((p.N + s.nt - 1) / s.nt);
  s.ngb = (G + GB - 1) / GB;
  auto clampP = [&](int64_t want) {
    int64_t v = want < s.ntiles ? want : s.ntiles;
    return (int)(v < 1 ? 1 : v);
  };
  s.Pn = clampP((kTargetCtas + s.BH - 1) / s.BH);
  s.Pg = clampP((kTargetCtas + (int64_t)s.BH * s.ngb - 1) / ((int64_t)s.BH * s.ngb));
  // the blocked tensor-core slot-owning kernels pick up to kBlkTcMaxP programs
  // per slot block (to fill whole waves); their partials need room for them
  const int Pgb = s.Pgb = blk_tc_shape(p) && s.Pg < kBlkTcMaxP ? clampP(kBlkTcMaxP) : s.Pg;
  const bool has_in = p.flags & FS_FLAG_STATS_IN;
  const bool has_out = p.flags & FS_FLAG_STATS_OUT;
  size_t off = 0;
  auto take = [&](int64_t floats) {
    const size_t o = off;
    off += ((size_t)floats * sizeof(float) + 255) & ~(size_t)255;
    return o;
  };
  const int64_t BH = s.BH;
  switch (op) {
    case FS_OP_SLICE_FWD:
      if (s.fused) {
        s.partA = take(BH * s.Pn * G * DV);
        s.partS = take(BH * s.Pn * G);
      } else {
        s.internal_stats = !has_in && !(p.family == FS_FAMILY_BLOCKED && has_out);
        s.partA = take(BH * Pgb * G * DV);
        s.partS = take(BH * Pgb * G);
      }
      break;
    case FS_OP_DESLICE_FWD:
      if (!s.fused) s.internal_stats = !has_in && !(p.family == FS_FAMILY_BLOCKED && has_out);
      break;
    case FS_OP_SLICE_BWD:
    case FS_OP_DESLICE_BWD: {
      const bool sl = op == FS_OP_SLICE_BWD;
      if (s.fused) {
        s.partA = take(BH * s.Pn * G * D);
        if (!sl) s.partB = take(BH * s.Pn * G * DV);
        s.partS = take(BH * s.Pn * G);
        s.partDt = take(BH * s.Pn);
      } else {
        s.internal_stats = !has_in;
        s.delta = take(BH * 2 * p.N);
        s.partDt = take(BH * s.Pn);
        s.partA = take(BH * Pgb * G * D);
        if (!sl) s.partB = take(BH * Pgb * G * DV);
        s.partS = take(BH * Pgb * G);
      }
      break;
    }
    default:
      break;
  }
  if (s.internal_stats) s.stats = take(BH * 2 * p.N);
  if (!s.fused && blk_tc_shape(p) &&
      (op == FS_OP_SLICE_FWD || op == FS_OP_DESLICE_FWD || op == FS_OP_SLICE_BWD ||
       op == FS_OP_DESLICE_BWD)) {
    s.has_img = true;
    s.img = take(BH * (G / 64) * (int64_t)tcx::blk_image_bytes(DV) / 4);
  }
  s.total = off;
  return s;
}

Params base_params(const fs_problem& p, const Setup& s, const float* W, const float* bias,
                   const float* tau) {
  Params q = {};
  q.B = (int)p.B; q.N = (int)p.N; q.H = (int)p.H;
  q.D = (int)p.D; q.DV = (int)p.DV; q.G = (int)p.G;
  q.ntiles = s.ntiles;
  q.W = W; q.bias = bias; q.tau = tau;
  q.swb = p.w_batch > 1 ? (int64_t)p.w_heads * p.G * p.D : 0;
  q.swh = p.w_heads > 1 ? p.G * p.D : 0;
  q.sbb = p.b_batch > 1 ? (int64_t)p.b_heads * p.G : 0;
  q.sbh = p.b_heads > 1 ? p.G : 0;
  return q;
}

Pt pt(const fs_tensor4* t) {
  Pt r;
  r.data = t ? t->data : nullptr;
  r.sb = t ? t->stride[0] : 0;
  r.sn = t ? t->stride[1] : 0;
  r.sh = t ? t->stride[2] : 0;
  r.sw = t ? t->stride[3] : 0;
  return r;
}

int check_ws(const Setup& s, void* ws, size_t bytes) {
  if (s.total == 0) return FS_OK;
  if (!ws) return fail(FS_ERR_WORKSPACE, "workspace of %zu bytes needed, got NULL", s.total);
  if (bytes < s.total)
    return fail(FS_ERR_WORKSPACE, "workspace of %zu bytes needed, got %zu", s.total, bytes);
  if ((uintptr_t)ws % 256) return fail(FS_ERR_WORKSPACE, "workspace is not 256-byte aligned");
  return FS_OK;
}

float* at(void* ws, size_t off) { return (float*)((char*)ws + off); }

int need(const void* ptr, const char* what) {
  if (!ptr) return fail(FS_ERR_ARGUMENT, "%s is NULL", what);
  return FS_OK;
}

#define FS_CHECK(expr)           \
  do {                           \
    const int rc_ = (expr);      \
    if (rc_ != FS_OK) return rc_; \
  } while (0)

// Launch kind k with at most P programs per (b, h) (per slot block for the
// slot-owning kinds): as many as fill the SMs' resident slots in one wave
// (a second, partial wave would leave most SMs idle while it runs). P comes
// back as the count used; the partials' reduction takes that count.
int launch_kind(Kind k, const fs_problem& p, const Setup& s, Params q, int& P, cudaStream_t st) {
  q.pl = make_plan(k, (int)p.D, (int)p.DV, s.nt);
  const bool slot_owning = k == Kind::SliceFwdG || k == Kind::SliceBwdG || k == Kind::DesliceBwdG;
  const int64_t per = (int64_t)s.BH * (slot_owning ? s.ngb : 1);
  const int fit = engine_resident(k, p.act_dtype, s.nt, q);
  if (fit > 0) {
    const int64_t want = (int64_t)fit * kSmCount / per;
    if (want >= 1 && want < P) P = (int)want;
  }
  q.P = P;
  FS_TRY(run_engine(k, p.act_dtype, s.nt, q, s.ngb, st));
  return FS_OK;
}

// The per-point statistics: on the tensor cores when the shape allows and
// the op's workspace holds operand images, else on the FMA engine.
int run_stats(const fs_problem& p, const Setup& s, const fs_tensor4* x, const float* W,
              const float* bias, const float* tau, float* dst, cudaStream_t st,
              void* workspace = nullptr) {
  tcx::TcParams tn;
  if (workspace && s.has_img && tc_tensor_ok(x) &&
      blk_tc_params(p, x, nullptr, W, bias, tau, nullptr, s.Pn, tn)) {
    tn.M = nullptr;
    tn.ds = nullptr;
    tn.img = (uint8_t*)at(workspace, s.img);
    tn.stats_out = dst;
    tn.P = pown_P(p, s);
    route_note("stats", "tensor-core-blocked", p, x, x);
    FS_TRY(tcx::run_tc(tcx::TcKind::BlkImage, tn, st));
    // the online or two-pass statistics, as the problem's stats mode asks
    FS_TRY(tcx::run_tc(p.stats_mode == 1 ? tcx::TcKind::BlkStats : tcx::TcKind::BlkStatsOnline,
                       tn, st));
    return FS_OK;
  }
  Params q = base_params(p, s, W, bias, tau);
  q.x = pt(x);
  q.stats_out = dst;
  int P = s.Pn;  // no partials: any count serves
  return launch_kind(p.stats_mode == 1 ? Kind::StatsTwoPass : Kind::StatsOnline, p, s, q, P, st);
}

}  // namespace

// ---------------------------------------------------------------------------
// Scratch for fs_slice_fwd_noalloc: a fixed device array, so that callers
// that cannot allocate device memory can still run the slice forward. It is
// created when the library is loaded on a device and lives until the process
// exits; every call shares it.
static __device__ __align__(256) float fs_noalloc_scratch[FS_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

// The device address of fs_noalloc_scratch in the calling thread's current
// context. The array's name in host code is only a host-side stand-in, and
// the address the runtime gives belongs to one context (a caller may run in
// a context of its own, or reset the device and get a new one), so it is
// asked for on every call: a host-only lookup that allocates nothing. The
// first call in a context loads this library's device code into it.
int noalloc_scratch(float** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, fs_noalloc_scratch);
  if (e != cudaSuccess || !ptr)
    return fail(FS_ERR_CUDA, "cudaGetSymbolAddress(fs_noalloc_scratch) failed: %s",
                cudaGetErrorString(e));
  *out = (float*)ptr;
  return FS_OK;
}

}  // namespace

extern "C" {

int fs_slice_fwd_noalloc(const fs_problem* p, const fs_tensor4* x_mid, const fs_tensor4* fx_mid,
                         const float* weight, const float* bias, const float* tau, float* z_num,
                         float* s_out, void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(fx_mid, "fx_mid"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(z_num, "z_num"));
  FS_CHECK(need(s_out, "s"));
  if (p->flags != 0) return fail(FS_ERR_ARGUMENT, "fs_slice_fwd_noalloc takes no statistics");
  if (p->row_splits) return ragged_unsupported("fs_slice_fwd_noalloc");
  const Setup s = setup(FS_OP_SLICE_FWD, *p);
  if (!s.fused)
    return fail(FS_ERR_UNSUPPORTED,
                "fs_slice_fwd_noalloc serves the single-tile family with G <= 32 and "
                "D, DV <= 64 only (G=%lld, D=%lld, DV=%lld)",
                (long long)p->G, (long long)p->D, (long long)p->DV);
  if (s.total > (size_t)FS_NOALLOC_SCRATCH_BYTES)
    return fail(FS_ERR_UNSUPPORTED,
                "fs_slice_fwd_noalloc: this problem needs %zu bytes of scratch, the static "
                "scratch holds %zu; use fs_slice_fwd with a workspace",
                s.total, (size_t)FS_NOALLOC_SCRATCH_BYTES);
  float* base = nullptr;
  FS_CHECK(noalloc_scratch(&base));
  cudaStream_t st = (cudaStream_t)stream;
  Params q = base_params(*p, s, weight, bias, tau);
  q.x = pt(x_mid);
  q.v = pt(fx_mid);
  q.partA = at(base, s.partA);
  q.partS = at(base, s.partS);
  int P = s.Pn;
  FS_CHECK(launch_kind(Kind::FusedSliceFwd, *p, s, q, P, st));
  FS_TRY(run_reduce(q.partA, z_num, s.BH, 1, P, p->G * p->DV, s.BH, 1, st));
  FS_TRY(run_reduce(q.partS, s_out, s.BH, 1, P, p->G, s.BH, 1, st));
  return FS_OK;
}

int fs_version(void) { return FS_ABI_VERSION; }

const char* fs_last_error(void) { return g_err.c_str(); }

uint64_t fs_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

uint64_t fs_tc_launch_count(void) { return tcx::g_tc_launches.load(std::memory_order_relaxed); }

int fs_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns > 2000000000ull)
    return fail(FS_ERR_ARGUMENT, "wait limit %llu ns is above the default 2e9",
                (unsigned long long)limit_ns);
  tcx::g_wait_limit_ns.store(limit_ns, std::memory_order_relaxed);
  return FS_OK;
}

int fs_device_status(int reset) {
  int* word = tcx::device_status();
  if (!word) return -1;
  if (cudaDeviceSynchronize() != cudaSuccess) return -2;
  int v = 0;
  if (cudaMemcpy(&v, word, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -3;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpy(word, &zero, sizeof zero, cudaMemcpyHostToDevice) != cudaSuccess) return -4;
  }
  return v;
}

int fs_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 2000000000ull)
    return fail(FS_ERR_ARGUMENT, "limit_ns must be in (0, 2e9], got %llu",
                (unsigned long long)limit_ns);
  FS_TRY(tcx::run_wait_selftest(limit_ns, (cudaStream_t)stream));
  return FS_OK;
}

size_t fs_workspace_bytes(int op, const fs_problem* p) {
  if (check_problem(p) != FS_OK) return 0;
  return setup(op, *p).total;
}

int fs_compute_stats(const fs_problem* p, const fs_tensor4* x_mid, const float* weight,
                     const float* bias, const float* tau, float* stats, void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(stats, "stats"));
  if (p->row_splits) return ragged_unsupported("statistics");
  const Setup s = setup(FS_OP_STATS, *p);
  return run_stats(*p, s, x_mid, weight, bias, tau, stats, (cudaStream_t)stream);
}

int fs_rank_sum(const float* parts, float* out, int world, int64_t n, void* stream) {
  if (!parts || !out) return fail(FS_ERR_ARGUMENT, "rank_sum: null pointer");
  if (world < 1 || n < 0) return fail(FS_ERR_ARGUMENT, "rank_sum: world %d, n %lld", world,
                                      (long long)n);
  if (n == 0) return FS_OK;
  FS_TRY(run_reduce(parts, out, 1, 1, world, n, 1, 1, (cudaStream_t)stream));
  return FS_OK;
}

int fs_slice_fwd(const fs_problem* p, const fs_tensor4* x_mid, const fs_tensor4* fx_mid,
                 const float* weight, const float* bias, const float* tau, const float* stats_in,
                 float* stats_out, float* z_num, float* s_out, void* workspace,
                 size_t workspace_bytes, void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(fx_mid, "fx_mid"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(z_num, "z_num"));
  FS_CHECK(need(s_out, "s"));
  if (!!stats_in != !!(p->flags & FS_FLAG_STATS_IN) ||
      !!stats_out != !!(p->flags & FS_FLAG_STATS_OUT))
    return fail(FS_ERR_ARGUMENT, "stats pointers disagree with problem flags");
  const Setup s = setup(FS_OP_SLICE_FWD, *p);
  FS_CHECK(check_ws(s, workspace, workspace_bytes));
  cudaStream_t st = (cudaStream_t)stream;
  Params q = base_params(*p, s, weight, bias, tau);
  q.x = pt(x_mid);
  q.v = pt(fx_mid);
  q.partA = at(workspace, s.partA);
  q.partS = at(workspace, s.partS);
  int P;
  tcx::TcParams tq;
  if (s.fused && tc_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(fx_mid) &&
      tc_params(*p, tcx::TcKind::SliceFwd, x_mid, fx_mid, weight, bias, tau, tq)) {
    // the partial buffers sized for the FMA kernels hold the (fewer) tensor-core CTAs'
    tq.partA = q.partA;
    tq.partS = q.partS;
    P = tq.P;
    route_note("slice_fwd", "tensor-core", *p, x_mid, fx_mid);
    FS_TRY(tcx::run_tc(tcx::TcKind::SliceFwd, tq, st));
  } else if (tc64_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(fx_mid) &&
             tc_params(*p, tcx::TcKind::SliceFwd64, x_mid, fx_mid, weight, bias, tau, tq)) {
    // partials of the slot-blocked layout: at most s.Pg programs per (b, h)
    if (tq.P > s.Pg) tq.P = s.Pg;
    tq.partA = q.partA;
    tq.partS = q.partS;
    P = tq.P;
    route_note("slice_fwd", "tensor-core-g64", *p, x_mid, fx_mid);
    FS_TRY(tcx::run_tc(tcx::TcKind::SliceFwd64, tq, st));
  } else if (p->row_splits) {
    return ragged_unsupported("slice forward");
  } else if (s.fused) {
    P = s.Pn;
    route_note("slice_fwd", "fma-fused", *p, x_mid, fx_mid);
    FS_CHECK(launch_kind(Kind::FusedSliceFwd, *p, s, q, P, st));
  } else {
    const float* stats = stats_in;
    if (!stats) {
      float* dst = s.internal_stats ? at(workspace, s.stats) : stats_out;
      FS_CHECK(run_stats(*p, s, x_mid, weight, bias, tau, dst, st, workspace));
      stats = dst;
    }
    q.stats_in = stats;
    tcx::TcParams tb;
    if (blk_tc_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(fx_mid) &&
        blk_tc_params(*p, x_mid, fx_mid, weight, bias, tau, stats, s.Pgb, tb)) {
      // the partial buffers sized for the FMA kernels hold the (fewer) CTAs'
      tb.partA = q.partA;
      tb.partS = q.partS;
      P = tb.P;
      route_note("slice_fwd", "tensor-core-blocked", *p, x_mid, fx_mid);
      FS_TRY(tcx::run_tc(tcx::TcKind::BlkSliceFwd, tb, st));
    } else {
      P = s.Pg;
      FS_CHECK(launch_kind(Kind::SliceFwdG, *p, s, q, P, st));
    }
  }
  const int BH = s.BH;
  FS_TRY(run_reduce(q.partA, z_num, BH, 1, P, p->G * p->DV, BH, 1, st));
  FS_TRY(run_reduce(q.partS, s_out, BH, 1, P, p->G, BH, 1, st));
  return FS_OK;
}

int fs_deslice_fwd(const fs_problem* p, const fs_tensor4* x_mid, const float* weight,
                   const float* bias, const float* tau, const float* tokens,
                   const float* stats_in, float* stats_out, const fs_tensor4* out,
                   void* workspace, size_t workspace_bytes, void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(tokens, "tokens"));
  FS_CHECK(need(out, "out"));
  if (!!stats_in != !!(p->flags & FS_FLAG_STATS_IN) ||
      !!stats_out != !!(p->flags & FS_FLAG_STATS_OUT))
    return fail(FS_ERR_ARGUMENT, "stats pointers disagree with problem flags");
  const Setup s = setup(FS_OP_DESLICE_FWD, *p);
  FS_CHECK(check_ws(s, workspace, workspace_bytes));
  cudaStream_t st = (cudaStream_t)stream;
  Params q = base_params(*p, s, weight, bias, tau);
  q.x = pt(x_mid);
  q.o1 = pt(out);
  q.M = tokens;
  tcx::TcParams tq;
  if (s.fused && tc_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(out) &&
      tc_params(*p, tcx::TcKind::DesliceFwd, x_mid, nullptr, weight, bias, tau, tq)) {
    tq.M = tokens;
    tq.out = (float*)out->data;
    for (int i = 0; i < 4; ++i) tq.so[i] = out->stride[i];
    route_note("deslice_fwd", "tensor-core", *p, x_mid, out);
    FS_TRY(tcx::run_tc(tcx::TcKind::DesliceFwd, tq, st));
    return FS_OK;
  }
  if (tc64_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(out) &&
      tc_params(*p, tcx::TcKind::DesliceFwd64, x_mid, nullptr, weight, bias, tau, tq)) {
    tq.M = tokens;
    tq.out = out->data;
    for (int i = 0; i < 4; ++i) tq.so[i] = out->stride[i];
    route_note("deslice_fwd", "tensor-core-g64", *p, x_mid, out);
    FS_TRY(tcx::run_tc(tcx::TcKind::DesliceFwd64, tq, st));
    return FS_OK;
  }
  if (p->row_splits) return ragged_unsupported("deslice forward");
  int P = s.Pn;  // no partials: any count serves
  // the blocked deslice with statistics: point-owning tensor-core kernel when
  // the shape allows, else the FMA kernel
  auto with_stats = [&](const float* stats) -> int {
    tcx::TcParams tn;
    if (s.has_img && tc_tensor_ok(x_mid) && tc_tensor_ok(out) &&
        blk_tc_params(*p, x_mid, out, weight, bias, tau, stats, s.Pn, tn)) {
      tn.M = tokens;
      tn.ds = nullptr;
      tn.img = (uint8_t*)at(workspace, s.img);
      tn.out = out->data;
      for (int i = 0; i < 4; ++i) tn.so[i] = out->stride[i];
      tn.P = pown_P(*p, s);
      route_note("deslice_fwd", "tensor-core-blocked", *p, x_mid, out);
      FS_TRY(tcx::run_tc(tcx::TcKind::BlkImage, tn, st));
      FS_TRY(tcx::run_tc(tcx::TcKind::BlkDesliceFwd, tn, st));
      return FS_OK;
    }
    route_note("deslice_fwd", "fma-blocked", *p, x_mid, out);
    q.stats_in = stats;
    return launch_kind(Kind::DesliceFwdStats, *p, s, q, P, st);
  };
  if (s.fused) {
    route_note("deslice_fwd", "fma-fused", *p, x_mid, out);
    return launch_kind(Kind::FusedDesliceFwd, *p, s, q, P, st);
  }
  if (stats_in) return with_stats(stats_in);
  float* dst = s.internal_stats ? at(workspace, s.stats) : stats_out;
  // Online statistics: formed in the same pass as out on the FMA engine; on
  // the tensor cores, by the online statistics kernel and then the deslice
  // with them (two passes over x_mid, each far faster).
  const bool blk_tc = s.has_img && tc_tensor_ok(x_mid) && tc_tensor_ok(out);
  if (p->stats_mode == 0 && !blk_tc) {
    route_note("deslice_fwd", "fma-blocked", *p, x_mid, out);
    q.stats_out = dst;
    return launch_kind(Kind::DesliceFwdOnline, *p, s, q, P, st);
  }
  FS_CHECK(run_stats(*p, s, x_mid, weight, bias, tau, dst, st, workspace));
  return with_stats(dst);
}

static int bwd_common(bool slice, const fs_problem* p, const fs_tensor4* x_mid,
                      const fs_tensor4* vals, const float* weight, const float* bias,
                      const float* tau, const float* mat, const float* ds, const float* stats_in,
                      const fs_tensor4* dx, const fs_tensor4* dfx, float* dtok, float* dW,
                      float* db, float* dtau, void* workspace, size_t workspace_bytes,
                      void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(vals, slice ? "fx_mid" : "d_out"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(mat, slice ? "dz_num" : "tokens"));
  FS_CHECK(need(dx, "dx_mid"));
  FS_CHECK(need(dW, "dW"));
  FS_CHECK(need(db, "db"));
  FS_CHECK(need(dtau, "dtau"));
  if (slice) {
    FS_CHECK(need(ds, "ds"));
    FS_CHECK(need(dfx, "dfx_mid"));
  } else {
    FS_CHECK(need(dtok, "dtokens"));
  }
  if (!!stats_in != !!(p->flags & FS_FLAG_STATS_IN) || (p->flags & FS_FLAG_STATS_OUT))
    return fail(FS_ERR_ARGUMENT, "stats pointers disagree with problem flags");
  if (p->family == FS_FAMILY_BLOCKED && !stats_in)
    return fail(FS_ERR_ARGUMENT, "the blocked backward needs the forward's statistics");
  const Setup s = setup(slice ? FS_OP_SLICE_BWD : FS_OP_DESLICE_BWD, *p);
  FS_CHECK(check_ws(s, workspace, workspace_bytes));
  cudaStream_t st = (cudaStream_t)stream;
  Params q = base_params(*p, s, weight, bias, tau);
  q.x = pt(x_mid);
  q.v = pt(vals);
  q.o1 = pt(dx);
  if (slice) q.o2 = pt(dfx);
  q.M = mat;
  q.ds = ds;
  q.partA = at(workspace, s.partA);
  if (!slice) q.partB = at(workspace, s.partB);
  q.partS = at(workspace, s.partS);
  q.partDt = at(workspace, s.partDt);
  int Pw, Pdt = s.Pn;
  tcx::TcParams tq;
  if (s.fused && tc_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(vals) &&
      tc_tensor_ok(dx) && (!slice || tc_tensor_ok(dfx)) &&
      tc_params(*p, slice ? tcx::TcKind::SliceBwd : tcx::TcKind::DesliceBwd, x_mid, vals, weight,
                bias, tau, tq)) {
    // the partial buffers sized for the FMA kernels hold the (fewer) tensor-core CTAs'
    tq.M = mat;
    tq.ds = ds;
    tq.out = (float*)dx->data;
    for (int i = 0; i < 4; ++i) tq.so[i] = dx->stride[i];
    if (slice) {
      tq.out2 = (float*)dfx->data;
      for (int i = 0; i < 4; ++i) tq.so2[i] = dfx->stride[i];
    }
    tq.partA = q.partA;
    tq.partB = q.partB;
    tq.partS = q.partS;
    tq.partDt = q.partDt;
    Pw = Pdt = tq.P;
    route_note(slice ? "slice_bwd" : "deslice_bwd", "tensor-core", *p, x_mid, vals);
    FS_TRY(tcx::run_tc(slice ? tcx::TcKind::SliceBwd : tcx::TcKind::DesliceBwd, tq, st));
  } else if (p->row_splits) {
    return ragged_unsupported(slice ? "slice backward" : "deslice backward");
  } else if (s.fused) {
    Pw = s.Pn;
    if (debug_routes())
      fprintf(stderr, "[flashslice_b200] shape %d x %d vals %d dx %d dfx %d\n", (int)tc_shape(*p),
              (int)tc_tensor_ok(x_mid), (int)tc_tensor_ok(vals), (int)tc_tensor_ok(dx),
              (int)(!slice || tc_tensor_ok(dfx)));
    route_note(slice ? "slice_bwd" : "deslice_bwd", "fma-fused", *p, x_mid, dx);
    FS_CHECK(launch_kind(slice ? Kind::FusedSliceBwd : Kind::FusedDesliceBwd, *p, s, q, Pw, st));
    Pdt = Pw;
  } else {
    const float* stats = stats_in;
    if (!stats) {
      float* dst = at(workspace, s.stats);
      FS_CHECK(run_stats(*p, s, x_mid, weight, bias, tau, dst, st, workspace));
      stats = dst;
    }
    q.stats_in = stats;
    q.delta = at(workspace, s.delta);
    tcx::TcParams tb;
    const bool blk_tc = blk_tc_shape(*p) && tc_tensor_ok(x_mid) && tc_tensor_ok(vals) &&
                        blk_tc_params(*p, x_mid, vals, weight, bias, tau, stats, s.Pgb, tb, 1);
    if (blk_tc && s.has_img && tc_tensor_ok(dx) && (!slice || tc_tensor_ok(dfx))) {
      tcx::TcParams tn = tb;
      tn.M = mat;
      tn.ds = slice ? ds : nullptr;
      tn.delta = q.delta;
      tn.img = (uint8_t*)at(workspace, s.img);
      tn.out = dx->data;
      for (int i = 0; i < 4; ++i) tn.so[i] = dx->stride[i];
      if (slice) {
        tn.out2 = dfx->data;
        for (int i = 0; i < 4; ++i) tn.so2[i] = dfx->stride[i];
      }
      tn.partDt = q.partDt;
      tn.P = Pdt = pown_P(*p, s);
      route_note(slice ? "slice_bwd (point-owning)" : "deslice_bwd (point-owning)",
                 "tensor-core-blocked", *p, x_mid, vals);
      FS_TRY(tcx::run_tc(tcx::TcKind::BlkImage, tn, st));
      FS_TRY(tcx::run_tc(slice ? tcx::TcKind::BlkSliceBwdN : tcx::TcKind::BlkDesliceBwdN, tn, st));
    } else {
      FS_CHECK(launch_kind(slice ? Kind::SliceBwdN : Kind::DesliceBwdN, *p, s, q, Pdt, st));
    }
    if (blk_tc) {
      tb.M = mat;
      tb.ds = ds;
      tb.delta = q.delta;
      tb.partA = q.partA;
      tb.partB = q.partB;
      tb.partS = q.partS;
      Pw = tb.P;
      route_note(slice ? "slice_bwd (slot-owning)" : "deslice_bwd (slot-owning)",
                 "tensor-core-blocked", *p, x_mid, vals);
      FS_TRY(tcx::run_tc(slice ? tcx::TcKind::BlkSliceBwdG : tcx::TcKind::BlkDesliceBwdG, tb, st));
    } else {
      Pw = s.Pg;
      FS_CHECK(launch_kind(slice ? Kind::SliceBwdG : Kind::DesliceBwdG, *p, s, q, Pw, st));
    }
  }
  const int B = (int)p->B, H = (int)p->H, BH = s.BH;
  FS_TRY(run_reduce(q.partA, dW, B, H, Pw, p->G * p->D, p->w_batch, p->w_heads, st));
  FS_TRY(run_reduce(q.partS, db, B, H, Pw, p->G, p->b_batch, p->b_heads, st));
  if (!slice) FS_TRY(run_reduce(q.partB, dtok, BH, 1, Pw, p->G * p->DV, BH, 1, st));
  FS_TRY(run_reduce(q.partDt, dtau, B, H, Pdt, 1, 1, H, st));
  return FS_OK;
}

int fs_slice_bwd(const fs_problem* p, const fs_tensor4* x_mid, const fs_tensor4* fx_mid,
                 const float* weight, const float* bias, const float* tau, const float* stats_in,
                 const float* dz_num, const float* ds, const fs_tensor4* dx_mid,
                 const fs_tensor4* dfx_mid, float* dW, float* db, float* dtau, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return bwd_common(true, p, x_mid, fx_mid, weight, bias, tau, dz_num, ds, stats_in, dx_mid,
                    dfx_mid, nullptr, dW, db, dtau, workspace, workspace_bytes, stream);
}

int fs_deslice_bwd(const fs_problem* p, const fs_tensor4* x_mid, const float* weight,
                   const float* bias, const float* tau, const float* tokens,
                   const float* stats_in, const fs_tensor4* d_out, const fs_tensor4* dx_mid,
                   float* dtokens, float* dW, float* db, float* dtau, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return bwd_common(false, p, x_mid, d_out, weight, bias, tau, tokens, nullptr, stats_in, dx_mid,
                    nullptr, dtokens, dW, db, dtau, workspace, workspace_bytes, stream);
}

int fs_coupled_supported(const fs_problem* p) {
  if (check_problem(p) != FS_OK) return 0;
  const bool tc32 = setup(FS_OP_SLICE_BWD, *p).fused && tc_shape(*p);
  return (tc32 || tc64_shape(*p)) && !p->flags && (!p->row_splits || p->B <= FS_MAX_SPLITS)
             ? 1
             : 0;
}

int fs_coupled_bwd(const fs_problem* p, const fs_tensor4* x_mid, const fs_tensor4* fx_mid,
                   const fs_tensor4* d_out, const float* weight, const float* bias,
                   const float* tau, const float* tokens, const float* dz_num, const float* ds,
                   const fs_tensor4* dx_mid, const fs_tensor4* dfx_mid, float* dW, float* db,
                   float* dtau, void* workspace, size_t workspace_bytes, void* stream) {
  FS_CHECK(check_problem(p));
  FS_CHECK(need(x_mid, "x_mid"));
  FS_CHECK(need(fx_mid, "fx_mid"));
  FS_CHECK(need(d_out, "d_out"));
  FS_CHECK(need(weight, "weight"));
  FS_CHECK(need(bias, "bias"));
  FS_CHECK(need(tau, "tau"));
  FS_CHECK(need(tokens, "tokens"));
  FS_CHECK(need(dz_num, "dz_num"));
  FS_CHECK(need(ds, "ds"));
  FS_CHECK(need(dx_mid, "dx_mid"));
  FS_CHECK(need(dfx_mid, "dfx_mid"));
  FS_CHECK(need(dW, "dW"));
  FS_CHECK(need(db, "db"));
  FS_CHECK(need(dtau, "dtau"));
  if (p->flags) return fail(FS_ERR_ARGUMENT, "the coupled backward takes no statistics");
  const Setup s = setup(FS_OP_SLICE_BWD, *p);
  FS_CHECK(check_ws(s, workspace, workspace_bytes));
  const bool g64 = tc64_shape(*p);
  if (!((g64 || (s.fused && tc_shape(*p))) && tc_tensor_ok(x_mid) && tc_tensor_ok(fx_mid) &&
        tc_tensor_ok(d_out) && tc_tensor_ok(dx_mid) && tc_tensor_ok(dfx_mid)))
    return fail(FS_ERR_UNSUPPORTED,
                "the coupled backward serves single-tile problems with D = DV = 32 and G = 32 "
                "or 64 (engine auto, fp32 or bf16 points) and point tensors of unit width "
                "stride and 16-byte aligned strides");
  const tcx::TcKind kind = g64 ? tcx::TcKind::CoupledBwd64 : tcx::TcKind::CoupledBwd;
  tcx::TcParams tq;
  if (!tc_params(*p, kind, x_mid, fx_mid, weight, bias, tau, tq) ||
      !point_map(&tq.mo, *p, d_out))
    return fail(FS_ERR_UNSUPPORTED, "no TMA tensor map for the point tensors");
  if (g64) {
    // one CTA per SM: two whole waves (B H P = 2 x 148 when B H divides it)
    // leave no SM idle where one wave of 148 / (B H) programs would; within
    // the tiles and the partials of the slot-blocked layout
    int64_t P = 2 * kSmCount / ((int64_t)p->B * p->H);
    if (P > tq.ntiles) P = tq.ntiles;
    if (P > s.Pg) P = s.Pg;
    if (P > s.Pn) P = s.Pn;
    tq.P = (int)(P < 1 ? 1 : P);
  }
  cudaStream_t st = (cudaStream_t)stream;
  tq.M = tokens;
  tq.M2 = dz_num;
  tq.ds = ds;
  tq.out = (float*)dx_mid->data;
  tq.out2 = (float*)dfx_mid->data;
  for (int i = 0; i < 4; ++i) {
    tq.so[i] = dx_mid->stride[i];
    tq.so2[i] = dfx_mid->stride[i];
  }
  // the partial buffers sized for the FMA kernels hold the (fewer) tensor-core CTAs'
  tq.partA = at(workspace, s.partA);
  tq.partS = at(workspace, s.partS);
  tq.partDt = at(workspace, s.partDt);
  route_note("coupled_bwd", g64 ? "tensor-core-g64" : "tensor-core", *p, x_mid, d_out);
  FS_TRY(tcx::run_tc(kind, tq, st));
  const int B = (int)p->B, H = (int)p->H, P = tq.P;
  FS_TRY(run_reduce(tq.partA, dW, B, H, P, p->G * p->D, p->w_batch, p->w_heads, st));
  FS_TRY(run_reduce(tq.partS, db, B, H, P, p->G, p->b_batch, p->b_heads, st));
  FS_TRY(run_reduce(tq.partDt, dtau, B, H, P, 1, 1, H, st));
  return FS_OK;
}

}  // extern "C"
