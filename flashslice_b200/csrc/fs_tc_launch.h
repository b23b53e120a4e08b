// flashslice_b200 -- host-side view of the tensor-core kernels
// (fs_tc_kernels.cu): parameters, kinds, TMA tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace fs {
namespace tcx {

enum class TcKind {
  SliceFwd,
  DesliceFwd,
  SliceBwd,
  DesliceBwd,
  CoupledBwd,
  BlkSliceFwd,     // blocked slot-owning slice forward, bf16 dots
  BlkSliceBwdG,    // blocked slot-owning slice backward (dW, db), bf16 dots
  BlkDesliceBwdG,  // blocked slot-owning deslice backward (dW, db, dtokens), bf16 dots
  BlkImage,        // per-(b, h, slot block) operand images of W, M, bias, ds (blocked)
  BlkSliceBwdN,    // blocked point-owning slice backward (dfx, delta, dx, dtau), bf16 dots
  BlkDesliceBwdN,  // blocked point-owning deslice backward (delta, dx, dtau), bf16 dots
  BlkDesliceFwd,   // blocked point-owning deslice forward with statistics, bf16 dots
  BlkStats,        // blocked per-point statistics (m, l), two passes, bf16 points
  BlkStatsOnline,  // the same statistics online, one pass
  SliceFwd64,      // single-tile family at G = 64 (D = DV = 32): slice forward
  DesliceFwd64,    // ... deslice forward
  CoupledBwd64,    // ... coupled backward of a round
};

constexpr int kMaxSplits = 128;  // FS_MAX_SPLITS

struct TcParams {
  CUtensorMap mx;  // x_mid: (32, H, N, B) fp32 tiles of 128 points
  CUtensorMap mv;  // fx_mid or d_out, same shape
  CUtensorMap mo;  // d_out of the coupled backward (mv is fx_mid there)
  int B, N, H, P, ntiles;
  int pdt;  // point tensors' type: 0 fp32, 1 bf16 (tiles, outputs)
  int dv, G;              // the blocked slice forward's value width and slot count
  const float* stats_in;  // its per-point statistics (B, H, 2, N)
  float* stats_out;       // the statistics kernel's output, same layout
  float* delta;           // the blocked backward's per-point delta and row sum (B, H, 2, N)
  const float* W;
  const float* bias;
  const float* tau;
  int64_t swb, swh, sbb, sbh;
  const float* M;   // tokens or dz_num (B, H, G, 32), G = 32 or 64
  const float* M2;  // dz_num of the coupled backward (M is tokens there)
  const float* ds;  // (B, H, G)
  void* out;        // deslice out / dx_mid (B, N, H, 32), element strides so
  int64_t so[4];
  void* out2;       // dfx_mid
  int64_t so2[4];
  float* partA;
  float* partB;
  float* partS;
  float* partDt;
  uint8_t* img;     // blocked point-owning kernels: operand images, one per (b, h, slot block)
  int* status;      // device word: set to a non-zero code when a bounded wait gives up
  uint64_t wait_ns;  // how long one device-side wait may take (0: the kernels' default)
  // ragged samples: nsplit = B > 0 and split[0 .. B] the row offsets of the
  // samples in the point tensors' single batch entry; 0 = dense
  int nsplit;
  int64_t split[kMaxSplits + 1];
};

cudaError_t run_tc(TcKind k, const TcParams& p, cudaStream_t s);

// Bytes of one operand image of the blocked point-owning kernels (one per
// b, h and block of 64 slots), value width dv.
constexpr int blk_image_bytes(int dv) { return 512 + 2 * 4096 + 2 * 64 * dv * 2; }

// one bounded wait that runs out (limit_ns), on `s`: sets the status word
cudaError_t run_wait_selftest(uint64_t limit_ns, cudaStream_t s);

// tensor-core kernels launched (also counted in fs::g_launches)
extern std::atomic<uint64_t> g_tc_launches;
int tc_ctas_per_sm(TcKind k);

// TMA map over a strided fp32 (B, N, H, 32) point tensor with 128-point
// boxes and 128-byte swizzle. False when the layout is not TMA-addressable
// (width stride != 1, unaligned base or strides) or the driver entry point is
// missing.
bool make_point_map(CUtensorMap* map, const void* data, int64_t B, int64_t N, int64_t H,
                    const int64_t stride[4], int pdt = 0, int width = 32);

// Address of this library's device status word on the current device.
int* device_status();

// The wait limit the next launches get (TcParams::wait_ns): 0 for the
// kernels' default; a short one lets a test make real kernels' waits run out.
extern std::atomic<uint64_t> g_wait_limit_ns;

}  // namespace tcx
}  // namespace fs
