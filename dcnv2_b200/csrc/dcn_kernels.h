// Kernel argument blocks and launchers shared between the API layer and the kernels.
#pragma once
#include <cuda_runtime.h>

#include <utility>

#include "dcn_plan.h"

namespace dcn {

// Study builds (-DDCN_STUDY, never the shipped library) honour measurement
// switches: DCN_DEBUG_SKIP drops parts of the kernels' work (results are then
// wrong), DCN_DEBUG_TS records per-stage timestamps of CTA 0, DCN_FWD_STAGES /
// DCN_FWD_CARVE / DCN_GOUT_PACKED change launch choices.  A normal build compiles
// all of that out: the kernels cannot skip work whatever the environment holds.
#ifdef DCN_STUDY
#define DCN_STUDY_ON 1
#else
#define DCN_STUDY_ON 0
#endif
// true when study bit `bit` of the launch's skip mask is set (always false in a normal build)
#define DCN_SKIP(bit) (DCN_STUDY_ON && (a.dbg & (bit)))

constexpr int kMaxStages = 12;
constexpr int kMaxASlots = 16;
constexpr size_t kFwdSmemBudget = 218 * 1024;  // dynamic smem of the forward kernel
constexpr size_t kBwdSmemBudget = 200 * 1024;
constexpr size_t kBwdSmemLimit = 226 * 1024;  // backward-data ring + transpose buffer

// Opaque 128-byte TMA tensor map (CUtensorMap), passed by value in kernel arguments.
struct alignas(64) TmaDesc {
  unsigned long long v[16];
};

struct FwdArgs {
  Plan plan;
  unsigned long long* ts;  // optional pipeline timestamps of CTA 0 (DCN_DEBUG_TS), else null
  const void* xt;       // packed NHWC input [B][H][W][dg][Cgp]
  const void* offset;   // [B][dg*2*K2][Ho][Wo]
  const void* mask;     // [B][dg*K2][Ho][Wo]
  const uint8_t* wpk;   // packed weight tiles [nCoT][nK][NT x 128 B x nsplit]
  const void* bias;     // [Co] or nullptr
  void* out;            // [B][Co][Ho][Wo]
  int vec_out;          // out is 16-byte aligned
  int* err;             // device error word
  int stages;
  int geo_bufs;         // geometry windows: 2 built by the epilogue warps, 1 by the producers
  int mma_bias;         // bias added by an extra K = 16 MMA slice (set by the launcher)
  int num_sms;
  int dbg;              // experiment switches (DCN_DEBUG_SKIP); 0 in normal use
};

// BwdDataArgs::gdirect / BwdWeightArgs::gdirect: where the GEMMs' grad_output
// tiles come from.  0: packed blocks (pack_grad_output); kGoutNchw: TMA boxes
// of NCHW grad_output (64 pixels contiguous per Co row, MN-major for the
// data GEMM, K-major for the weight GEMM); kGoutNhwc: TMA boxes of
// channels-last grad_output (64 Co contiguous per pixel row: the packed
// block's layout, so the packed operand descriptors apply).
enum : int { kGoutNchw = 1, kGoutNhwc = 2 };

struct BwdDataArgs {
  TmaDesc gmap;         // grad_output box 64 x 64, SW128: NCHW as [B][Co][HoWo], channels-last
                        // as [1][totalP][Co] (gdirect)
  TmaDesc xmap;         // packed input [B][H][W][CS], box 16 x 16 pixels x 64 channels, SW128 (tile scatter)
  TmaDesc cmap;         // gcol [B][Ho][Wo][K2*dg*Cgp], box 8 x 8 pixels x 64 channels, SW128 (tile scatter)
  TmaDesc rmap;         // fp32 grad_input accumulator [B][H][W][CS], box 8 x 16 pixels x 32 channels,
                        // SW128 (tile scatter: TMA reductions of its windows)
  int gdirect;          // 0, kGoutNchw or kGoutNhwc: A tiles loaded from grad_output by TMA
                        // (no packed copy); 16-bit types, 16-byte aligned grad_output
  Plan plan;
  unsigned long long* ts;  // optional pipeline timestamps of CTA 0 (DCN_DEBUG_TS), else null
  const void* xt;       // packed NHWC input
  const void* offset;
  const void* mask;
  const void* gout;     // grad_output [B][Co][Ho][Wo]
  const uint8_t* gpk;   // packed grad_output blocks [nPB][nKo][64 x 128 B x nsplit]
  const uint8_t* wpk;   // packed W^T tiles [nU][nKo][NC x 128 B x nsplit]
  void* gcol;           // [npix][K2][dg][Cgp] column gradients of the chunk (T, f32 for f32)
  int pix0, npix;       // pixel chunk handled by this launch (pix0 % 128 == 0)
  float* gx_nhwc;       // fp32 [B][H][W][dg][Cgp], zero-initialised, accumulated by red.add
  void* goffset;        // [B][dg*2*K2][Ho][Wo]
  void* gmask;          // [B][dg*K2][Ho][Wo]
  int* err;
  int stages;
  int num_sms;
  int dbg;              // experiment switches (DCN_DEBUG_SKIP); 0 in normal use
  int a_slots;          // grad_out chunk slots in smem (set by the launcher)
  int vec_gout;         // grad_output 16-byte aligned (vector loads allowed when HoWo % 8 == 0)
  uint8_t* cols;        // sampled columns of the chunk for the weight gradient, written by the
                        // scatter: [npix/64][nsplit][nU*NC/64] 8 KB blocks of 64 pixels x 64
                        // channels (pixel rows of 128 B, SW128 swizzled; MN-major UMMA B tiles)
};

struct BwdWeightArgs {
  TmaDesc gmap;         // as BwdDataArgs::gmap
  int gdirect;          // as BwdDataArgs::gdirect; grad_bias then summed here
  float* gb;            // fp32 [Co] grad_bias accumulator (gdirect and bias), else null
  Plan plan;
  unsigned long long* ts;  // optional pipeline timestamps of CTA 0 (DCN_DEBUG_TS), else null
  const uint8_t* cols;  // sampled columns of the chunk (BwdDataArgs::cols)
  int ks0, nks;         // the chunk's first 64-pixel block and its number of blocks
  const uint8_t* gpk;   // packed grad_output blocks (as above)
  float* gw;            // fp32 [Co][K2][dg][Cgp], zero-initialised, accumulated
  int* err;
  int stages;
  int num_sms;
  int dbg;              // experiment switches (DCN_DEBUG_SKIP); 0 in normal use
};

// Programmatic dependent launch of the library's kernels (each one waits with
// griddepcontrol.wait before touching global memory); DCN_NO_PDL=1 turns it off.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Packing / finishing kernels (dcn_pack.cu)
// x NCHW -> packed NHWC xt; optionally zeroes an fp32 accumulator of xt's
// layout (`zero_acc`) and the status word (`status`) in the same pass.
int launch_pack_input(const Plan& p, const void* x, void* xt, float* zero_acc, int* status,
                      cudaStream_t s);
int launch_pack_weight_fwd(const Plan& p, const void* w, uint8_t* wpk, cudaStream_t s);
// 16-bit NCHW input (H*W % 8 == 0, 16-byte aligned) and the forward weight
// tiles packed by one launch; clears the status word
int launch_pack_forward(const Plan& p, const void* x, void* xt, int* status, const void* w, uint8_t* wpk,
                        cudaStream_t s);
// W -> backward-data B tiles; also zeroes `zero_bytes` (a multiple of 16) at
// `zero_acc` when it is not null, and the status word when `status` is not null.
int launch_pack_weight_bwd(const Plan& p, const void* w, uint8_t* wpk, float* zero_acc, size_t zero_bytes,
                           int* status, cudaStream_t s);
int launch_pack_gout(const Plan& p, const void* gout, uint8_t* gpk, float* gb, int vec,
                     cudaStream_t s);
int launch_finish_grad_input(const Plan& p, const float* gx_nhwc, void* gx, cudaStream_t s);
// NCHW grad_input and grad_weight / grad_bias finished by one launch
int launch_finish_grads(const Plan& p, const float* gx_nhwc, void* gx, const float* gw, const float* gb,
                        void* gw_out, void* gb_out, cudaStream_t s);
int launch_finish_grad_weight(const Plan& p, const float* gw, const float* gb, void* gw_out,
                              void* gb_out, cudaStream_t s);

// Main kernels
int launch_forward(const FwdArgs& a, cudaStream_t s);
int launch_backward_data(const BwdDataArgs& a, cudaStream_t s);
int launch_backward_scatter(const BwdDataArgs& a, cudaStream_t s);
// Tile path of the scatter (dcn_bwd_scatter_tc.cu): grad_input summed on the
// tensor cores over 16 x 16 input windows; needs a.xmap, a.cmap and a.rmap.
bool backward_scatter_tc_eligible(const Plan& p);
size_t backward_scatter_tc_smem(const Plan& p);
int launch_backward_scatter_tc(const BwdDataArgs& a, cudaStream_t s);
// Tensor maps of the tile scatter; false when the encoder rejects them.
bool make_scatter_tmaps(const Plan& p, const void* xt, const void* gcol, const float* gx, TmaDesc* xmap,
                        TmaDesc* cmap, TmaDesc* rmap);
int launch_backward_weight(const BwdWeightArgs& a, cudaStream_t s);

// Tensor map of grad_output [B][Co][HoWo] (16-bit) with a 64 x 64 box and the
// 128-byte swizzle; false when the driver's encoder is unavailable or rejects it.
bool make_gout_tmap(const Plan& p, const void* gout, TmaDesc* out);

}  // namespace dcn
