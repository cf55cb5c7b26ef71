// C ABI of libdcn_b200 (declared in include/dcn_b200.h): problem planning,
// workspace layout and the launch sequences of forward and backward.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "dcn_b200.h"
#include "dcn_kernels.h"
#include "dcn_plan.h"
#include "dcn_trace.h"

namespace dcn {

namespace {

// Study switch (DCN_STUDY builds only, read at every call): bit 0 skips the
// bilinear gathers, bit 1 output stores / scatters, bit 2 the MMAs (results are
// wrong when set); bit 3 withholds the forward's weight-tile copies, so the
// pipeline waits run out (the failure-detection test: the kernel must give up,
// report DCN_DEVERR_TIMEOUT and leave the context usable).
int debug_skip() {
#ifdef DCN_STUDY
  const char* e = getenv("DCN_DEBUG_SKIP");
  return e ? atoi(e) : 0;
#else
  return 0;
#endif
}

// Pixel budget of one backward chunk in MB of gcol + sampled columns (results
// do not depend on it; a test sets DCN_GCOL_MB=1 to exercise ragged chunks).
long long gcol_budget_mb() {
  static long long v = [] {
    const char* e = getenv("DCN_GCOL_MB");
    return e ? atoll(e) : 1024LL;
  }();
  return v;
}

// Study switch (DCN_STUDY builds only): DCN_GOUT_PACKED=1 keeps the packed
// grad_output copy even where the GEMMs could read grad_output directly.
bool gout_packed_forced() {
#ifdef DCN_STUDY
  static bool v = [] {
    const char* e = getenv("DCN_GOUT_PACKED");
    return e != nullptr && atoi(e) != 0;
  }();
  return v;
#else
  return false;
#endif
}

// DCN_SCATTER_TC=0 runs the plain scatter kernel even where the tile path
// applies (both give the same results; for comparisons).
bool scatter_tc_disabled() {
  static bool v = [] {
    const char* e = getenv("DCN_SCATTER_TC");
    return e != nullptr && atoi(e) == 0;
  }();
  return v;
}

#ifdef DCN_STUDY
// Study switch: DCN_DEBUG_TS prints per-stage global-timer stamps of CTA 0 of
// a kernel to stderr.  One buffer per device (tag 0..2: forward, backward
// data, backward weight); allocates and synchronises, so never in a normal build.
unsigned long long* study_ts_buffer(int tag, cudaStream_t s) {
  if (!getenv("DCN_DEBUG_TS")) return nullptr;
  static unsigned long long* bufs[64][4];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!bufs[dev][tag] && cudaMalloc(&bufs[dev][tag], 1024 * sizeof(unsigned long long)) != cudaSuccess)
    bufs[dev][tag] = nullptr;
  if (bufs[dev][tag]) cudaMemsetAsync(bufs[dev][tag], 0, 1024 * sizeof(unsigned long long), s);
  return bufs[dev][tag];
}

void study_ts_print(const char* label, unsigned long long* d, cudaStream_t s) {
  if (!d) return;
  unsigned long long h[1024];
  cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, s);
  cudaStreamSynchronize(s);
  fprintf(stderr, "%s", label);
  for (int i = 0; i < 1024; ++i) fprintf(stderr, " %llu", h[i]);
  fprintf(stderr, "\n");
}
#endif

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up once through the runtime.
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

int device_sms() {
  static int cached[64];
  static std::once_flag flags[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::call_once(flags[dev], [dev] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  });
  return cached[dev];
}

// Backward-weight work split: M tiles per CTA and units per CTA, chosen to
// reuse each gathered column across as many Co rows as TMEM holds, with at
// least two pipeline stages in shared memory.
void plan_weight_grad(Plan* p, int num_sms) {
  const size_t aTile = 128 * 128;
  int best_m = 1, best_u = 1;
  for (int m = p->nMT; m >= 1; --m) {
    int u = 512 / (m * p->NC);
    if (u < 1) continue;
    if (u > p->nU) u = p->nU;
    // balance the unit sets
    const int nsets = ceil_div(p->nU, u);
    u = ceil_div(p->nU, nsets);
    while (u >= 1) {
      const size_t stage = (size_t)p->nsplit * (m * aTile + (size_t)u * p->NC * 128);
      if (2 * stage + 1024 <= kBwdSmemBudget) break;
      --u;
    }
    if (u >= 1) {
      best_m = m;
      best_u = u;
      break;
    }
  }
  p->wg_mt_per_cta = best_m;
  p->wg_ncg = ceil_div(p->nMT, best_m);
  p->wg_units_per_set = best_u;
  p->wg_nsets = ceil_div(p->nU, best_u);
  p->wg_ksteps = (int)((p->totalP + 63) / 64);
  const int base = p->wg_ncg * p->wg_nsets;
  int ns = num_sms / base;
  if (ns < 1) ns = 1;
  if (ns > p->wg_ksteps) ns = p->wg_ksteps;
  if (ns < 1) ns = 1;
  p->wg_nsplit_px = ns;
}

}  // namespace

bool pdl_enabled() {
  static bool v = [] {
    const char* e = getenv("DCN_NO_PDL");
    return !(e != nullptr && atoi(e) != 0);
  }();
  return v;
}

bool make_gout_tmap(const Plan& P, const void* gout, TmaDesc* out) {
  static_assert(sizeof(CUtensorMap) == sizeof(TmaDesc), "tensor map size");
  EncodeTiledFn fn = encode_tiled();
  if (!fn || !gout || P.esz != 2) return false;
  cuuint64_t dims[3], strides[2];
  if (P.nhwc) {
    // channels-last grad_output is a [totalP][Co] matrix: a box of 64 Co x 64
    // pixels lands in shared memory as the packed block (pixel rows of 128 B,
    // SW128), so the GEMMs keep the packed operand layouts; blocks may straddle
    // images and rows past totalP read zeros
    if ((P.Co % 8) != 0) return false;
    dims[0] = (cuuint64_t)P.Co;
    dims[1] = (cuuint64_t)P.totalP;
    dims[2] = 1;
    strides[0] = (cuuint64_t)P.Co * 2u;
    strides[1] = (cuuint64_t)P.totalP * P.Co * 2u;
  } else {
    if ((P.HoWo % 64) != 0) return false;
    dims[0] = (cuuint64_t)P.HoWo;
    dims[1] = (cuuint64_t)P.Co;
    dims[2] = (cuuint64_t)P.B;
    strides[0] = (cuuint64_t)P.HoWo * 2u;
    strides[1] = (cuuint64_t)P.Co * P.HoWo * 2u;
  }
  const cuuint32_t box[3] = {64u, 64u, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt =
      P.dtype == DCN_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap m;
  const CUresult r = fn(&m, dt, 3, const_cast<void*>(gout), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  memcpy(out, &m, sizeof(m));
  return true;
}

bool make_scatter_tmaps(const Plan& P, const void* xt, const void* gcol, const float* gx, TmaDesc* xmap,
                        TmaDesc* cmap, TmaDesc* rmap) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || P.esz != 2) return false;
  const CUtensorMapDataType dt =
      P.dtype == DCN_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  auto enc = [&](CUtensorMapDataType t, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                 const cuuint32_t* box, TmaDesc* out) {
    CUtensorMap m;
    if (fn(&m, t, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
    memcpy(out, &m, sizeof(m));
    return true;
  };
  // packed input [B][H][W][CS]: a 16 x 16 pixel window of one 64-channel block
  const cuuint64_t xd[4] = {(cuuint64_t)P.CS, (cuuint64_t)P.W, (cuuint64_t)P.H, (cuuint64_t)P.B};
  const cuuint64_t xs[3] = {(cuuint64_t)P.CS * 2u, (cuuint64_t)P.W * P.CS * 2u, (cuuint64_t)P.H * P.W * P.CS * 2u};
  const cuuint32_t xb[4] = {64u, 16u, 16u, 1u};
  // gcol [B][Ho][Wo][K2*dg*Cgp] (one pixel chunk): 8 x 8 pixels x 64 channels of one (tap, group)
  const cuuint64_t row = (cuuint64_t)P.K2 * P.dg * P.Cgp;
  const cuuint64_t cd[4] = {row, (cuuint64_t)P.Wo, (cuuint64_t)P.Ho, (cuuint64_t)P.B};
  const cuuint64_t cs[3] = {row * 2u, (cuuint64_t)P.Wo * row * 2u, (cuuint64_t)P.HoWo * row * 2u};
  const cuuint32_t cbx[4] = {64u, 8u, 8u, 1u};
  // fp32 grad_input accumulator [B][H][W][CS]: 8 rows x 16 pixels x 32 channels
  const cuuint64_t rs[3] = {(cuuint64_t)P.CS * 4u, (cuuint64_t)P.W * P.CS * 4u, (cuuint64_t)P.H * P.W * P.CS * 4u};
  const cuuint32_t rb[4] = {32u, 16u, 8u, 1u};
  return enc(dt, xt, xd, xs, xb, xmap) && enc(dt, gcol, cd, cs, cbx, cmap) &&
         enc(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, gx, xd, rs, rb, rmap);
}

// Strides of the offset and mask tensors (see Plan::off_bs); `om`: both are the
// channels of one predictor output [B][3*dg*K2][Ho][Wo], offsets first.
void set_offset_mask_strides(Plan* p, int om) {
  const int noff = 2 * p->dg * p->K2, nmsk = p->dg * p->K2;
  const int ctot_off = om ? 3 * nmsk : noff, ctot_msk = om ? 3 * nmsk : nmsk;
  p->off_bs = ctot_off * p->HoWo;
  p->msk_bs = ctot_msk * p->HoWo;
  if (p->nhwc) {
    p->off_cs = p->msk_cs = 1;
    p->off_ps = ctot_off;
    p->msk_ps = ctot_msk;
  } else {
    p->off_cs = p->msk_cs = p->HoWo;
    p->off_ps = p->msk_ps = 1;
  }
  p->mask_logit = om;
}

// Element offset of the mask channels inside the predictor output of the fused
// path (channel 2*dg*K2 of pixel 0 of batch 0).
size_t om_mask_offset(const Plan& p) {
  const size_t c0 = (size_t)2 * p.dg * p.K2;
  return p.nhwc ? c0 : c0 * p.HoWo;
}

int make_plan(const dcn_desc* d, Plan* p, int num_sms) {
  if (d == nullptr || p == nullptr) return DCN_E_NULLPTR;
  memset(p, 0, sizeof(*p));
  if (d->B < 0 || d->C <= 0 || d->H <= 0 || d->W <= 0 || d->Co <= 0 || d->kh <= 0 ||
      d->kw <= 0 || d->sh <= 0 || d->sw <= 0 || d->ph < 0 || d->pw < 0 || d->dh <= 0 ||
      d->dw <= 0 || d->dg <= 0 || d->C % d->dg != 0)
    return DCN_E_INVALID;
  if (d->dtype != DCN_F32 && d->dtype != DCN_F16 && d->dtype != DCN_BF16) return DCN_E_INVALID;
  if (d->layout != DCN_NCHW && d->layout != DCN_NHWC) return DCN_E_INVALID;
  if ((d->flags & ~(DCN_FLAG_INPUT_PACKED | DCN_FLAG_WEIGHT_PACKED)) != 0) return DCN_E_INVALID;
  p->B = d->B; p->C = d->C; p->H = d->H; p->W = d->W; p->Co = d->Co;
  p->kh = d->kh; p->kw = d->kw; p->sh = d->sh; p->sw = d->sw; p->ph = d->ph; p->pw = d->pw;
  p->dh = d->dh; p->dw = d->dw; p->dg = d->dg; p->dtype = d->dtype; p->has_bias = d->has_bias;
  p->nhwc = d->layout == DCN_NHWC;
  const long long ho = ((long long)d->H + 2LL * d->ph - ((long long)d->dh * (d->kh - 1) + 1)) / d->sh + 1;
  const long long wo = ((long long)d->W + 2LL * d->pw - ((long long)d->dw * (d->kw - 1) + 1)) / d->sw + 1;
  if (ho <= 0 || wo <= 0) return DCN_E_INVALID;
  if (ho * wo > (1LL << 30) || (long long)d->H * d->W > (1LL << 30)) return DCN_E_UNSUPPORTED;
  p->Ho = (int)ho; p->Wo = (int)wo; p->HoWo = (int)(ho * wo);
  // 32-bit element indexing inside the kernels
  {
    const long long cgp = (long long)ceil_div(d->C / d->dg, kChunk) * kChunk;
    const long long big = 1LL << 31;
    if ((long long)d->B * d->H * d->W * d->dg * cgp >= big ||
        (long long)d->B * d->dg * 2 * d->kh * d->kw * ho * wo >= big ||
        (long long)d->B * d->Co * ho * wo >= big || (long long)d->B * d->C * d->H * d->W >= big)
      return DCN_E_UNSUPPORTED;
  }
  p->K2 = d->kh * d->kw;
  p->totalP = (long long)d->B * p->HoWo;
  p->Cg = d->C / d->dg;
  p->Cgp = ceil_div(p->Cg, kChunk) * kChunk;
  p->nCB = p->Cgp / kChunk;
  p->CS = d->dg * p->Cgp;
  p->esz = d->dtype == DCN_F32 ? 4 : 2;
  p->xesz = p->esz;
  p->nsplit = d->dtype == DCN_F32 ? 2 : 1;
  // forward
  p->nK = p->K2 * d->dg * p->nCB;
  p->nCoT = ceil_div(d->Co, 256);
  p->NT = ceil_div(ceil_div(d->Co, p->nCoT), 16) * 16;
  p->nPT = (int)((p->totalP + kTileM - 1) / kTileM);

  // backward data
  p->Cop = ceil_div(d->Co, kChunk) * kChunk;
  p->nKo = p->Cop / kChunk;
  p->NC = p->Cgp < 256 ? p->Cgp : 256;
  p->nCC = ceil_div(p->Cgp, p->NC);
  p->nU = p->K2 * d->dg * p->nCC;
  {
    const int nTG = p->K2 * d->dg;
    // (tap, group)s per unit: at most 256 columns, balanced over the units
    int gmax = p->nCC == 1 ? 256 / p->NC : 1;
    if (gmax > nTG) gmax = nTG;
    if (gmax < 1) gmax = 1;
    const int nset = ceil_div(nTG, gmax);
    p->gT = ceil_div(nTG, nset);
    p->gNC = p->gT * p->NC;
    p->gnU = ceil_div(nTG, p->gT) * p->nCC;
  }
  // backward weight
  p->nMT = ceil_div(d->Co, 128);
  plan_weight_grad(p, num_sms);
  // packed tiles
  p->wf_tile_bytes = (size_t)p->nsplit * p->NT * 128;
  p->wd_tile_bytes = (size_t)p->nsplit * p->gNC * 128;
  // workspace layout
  size_t off = 0;
  p->off_status = off; off += kWsAlign;
  p->off_x = off; off = align_up(off + (size_t)d->B * d->H * d->W * p->CS * p->xesz, kWsAlign);
  const size_t common = off;
  p->off_wf = off; off = align_up(off + (size_t)p->nCoT * p->nK * p->wf_tile_bytes, kWsAlign);
  p->fwd_bytes = off;
  off = common;
  p->off_wd = off; off = align_up(off + (size_t)p->gnU * p->nKo * p->wd_tile_bytes, kWsAlign);
  p->nPB = (int)((p->totalP + 63) / 64);
  p->off_go = off; off = align_up(off + (size_t)p->nPB * p->nKo * p->nsplit * 8192, kWsAlign);
  // the backward runs in pixel chunks whose column gradients and sampled
  // columns fit a fixed budget (1 GB; DCN_GCOL_MB overrides), keeping 32-bit
  // indexing and the workspace bounded for large batches
  {
    const long long row_bytes = (long long)p->K2 * p->CS * p->esz;
    const long long cols_row = (long long)p->nsplit * p->nU * p->NC * 2;
    long long chunk = (gcol_budget_mb() << 20) / (row_bytes + cols_row) / kTileM * kTileM;
    if (chunk < kTileM) chunk = kTileM;
    const long long need = (p->totalP + kTileM - 1) / kTileM * kTileM;
    if (chunk > need) chunk = need;
    if (chunk * row_bytes / p->esz >= (1LL << 31)) return DCN_E_UNSUPPORTED;
    p->gcol_chunk = (int)chunk;
  }
  p->off_gcol = off;
  off = align_up(off + (size_t)p->gcol_chunk * p->K2 * p->CS * p->esz, kWsAlign);
  p->off_cols = off;
  off = align_up(off + (size_t)p->gcol_chunk * p->nsplit * p->nU * p->NC * 2, kWsAlign);
  p->off_gx = off; off = align_up(off + (size_t)d->B * d->H * d->W * p->CS * 4, kWsAlign);
  p->off_gw = off; off = align_up(off + (size_t)d->Co * p->K2 * p->CS * 4, kWsAlign);
  p->off_gb = off; off = align_up(off + (size_t)d->Co * 4, kWsAlign);
  p->bwd_bytes = off;
  p->fd_howo = make_fastdiv((uint32_t)p->HoWo);
  p->fd_wo = make_fastdiv((uint32_t)p->Wo);
  p->fd_kw = make_fastdiv((uint32_t)p->kw);
  p->fd_dg = make_fastdiv((uint32_t)p->dg);
  p->fd_ntg = make_fastdiv((uint32_t)(p->K2 * p->dg));
  set_offset_mask_strides(p, 0);
  return DCN_OK;
}

}  // namespace dcn

using namespace dcn;

namespace {

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

}  // namespace

extern "C" {

int dcn_output_size(const dcn_desc* d, int32_t* Ho, int32_t* Wo) {
  Plan p;
  const int rc = make_plan(d, &p, 148);
  if (rc != DCN_OK) return rc;
  if (Ho) *Ho = p.Ho;
  if (Wo) *Wo = p.Wo;
  return DCN_OK;
}

size_t dcn_forward_workspace_size(const dcn_desc* d) {
  Plan p;
  return make_plan(d, &p, device_sms()) == DCN_OK ? p.fwd_bytes : 0;
}

size_t dcn_backward_workspace_size(const dcn_desc* d) {
  Plan p;
  return make_plan(d, &p, device_sms()) == DCN_OK ? p.bwd_bytes : 0;
}

// om != 0: `offset` is the predictor output [B][3*dg*K2][Ho][Wo] (offsets in
// channels 0 .. 2*dg*K2-1, mask logits after them) and `mask` is ignored.
static int forward_impl(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                        const void* offset, const void* bias, void* output, void* workspace,
                        size_t workspace_bytes, void* stream, int om) {
  Plan P;
  int rc = make_plan(d, &P, device_sms());
  if (rc != DCN_OK) return rc;
  if (om) {
    set_offset_mask_strides(&P, 1);
    mask = offset ? static_cast<const uint8_t*>(offset) + om_mask_offset(P) * P.esz : nullptr;
  }
  if (!workspace) return DCN_E_NULLPTR;
  if (workspace_bytes < P.fwd_bytes || ((uintptr_t)workspace & (kWsAlign - 1)) != 0)
    return DCN_E_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(ws + P.off_status);
  if (P.totalP == 0)
    return cudaMemsetAsync(status, 0, sizeof(int), s) == cudaSuccess ? DCN_OK : DCN_E_CUDA;
  if (!input || !weight || !mask || !offset || !output) return DCN_E_NULLPTR;
  if (d->has_bias && !bias) return DCN_E_NULLPTR;
  const bool wpacked = (d->flags & DCN_FLAG_WEIGHT_PACKED) != 0;
  const bool fused = !wpacked && !P.nhwc && P.esz == 2 && (P.H * P.W) % 8 == 0 && aligned16(input);
  if (fused) {
    // 16-bit NCHW: input and weight packs in one launch (traced as pack_input);
    // the input pack also clears the status word
    TraceScope ts(TR_PACK_INPUT, s);
    if ((rc = launch_pack_forward(P, input, ws + P.off_x, status, weight, ws + P.off_wf, s)) != DCN_OK) return rc;
  } else {
    {
      // the input pack also clears the status word
      TraceScope ts(TR_PACK_INPUT, s);
      if ((rc = launch_pack_input(P, input, ws + P.off_x, nullptr, status, s)) != DCN_OK) return rc;
    }
    if (!wpacked) {
      TraceScope ts(TR_PACK_WEIGHT_FWD, s);
      if ((rc = launch_pack_weight_fwd(P, weight, ws + P.off_wf, s)) != DCN_OK) return rc;
    }
  }
  FwdArgs a;
  memset(&a, 0, sizeof(a));
  a.plan = P;
  a.xt = ws + P.off_x;
  a.offset = offset;
  a.mask = mask;
  a.wpk = ws + P.off_wf;
  a.bias = d->has_bias ? bias : nullptr;
  a.out = output;
  a.vec_out = aligned16(output);
  a.err = reinterpret_cast<int*>(ws + P.off_status);
  a.num_sms = device_sms();
  a.dbg = debug_skip();
#ifdef DCN_STUDY
  a.ts = study_ts_buffer(0, s);
#endif
  {
    TraceScope ts(TR_FORWARD, s);
    rc = launch_forward(a, s);
  }
#ifdef DCN_STUDY
  study_ts_print("DCN_TS", a.ts, s);
#endif
  return rc;
}

// om != 0: `offset` / `grad_offset` are the predictor output and its gradient
// (grad_offset then receives the gradient of the mask logits in its last dg*K2
// channels); `mask` / `grad_mask` are ignored.
static int backward_impl(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                         const void* offset, const void* bias, const void* grad_output, void* grad_input,
                         void* grad_offset, void* grad_mask, void* grad_weight, void* grad_bias,
                         void* workspace, size_t workspace_bytes, void* stream, int om) {
  (void)bias;
  Plan P;
  int rc = make_plan(d, &P, device_sms());
  if (rc != DCN_OK) return rc;
  if (om) {
    const size_t mofs = om_mask_offset(P) * P.esz;
    set_offset_mask_strides(&P, 1);
    mask = offset ? static_cast<const uint8_t*>(offset) + mofs : nullptr;
    grad_mask = grad_offset ? static_cast<uint8_t*>(grad_offset) + mofs : nullptr;
  }
  if (!weight || !grad_weight || !workspace) return DCN_E_NULLPTR;
  if (P.totalP > 0 && (!input || !mask || !offset || !grad_output || !grad_input ||
                       !grad_offset || !grad_mask))
    return DCN_E_NULLPTR;
  if (d->has_bias && !grad_bias) return DCN_E_NULLPTR;
  if (workspace_bytes < P.bwd_bytes || ((uintptr_t)workspace & (kWsAlign - 1)) != 0)
    return DCN_E_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* gxn = reinterpret_cast<float*>(ws + P.off_gx);
  float* gw = reinterpret_cast<float*>(ws + P.off_gw);
  float* gb = reinterpret_cast<float*>(ws + P.off_gb);
  int* status = reinterpret_cast<int*>(ws + P.off_status);
  if (P.totalP == 0) {
    // gx, gw and gb accumulators are contiguous: one memset
    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess ||
        cudaMemsetAsync(ws + P.off_gx, 0, P.bwd_bytes - P.off_gx, s) != cudaSuccess)
      return DCN_E_CUDA;
    if ((rc = launch_finish_grad_weight(P, gw, gb, grad_weight, d->has_bias ? grad_bias : nullptr, s)) != DCN_OK)
      return rc;
    // empty output but non-empty input (cannot happen with Ho, Wo > 0): zero grad_input
    if ((long long)P.B * P.C * P.H * P.W > 0 && grad_input)
      return launch_finish_grad_input(P, gxn, grad_input, s);
    return DCN_OK;
  }
  const bool packed = (d->flags & DCN_FLAG_INPUT_PACKED) != 0;
  if (!packed) {
    // the input pack also clears the status word and the grad_input accumulator
    TraceScope ts(TR_PACK_INPUT, s);
    if ((rc = launch_pack_input(P, input, ws + P.off_x, gxn, status, s)) != DCN_OK) return rc;
  }
  {
    TraceScope ts(TR_PACK_WEIGHT_BWD, s);
    // ... and the weight pack the gw and gb accumulators (contiguous); with the
    // forward's packed input reused it clears the grad_input accumulator (just
    // before gw) and the status word too
    uint8_t* z0 = ws + (packed ? P.off_gx : P.off_gw);
    if ((rc = launch_pack_weight_bwd(P, weight, ws + P.off_wd, reinterpret_cast<float*>(z0),
                                     P.bwd_bytes - (size_t)(z0 - ws), packed ? status : nullptr, s)) != DCN_OK)
      return rc;
  }
  // 16-bit grad_output is read by the GEMMs directly (TMA tiles of 64 pixels x
  // 64 Co) when NCHW with 64-pixel blocks that never straddle two images, or
  // channels-last with Co % 8 == 0; otherwise it is packed into swizzled
  // blocks first (and f32 is split into bf16 hi/lo).
  BwdDataArgs a;
  memset(&a, 0, sizeof(a));
  a.gdirect = (P.esz == 2 && aligned16(grad_output) && !gout_packed_forced() &&
               make_gout_tmap(P, grad_output, &a.gmap))
                  ? (P.nhwc ? kGoutNhwc : kGoutNchw)
                  : 0;
  if (!a.gdirect) {
    TraceScope ts(TR_PACK_GRAD_OUTPUT, s);
    const int vec = aligned16(grad_output) && (P.HoWo % 8 == 0);
    if ((rc = launch_pack_gout(P, grad_output, ws + P.off_go, d->has_bias ? gb : nullptr, vec, s)) !=
        DCN_OK)
      return rc;
  }
  a.plan = P;
  a.xt = ws + P.off_x;
  a.offset = offset;
  a.mask = mask;
  a.gout = grad_output;
  a.gpk = ws + P.off_go;
  a.wpk = ws + P.off_wd;
  a.gx_nhwc = gxn;
  a.gcol = ws + P.off_gcol;
  a.goffset = grad_offset;
  a.gmask = grad_mask;
  a.err = reinterpret_cast<int*>(ws + P.off_status);
  a.num_sms = device_sms();
  a.dbg = debug_skip();
  a.vec_gout = aligned16(grad_output);
  a.cols = ws + P.off_cols;
#ifdef DCN_STUDY
  unsigned long long* const dts_d = study_ts_buffer(1, s);
  a.ts = dts_d;
  unsigned long long* dts_s = nullptr;
#endif
  BwdWeightArgs w;
  memset(&w, 0, sizeof(w));
  w.plan = P;
  w.gmap = a.gmap;
  w.gdirect = a.gdirect;
  w.gb = (a.gdirect && d->has_bias) ? gb : nullptr;
  w.cols = a.cols;
  w.gpk = ws + P.off_go;
  w.gw = gw;
  w.err = a.err;
  w.num_sms = a.num_sms;
  w.dbg = a.dbg;
#ifdef DCN_STUDY
  unsigned long long* const dts = study_ts_buffer(2, s);
  w.ts = dts;
#endif
  // the tile scatter (grad_input summed on the tensor cores) where it applies
  const bool use_tc = !scatter_tc_disabled() && backward_scatter_tc_eligible(P) &&
                      make_scatter_tmaps(P, a.xt, a.gcol, a.gx_nhwc, &a.xmap, &a.cmap, &a.rmap);
  // per pixel chunk: column gradients (tcgen05), then the scatter (grad_input,
  // grad_offset, grad_mask and the sampled columns), then the weight gradient
  for (long long p0 = 0; p0 < P.totalP; p0 += P.gcol_chunk) {
    a.pix0 = (int)p0;
    a.npix = (int)(P.totalP - p0 < P.gcol_chunk ? P.totalP - p0 : P.gcol_chunk);
    {
      TraceScope ts(TR_BACKWARD_DATA, s);
      if ((rc = launch_backward_data(a, s)) != DCN_OK) return rc;
    }
    {
      TraceScope ts(TR_BACKWARD_SCATTER, s);
      BwdDataArgs sa = a;
#ifdef DCN_STUDY
      sa.ts = a.ts ? study_ts_buffer(3, s) : nullptr;
      dts_s = sa.ts ? sa.ts : dts_s;
#endif
      if ((rc = use_tc ? launch_backward_scatter_tc(sa, s) : launch_backward_scatter(sa, s)) != DCN_OK) return rc;
    }
    w.ks0 = (int)(p0 / 64);
    w.nks = (a.npix + 63) / 64;
    {
      TraceScope ts(TR_BACKWARD_WEIGHT, s);
      if ((rc = launch_backward_weight(w, s)) != DCN_OK) return rc;
    }
    if (w.ts) w.ts = nullptr;   // timestamps of the first chunk only
    if (a.ts) a.ts = nullptr;
  }
#ifdef DCN_STUDY
  study_ts_print("DCN_TSD", dts_d, s);
  study_ts_print("DCN_TSS", dts_s, s);
  study_ts_print("DCN_TSW", dts, s);
#endif
  if (!P.nhwc) {
    // NCHW: both finishing passes in one launch (traced as finish_grad_input)
    TraceScope ts(TR_FINISH_GRAD_INPUT, s);
    return launch_finish_grads(P, gxn, grad_input, gw, gb, grad_weight, d->has_bias ? grad_bias : nullptr, s);
  }
  {
    TraceScope ts(TR_FINISH_GRAD_INPUT, s);
    if ((rc = launch_finish_grad_input(P, gxn, grad_input, s)) != DCN_OK) return rc;
  }
  TraceScope ts(TR_FINISH_GRAD_WEIGHT, s);
  return launch_finish_grad_weight(P, gw, gb, grad_weight, d->has_bias ? grad_bias : nullptr, s);
}

int dcn_forward(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                const void* offset, const void* bias, void* output, void* workspace,
                size_t workspace_bytes, void* stream) {
  return forward_impl(d, input, weight, mask, offset, bias, output, workspace, workspace_bytes, stream, 0);
}

int dcn_backward(const dcn_desc* d, const void* input, const void* weight, const void* mask,
                 const void* offset, const void* bias, const void* grad_output, void* grad_input,
                 void* grad_offset, void* grad_mask, void* grad_weight, void* grad_bias,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return backward_impl(d, input, weight, mask, offset, bias, grad_output, grad_input, grad_offset,
                       grad_mask, grad_weight, grad_bias, workspace, workspace_bytes, stream, 0);
}

int dcn_forward_om(const dcn_desc* d, const void* input, const void* weight, const void* offset_mask,
                   const void* bias, void* output, void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(d, input, weight, nullptr, offset_mask, bias, output, workspace, workspace_bytes,
                      stream, 1);
}

int dcn_backward_om(const dcn_desc* d, const void* input, const void* weight, const void* offset_mask,
                    const void* bias, const void* grad_output, void* grad_input, void* grad_offset_mask,
                    void* grad_weight, void* grad_bias, void* workspace, size_t workspace_bytes,
                    void* stream) {
  return backward_impl(d, input, weight, nullptr, offset_mask, bias, grad_output, grad_input,
                       grad_offset_mask, nullptr, grad_weight, grad_bias, workspace, workspace_bytes,
                       stream, 1);
}

int dcn_read_device_status(void* workspace, void* stream) {
  if (!workspace) return DCN_E_NULLPTR;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return DCN_E_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return DCN_E_CUDA;
  if (cudaMemsetAsync(workspace, 0, sizeof(int), s) != cudaSuccess) return DCN_E_CUDA;
  return h;
}

const char* dcn_strerror(int code) {
  switch (code) {
    case DCN_OK: return "ok";
    case DCN_E_INVALID: return "invalid shape or parameter";
    case DCN_E_NULLPTR: return "required pointer is NULL";
    case DCN_E_WORKSPACE: return "workspace too small or not 256-byte aligned";
    case DCN_E_CUDA: return "CUDA runtime error";
    case DCN_E_UNSUPPORTED: return "unsupported configuration";
    case DCN_E_DEVICE: return "error recorded by a kernel";
    case DCN_E_SCRATCH_LIMIT:
      return "problem exceeds the fixed scratch of dcn_forward_noalloc (DCN_NOALLOC_SCRATCH_BYTES)";
    default: return "unknown error";
  }
}

const char* dcn_version(void) { return "dcn_b200 0.1.0 sm_100a"; }

}  // extern "C"
