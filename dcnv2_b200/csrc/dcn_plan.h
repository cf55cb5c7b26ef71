// Host/device shared problem plan: derived sizes, tiling and workspace layout.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "dcn_b200.h"

namespace dcn {

constexpr int kTileM = 128;   // pixels per output tile (UMMA M)
constexpr int kChunk = 64;    // 16-bit elements per 128-byte swizzle row (one K chunk)
constexpr size_t kWsAlign = 256;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Division by a run-time constant d >= 1 for numerators 0 <= n < 2^31 with one
// multiply-high and a shift: m = ceil(2^(31+s) / d), s = ceil(log2 d), then
// n / d = umulhi(n, m) >> (s - 1).  Exact: with m = (2^(31+s) + e) / d,
// 0 <= e < d, the error term n e / (d 2^(31+s)) stays below 2^-s <= 1/d.
struct FastDiv {
  uint32_t d, m, sh;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d ? d : 1;
  uint32_t s = 0;
  while ((1ull << s) < f.d) ++s;
  f.m = f.d == 1 ? 0u : (uint32_t)(((1ull << (31 + s)) + f.d - 1) / f.d);
  f.sh = s ? s - 1 : 0;
  return f;
}
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

struct Plan {
  // problem
  int B, C, H, W, Co, kh, kw, sh, sw, ph, pw, dh, dw, dg, dtype, has_bias;
  int nhwc;           // activations channels-last (DCN_NHWC)
  int Ho, Wo, HoWo, K2;
  long long totalP;   // B*Ho*Wo output pixels
  int Cg, Cgp, nCB;   // channels per group, padded to 64, 64-channel blocks per group
  int CS;             // channels per packed input pixel = dg*Cgp
  int esz;            // bytes per element of the tensors (2 or 4)
  int xesz;           // bytes per element of the packed input (esz)
  int nsplit;         // 2 for f32 (bf16 hi/lo operands), else 1
  // forward GEMM: M = pixels, N = Co tile, K = taps x groups x channel blocks
  int nK;             // K chunks = K2*dg*nCB
  int NT, nCoT;       // Co tile, number of Co tiles
  int nPT;            // pixel tiles
  // backward-data GEMM: M = pixels, N = channel chunk of a group, K = Co
  int Cop, nKo;       // Co padded to 64, 64-channel Co chunks
  int NC, nCC;        // channel chunk (<=256), chunks per group
  int nU;             // units (t, g, channel chunk) = K2*dg*nCC (backward-weight)
  int gT, gNC, gnU;   // backward-data GEMM units: gT (tap, group)s x NC channels = gNC
                      // columns (<= 256), gnU = ceil(K2*dg / gT) * nCC units
  // backward-weight GEMM: M = Co (128 rows per M tile), N = channel sets, K = pixels
  int nMT;            // 128-row Co tiles
  int wg_mt_per_cta;  // M tiles handled by one CTA
  int wg_ncg;         // Co groups (nMT / wg_mt_per_cta)
  int wg_units_per_set, wg_nsets;  // (t,g,cc) units per CTA and the number of sets
  int wg_nsplit_px;   // CTAs along the pixel reduction
  int wg_ksteps;      // 64-pixel K steps in total (ceil(totalP/64))
  // workspace layout (bytes)
  size_t off_status, off_x, off_wf, off_wd, off_go, off_gcol, off_cols, off_gx, off_gw, off_gb;
  int nPB;               // 64-pixel blocks of the packed grad_output
  int gcol_chunk;        // pixels per backward chunk (multiple of 128)
  size_t fwd_bytes, bwd_bytes;
  size_t wf_tile_bytes;   // one forward weight tile (NT rows x 128 B x nsplit)
  size_t wd_tile_bytes;   // one backward-data weight tile (gNC rows x 128 B x nsplit)
  // divisors of the index arithmetic in the kernels
  FastDiv fd_howo, fd_wo, fd_kw, fd_dg, fd_ntg;
  // offset / mask addressing: element (b, channel, pixel) of the offset tensor is
  // at b*off_bs + channel*off_cs + pixel*off_ps, likewise the mask (NCHW: channel
  // stride HoWo, pixel stride 1; channels-last: channel stride 1, pixel stride =
  // the channel count; the predictor output of the fused path holds both, with
  // 3*dg*K2 channels), and whether the mask values are logits that the kernels
  // pass through a sigmoid
  int off_bs, off_cs, off_ps, msk_bs, msk_cs, msk_ps, mask_logit;
};

// Fills `p` from `d`; returns DCN_OK or DCN_E_INVALID / DCN_E_UNSUPPORTED.
int make_plan(const dcn_desc* d, Plan* p, int num_sms);

}  // namespace dcn
