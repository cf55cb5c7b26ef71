// Forward DCNv2 as one fused, persistent, warp-specialised implicit GEMM on
// tcgen05 tensor cores (replaces the reference's im2col + WMMA GEMM pair,
// com.cu:151-195 and com.cu:46-117, and never materialises the columns).
//
//   D[pixel, co] = sum_{t, g, c} A[pixel, (t,g,c)] * Wt[co, (t,g,c)]
//   A[pixel, (t,g,c)] = mask * bilinear(x_nhwc[b, :, :, g, c], pos(pixel, t) + offset)
//
// CTA roles (896 threads for 16-bit types, one CTA per SM, persistent over
// (pixel, Co) tiles; f32 uses 8 producer warps of 16 rows, 640 threads):
//   warps 0-15  gather producers: 8 pixel rows per warp, 8 lanes per pixel so
//               each warp-wide load reads whole corner lines; build the A tile
//               (128 pixels x 64 channels, K-major, 128B swizzle) in smem
//   warps 16-23 epilogue: TMEM -> registers, + bias, NCHW store; between tiles
//               they also build the next tile's sampling geometry (corner index
//               and the four weights x mask per row and tap) in shared memory
//   warp 24     bulk-copy (TMA) producer of the pre-packed weight tile
//   warp 25     TMEM owner and single-thread tcgen05.mma issuer (warps 26-27 idle)
// Registers are moved with setmaxnreg (producers 80 (f32: 160), epilogue 64,
// control 32).
// A/B stages form an mbarrier ring; the accumulator is double-buffered in TMEM so
// the epilogue of tile i overlaps the main loop of tile i+1.
#include <stdlib.h>

#include <type_traits>

#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

#define DCN_TS(slot) \
  do { if (DCN_STUDY_ON && a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

constexpr int kMaxCo = 2048;  // bias staged in smem: Co up to 2048
constexpr int kGeoTaps = 9;   // (tap, group)s per geometry window
// Warp layout of the CTA for PW gather-producer warps: PW/4 producer warpgroups,
// two epilogue warpgroups, one control warpgroup (weight copies, MMA, two idle
// warps).  16-bit types use 16 producer warps of 8 rows at 80 registers, f32 (two
// 16-byte loads per corner slice) 8 warps of 16 rows at 160 registers.
template <int PW>
struct FwdLayout {
  static constexpr int kProdWarps = PW;
  static constexpr int kProdThreads = PW * 32;
  static constexpr int kRowsPerWarp = kTileM / PW;       // A-tile rows per producer warp
  static constexpr int kEpiWarp0 = PW;
  static constexpr int kEpiWarps = 8;                    // two per TMEM lane quarter
  static constexpr int kTmaWarp = kEpiWarp0 + kEpiWarps;
  static constexpr int kMmaWarp = kTmaWarp + 1;
  static constexpr int kThreads = (kTmaWarp + 4) * 32;   // 896 (PW 16) or 640 (PW 8)
  static constexpr int kLaunchRegs = (65536 / kThreads) & ~7;   // 72 or 96
  // setmaxnreg split of the launch pool: PW 16: 4 x 128 x 80 + 2 x 128 x 64 +
  // 128 x 32 = 61440 <= 64512; PW 8: 2 x 128 x 160 + 2 x 128 x 64 + 128 x 32 = 61440
  static constexpr int kProdRegs = PW == 16 ? 80 : 160, kEpiRegs = 64, kCtlRegs = 32;
  static_assert(kProdThreads * kProdRegs + kEpiWarps * 32 * kEpiRegs + 128 * kCtlRegs <= kThreads * kLaunchRegs,
                "register split exceeds the launch pool");
};

template <typename T, int PW>
__global__ void __launch_bounds__(FwdLayout<PW>::kThreads, 1)
    dcn_fwd_kernel(const __grid_constant__ FwdArgs a) {
  using L = FwdLayout<PW>;
  constexpr int kProdThreads = L::kProdThreads, kRowsPerWarp = L::kRowsPerWarp;
  constexpr int kEpiWarp0 = L::kEpiWarp0, kEpiWarps = L::kEpiWarps;
  constexpr int kTmaWarp = L::kTmaWarp, kMmaWarp = L::kMmaWarp, kFwdThreads = L::kThreads;
  constexpr int kProdRegs = L::kProdRegs, kEpiRegs = L::kEpiRegs, kCtlRegs = L::kCtlRegs;
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;  // 128 rows x 128 B
  const Plan& P = a.plan;
  const int NT = P.NT;
  const uint32_t bTile = (uint32_t)NT * 128u;
  const uint32_t stageBytes = NS * (kATile + bTile);
  const int S = a.stages;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 11];
  __shared__ uint32_t tmem_slot;
  __shared__ __align__(16) uint8_t epi_stage[kEpiWarps][16 * 32 * 2];
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 2]);
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 4]);
  const uint32_t geof = smem_u32(&bars[2 * kMaxStages + 5]);  // geometry window written
  const uint32_t geoe = smem_u32(&bars[2 * kMaxStages + 6]);  // geometry window consumed
  const uint32_t gready0 = smem_u32(&bars[2 * kMaxStages + 7]);  // geometry window built (x2)
  const uint32_t gfree0 = smem_u32(&bars[2 * kMaxStages + 9]);   // geometry window released (x2)
  // geometry windows after the stage ring: NB x [kGeoTaps][128] corner weights
  // and indices, then the bias.  NB = 2: the epilogue warps build the window of
  // tile i+1 while the producers gather tile i (every (tap, group) of a tile
  // fits one window); NB = 1: the producers build each window themselves.
  const int NB = a.geo_bufs;
  float4* sgeo_w = reinterpret_cast<float4*>(smem_raw + ((sbase - smem_u32(smem_raw)) + S * stageBytes));
  int* sgeo_idx = reinterpret_cast<int*>(sgeo_w + NB * kGeoTaps * kTileM);
  float* sbias = reinterpret_cast<float*>(sgeo_idx + NB * kGeoTaps * kTileM);  // [Co]
  // bias as an MMA operand (16-bit, up to two Co tiles): a K = 16 slice whose
  // only non-zero column is A = 1 (128 rows) and B = bias (NT rows per Co tile), in the
  // no-swizzle K-major layout (8-row x 16-byte core matrices, the two K halves
  // 128 B apart, 8-row groups 256 B apart); the first MMA of every tile then
  // starts the accumulator at the bias and the epilogue adds nothing
  const uint32_t sbias_a = (smem_u32(sbias + P.nCoT * NT) + 127u) & ~127u;
  const uint32_t sbias_b = sbias_a + kTileM * 32u;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, kProdThreads / 32 + 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, kEpiWarps);
    }
    mbar_init(drain, 1);
    mbar_init(geof, kProdThreads / 32);
    mbar_init(geoe, kProdThreads / 32);
    for (int i = 0; i < 2; ++i) {
      mbar_init(gready0 + 8 * i, kEpiWarps);
      mbar_init(gfree0 + 8 * i, kProdThreads / 32);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_wait();
  // bias staged once per CTA (the epilogue reads it for every output element)
  for (int c = tid; c < P.nCoT * NT; c += kFwdThreads)
    sbias[c] = (a.bias != nullptr && c < P.Co) ? ldf(reinterpret_cast<const T*>(a.bias) + c) : 0.f;
  if constexpr (NS == 1) {
    if (a.mma_bias) {
      // word w of row r (elements 2w, 2w+1) at (r/8)*256 + (w/4)*128 + (r%8)*16 + (w%4)*4
      for (int e = tid; e < (kTileM + P.nCoT * NT) * 8; e += kFwdThreads) {
        const int r = e >> 3, w = e & 7;
        uint32_t val = 0u;
        if (w == 0) {
          const float f = r < kTileM ? 1.f : (r - kTileM < P.Co ? ldf(reinterpret_cast<const T*>(a.bias) + (r - kTileM)) : 0.f);
          val = pack2<OpOf<T>::kBF16>(f, 0.f);
        }
        const int rr = r < kTileM ? r : r - kTileM;
        const uint32_t base = r < kTileM ? sbias_a : sbias_b;
        sts_u32(base + (uint32_t)((rr >> 3) * 256 + (w >> 2) * 128 + (rr & 7) * 16 + (w & 3) * 4), val);
      }
      fence_proxy_async_smem();
    }
  }
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * NT)) tmem_cols <<= 1;
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_slot), tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  const int nTiles = P.nPT * P.nCoT;
  const int HoWo = P.HoWo;
  if (warp == 0) DCN_TS(1000);

  // Builds geometry window slot `buf` for pixel tile pt and (tap, group)s
  // tg0 .. tg0 + wt - 1 with NTHR threads (this one is thread gt).  Thread gt
  // owns row gt % 128 and slots gt / 128 + (NTHR / 128) k: the row's
  // coordinates are computed once, and every offset / mask load of the window
  // is issued before the first one is used, so their latencies overlap.
  auto build_geometry = [&](auto nthr_c, int pt, int tg0, int wt, int buf, int gt) {
    constexpr int NTHR = decltype(nthr_c)::value;
    constexpr int SSTEP = NTHR / kTileM;
    constexpr int KI = (kGeoTaps * kTileM + NTHR - 1) / NTHR;
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    const int HW = P.H * P.W;
    const int row = gt & (kTileM - 1), slot0 = gt / kTileM;
    const int pix = pt * kTileM + row;
    const bool pv = pix < P.totalP && !DCN_SKIP(1);
    const int b = pv ? fdiv(pix, P.fd_howo) : 0, p = pv ? pix - b * HoWo : 0;
    const int ho = fdiv(p, P.fd_wo), wo = p - ho * P.Wo;
    uint32_t rh[KI], rw[KI], rm[KI];
#pragma unroll
    for (int k = 0; k < KI; ++k) {
      const int slot = slot0 + SSTEP * k;
      rh[k] = rw[k] = rm[k] = 0u;
      if (pv && slot < wt) {
        const int tgi = tg0 + slot;
        const int t = fdiv(tgi, P.fd_dg), gi = tgi - t * P.dg;
        const int ob = b * P.off_bs + (gi * 2 * P.K2 + 2 * t) * P.off_cs + p * P.off_ps;
        rh[k] = ldg_raw<T>(off + ob);
        rw[k] = ldg_raw<T>(off + ob + P.off_cs);
        rm[k] = ldg_raw<T>(msk + b * P.msk_bs + (gi * P.K2 + t) * P.msk_cs + p * P.msk_ps);
      }
    }
#pragma unroll
    for (int k = 0; k < KI; ++k) {
      const int slot = slot0 + SSTEP * k;
      if (slot < wt) {
        PixGeo r = zero_pixgeo();
        if (pv) {
          const int t = fdiv(tg0 + slot, P.fd_dg);
          const int i = fdiv(t, P.fd_kw), j = t - i * P.kw;
          const float hs = (float)(ho * P.sh - P.ph + i * P.dh) + raw_to_f<T>(rh[k]);
          const float ws = (float)(wo * P.sw - P.pw + j * P.dw) + raw_to_f<T>(rw[k]);
          float mv = raw_to_f<T>(rm[k]);
          if (P.mask_logit) mv = 1.f / (1.f + __expf(-mv));   // sigmoid of a predictor logit
          r = make_pixgeo_clamped(b * HW, hs, ws, mv, P.H, P.W);
        }
        const int e = (buf * kGeoTaps + slot) * kTileM + row;
        sgeo_idx[e] = (int)((unsigned)r.gidx * (unsigned)P.CS);   // element offset of the corner line
        sgeo_w[e] = make_float4(r.w[0], r.w[1], r.w[2], r.w[3]);
      }
    }
  };

  // Roles by warpgroup; setmaxnreg at the top of each branch (one instruction
  // per warpgroup).  16-bit types: launch 896 threads x 72 registers; after the
  // split producers 4 x 4 warps x 80, epilogue 2 x 4 warps x 64, control 4 warps
  // x 32.  f32: launch 640 threads x 96 registers; producers 2 x 4 warps x 160,
  // epilogue and control as above.  Both sums are 61440 registers, within the
  // launch pool (checked by FwdLayout's static_assert).
  if (warp < kProdThreads / 32) {
    regs_inc<kProdRegs>();
    // ------------------------------------------------ gather producers
    // Warp w builds rows w*R .. w*R+R-1 (R = kRowsPerWarp) of every A tile, 4
    // rows at a time with 8 lanes per row.
    using GS = GatherShape<T>;
    constexpr int LPP = GS::kLPP, CPL = GS::kCPL, PPI = GS::kPPI;
    constexpr int ITER = kRowsPerWarp / PPI;
    constexpr int BATCH = sizeof(T) == 4 ? (ITER >= 2 ? 2 : 1) : (ITER < 4 ? ITER : 4);
    const int lp = lane / LPP, q = lane % LPP;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    // element distance of the right and the lower corner line of a clamped block
    const size_t dxe = P.W > 1 ? (size_t)P.CS : 0, dye = P.H > 1 ? (size_t)P.W * P.CS : 0;
    uint32_t kidx = 0, gcnt = 0, gbuf = 0;
    int rs = 0;                                   // ring stage of step kidx and its phase
    uint32_t rph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      const int pt = tile / P.nCoT;
      // Sampling geometry of the tile's 128 rows for a window of up to kGeoTaps
      // (tap, group)s is computed by all producer threads at once (every offset
      // load of the window in flight together) into shared memory; the gather
      // lanes then read it with broadcast loads.  Two bounded mbarrier handoffs
      // per window: everyone is done with the previous window, everyone wrote
      // the new one.
      const int nTG = P.K2 * P.dg;
      const int nwin_t = nTG < kGeoTaps ? nTG : kGeoTaps;
      PixGeo geo[ITER];
      // (tap, group) tg, channel block cb, group g, tap slot tl of step kc, kept
      // as counters (no divisions in the step loop)
      int tg = 0, cb = 0, g = 0, tl = 0;
      for (int kc = 0; kc < P.nK && ok; ++kc, ++kidx) {
        if (cb == 0 && tl == 0) {
          if (NB == 2) {
            // window built by the epilogue warps: release the previous one, wait for this one
            __syncwarp();
            if (gcnt > 0 && lane == 0) mbar_arrive(gfree0 + 8 * ((gcnt - 1) & 1u));
            if (!mbar_wait_warp(gready0 + 8 * (gcnt & 1u), (gcnt >> 1) & 1u, a.err, &abort_flag)) { ok = false; break; }
            gbuf = gcnt & 1u;
          } else {
            // built here by all producer threads; two bounded handoffs per window
            __syncwarp();
            if (lane == 0) mbar_arrive(geoe);
            if (!mbar_wait_warp(geoe, gcnt & 1u, a.err, &abort_flag)) { ok = false; break; }
            build_geometry(std::integral_constant<int, kProdThreads>{}, pt, tg, min(nwin_t, nTG - tg), 0, tid);
            __syncwarp();
            if (lane == 0) mbar_arrive(geof);
            if (!mbar_wait_warp(geof, gcnt & 1u, a.err, &abort_flag)) { ok = false; break; }
            gbuf = 0;
          }
          ++gcnt;
        }
        if (cb == 0) {
#pragma unroll
          for (int it = 0; it < ITER; ++it) {
            const int e = (gbuf * kGeoTaps + tl) * kTileM + warp * kRowsPerWarp + it * PPI + lp;
            const float4 w4 = sgeo_w[e];
            geo[it].gidx = sgeo_idx[e];
            geo[it].w[0] = w4.x;
            geo[it].w[1] = w4.y;
            geo[it].w[2] = w4.z;
            geo[it].w[3] = w4.w;
          }
        }
        if (warp == 0) DCN_TS(4 * kidx);
        const int s = rs;
        const uint32_t ph = rph;
        if (++rs == S) { rs = 0; rph ^= 1u; }
        const uint32_t atile = sbase + s * stageBytes;
        const int cofs = g * P.Cgp + cb * kChunk + q * CPL;
        uint4 v[BATCH][4][GS::kLD];
#pragma unroll
        for (int i0 = 0; i0 < ITER; i0 += BATCH) {
#pragma unroll
          for (int it = 0; it < BATCH; ++it)
            load_block<T>(xt + ((size_t)(unsigned)geo[i0 + it].gidx + cofs), dxe, dye, v[it]);
          if (i0 == 0 && !mbar_wait_warp(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          if (warp == 0 && i0 == 0) DCN_TS(4 * kidx + 1);
#pragma unroll
          for (int it = 0; it < BATCH; ++it)
            blend_store<T>(v[it], geo[i0 + it], atile, kATile, warp * kRowsPerWarp + (i0 + it) * PPI + lp, q);
        }
        if (!ok) break;
        if (warp == 0) DCN_TS(4 * kidx + 2);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(full0 + 8 * s);
        if (warp == 0) DCN_TS(4 * kidx + 3);
        if (++cb == P.nCB) {
          cb = 0;
          ++tg;
          if (++g == P.dg) g = 0;
          if (++tl == nwin_t) tl = 0;
        }
      }
    }
  } else if (warp < kTmaWarp) {
    regs_dec<kEpiRegs>();
    // ------------------------------------------------ epilogue
    const int q = warp & 3;
    constexpr int kEpiPerQuarter = kEpiWarps / 4;
    const int chalf = (warp - kEpiWarp0) >> 2;   // warps of one lane quarter interleave 16-column blocks
    const int row = q * 32 + lane;
    T* __restrict__ y = reinterpret_cast<T*>(a.out);
    int it = 0;
    int gnext = 0;                                  // next geometry window to build (NB == 2)
    for (int tile = blockIdx.x; tile < nTiles; tile += gridDim.x, ++it) {
      const int pt = tile / P.nCoT, ct = tile - pt * P.nCoT;
      const int ab = it & 1;
      if (NB == 2) {
        // windows of this tile and the next one (one window per tile): the slot
        // of window w is free once the producers started window w - 1
        bool gok = true;
        for (; gnext <= it + 1 && blockIdx.x + gnext * (int)gridDim.x < nTiles; ++gnext) {
          const int gb = gnext & 1;
          if (!mbar_wait_warp(gfree0 + 8 * gb, ((gnext >> 1) & 1) ^ 1, a.err, &abort_flag)) { gok = false; break; }
          const int gpt = (blockIdx.x + gnext * (int)gridDim.x) / P.nCoT;
          build_geometry(std::integral_constant<int, kEpiWarps * 32>{}, gpt, 0, P.K2 * P.dg, gb,
                         tid - kEpiWarp0 * 32);
          __syncwarp();
          if (lane == 0) mbar_arrive(gready0 + 8 * gb);
        }
        if (!gok) break;
      }
      if (!mbar_wait_warp(accf0 + 8 * ab, (it >> 1) & 1, a.err, &abort_flag)) break;
      if (warp == kEpiWarp0) DCN_TS(800 + 2 * it);
      tc_fence_after();
      const int pix = pt * kTileM + row;
      const bool pv = pix < P.totalP;
      const int b = pv ? (int)(pix / HoWo) : 0;
      const int p = pv ? (int)(pix - b * HoWo) : 0;
      T* yb = y + (size_t)b * P.Co * HoWo + p;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * NT);
      // vector path: the warp's 32 pixels form aligned 16-byte runs, each inside one image
      const int wpix0 = pt * kTileM + q * 32;
      const bool vec = a.vec_out && (HoWo % 8 == 0) && (wpix0 + 32 <= P.totalP);
      T* stg = reinterpret_cast<T*>(epi_stage[warp - kEpiWarp0]);
      constexpr int EPV = 16 / (int)sizeof(T);       // elements per 16-byte vector
      constexpr int VPR = 32 / EPV;                  // vectors per 32-pixel row
      constexpr int JH = sizeof(T) == 4 ? 8 : 16;    // columns staged per pass
      // this lane always stores run lane % VPR of the warp's 32 pixels (a run
      // never crosses an image since HoWo % 8 == 0): its output offset is fixed
      const int cvl = lane % VPR;
      const int rpl = wpix0 + cvl * EPV;
      const int rbl = vec ? rpl / HoWo : 0;
      T* yrun = y + (size_t)rbl * P.Co * HoWo + (rpl - rbl * HoWo);
      for (int c0 = 16 * chalf; c0 < NT; c0 += 16 * kEpiPerQuarter) {
        float v[16];
        tmem_ld16(tbase + c0, v);
        if (P.nhwc) {
          // channels-last output: the lane's pixel row holds Co contiguously, so
          // its 16 columns are one 32-byte (64 for f32) run, stored directly
          const int co = ct * NT + c0;
          if (!a.mma_bias) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += sbias[co + j];
          }
          if (pv && !DCN_SKIP(2)) {
            T* dst = y + (size_t)pix * P.Co + co;
            if (a.vec_out && (P.Co % (16 / (int)sizeof(T))) == 0 && co + 16 <= P.Co) {
              if constexpr (sizeof(T) == 4) {
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                  *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              } else {
                constexpr int kBF = OpOf<T>::kBF16;
#pragma unroll
                for (int j = 0; j < 16; j += 8)
                  *reinterpret_cast<uint4*>(dst + j) =
                      make_uint4(pack2<kBF>(v[j], v[j + 1]), pack2<kBF>(v[j + 2], v[j + 3]),
                                 pack2<kBF>(v[j + 4], v[j + 5]), pack2<kBF>(v[j + 6], v[j + 7]));
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (co + j < P.Co) dst[j] = Elem<T>::from_f(v[j]);
            }
          }
        } else if (vec) {
          if constexpr (sizeof(T) == 2) {
            // stage [8 co pairs][32 px] words (co 2p in the low half, 2p+1 in the
            // high half: one packed conversion and one 32-bit store per pair), then
            // lane (pair lane / 4, run lane % 4) reads its 8 pixels of the pair and
            // splits them into the two co rows' 16-byte runs
            constexpr int kBF = OpOf<T>::kBF16;
            const uint32_t sw = smem_u32(stg);
            if (a.mma_bias) {   // the bias is already in the accumulator
#pragma unroll
              for (int p2 = 0; p2 < 8; ++p2)
                sts_u32(sw + (p2 * 32 + lane) * 4u, pack2<kBF>(v[2 * p2], v[2 * p2 + 1]));
            } else {
#pragma unroll
              for (int p2 = 0; p2 < 8; p2 += 2) {
                const float4 b4 = *reinterpret_cast<const float4*>(sbias + ct * NT + c0 + 2 * p2);
                sts_u32(sw + (p2 * 32 + lane) * 4u, pack2<kBF>(v[2 * p2] + b4.x, v[2 * p2 + 1] + b4.y));
                sts_u32(sw + ((p2 + 1) * 32 + lane) * 4u, pack2<kBF>(v[2 * p2 + 2] + b4.z, v[2 * p2 + 3] + b4.w));
              }
            }
            __syncwarp();
            const int pp = lane >> 2;
            const uint4 w0 = lds_v4(sw + (pp * 32 + cvl * 8) * 4u);
            const uint4 w1 = lds_v4(sw + (pp * 32 + cvl * 8 + 4) * 4u);
            const uint4 ev = make_uint4(__byte_perm(w0.x, w0.y, 0x5410), __byte_perm(w0.z, w0.w, 0x5410),
                                        __byte_perm(w1.x, w1.y, 0x5410), __byte_perm(w1.z, w1.w, 0x5410));
            const uint4 od = make_uint4(__byte_perm(w0.x, w0.y, 0x7632), __byte_perm(w0.z, w0.w, 0x7632),
                                        __byte_perm(w1.x, w1.y, 0x7632), __byte_perm(w1.z, w1.w, 0x7632));
            const int co = ct * NT + c0 + 2 * pp;
            if (!DCN_SKIP(2)) {
              if (co < P.Co) *reinterpret_cast<uint4*>(yrun + (size_t)co * HoWo) = ev;
              if (co + 1 < P.Co) *reinterpret_cast<uint4*>(yrun + (size_t)(co + 1) * HoWo) = od;
            }
            __syncwarp();
          } else {
          float bz[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(sbias + ct * NT + c0 + j);
            bz[j] = b4.x; bz[j + 1] = b4.y; bz[j + 2] = b4.z; bz[j + 3] = b4.w;
          }
          // stage [JH co][32 px] (8 columns per pass for f32 so the stage stays
          // 1 KB a warp) then store 16-byte runs of pixels per co row
#pragma unroll
          for (int h = 0; h < 16 / JH; ++h) {
#pragma unroll
            for (int j = 0; j < JH; ++j)
              stg[j * 32 + lane] = Elem<T>::from_f(v[h * JH + j] + bz[h * JH + j]);
            __syncwarp();
#pragma unroll
            for (int k = 0; k < JH * VPR / 32; ++k) {
              const int j = lane / VPR + k * (32 / VPR);
              const int co = ct * NT + c0 + h * JH + j;
              if (co < P.Co && !DCN_SKIP(2)) {
                const uint4 val = *reinterpret_cast<const uint4*>(stg + j * 32 + cvl * EPV);
                *reinterpret_cast<uint4*>(yrun + (size_t)co * HoWo) = val;
              }
            }
            __syncwarp();
          }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int co = ct * NT + c0 + j;
            if (pv && co < P.Co && !DCN_SKIP(2))
              yb[(size_t)co * HoWo] = Elem<T>::from_f(a.mma_bias ? v[j] : v[j] + sbias[co]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * ab);
      if (warp == kEpiWarp0) DCN_TS(801 + 2 * it);
    }
  } else {
    regs_dec<kCtlRegs>();
    if (warp == kTmaWarp) {
    // ------------------------------------------------ weight tiles (bulk copy)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        const int ct = tile % P.nCoT;
        const uint8_t* wsrc = a.wpk + (size_t)ct * P.nK * P.wf_tile_bytes;
        for (int kc = 0; kc < P.nK; ++kc, (++s == S ? (s = 0, ph ^= 1u) : 0u)) {
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          if (DCN_SKIP(8)) continue;   // study: the stage never fills, its waits run out
          const uint32_t btile = sbase + s * stageBytes + NS * kATile;
          mbar_arrive_expect_tx(full0 + 8 * s, NS * bTile);
          bulk_g2s(btile, wsrc + (size_t)kc * P.wf_tile_bytes, NS * bTile, full0 + 8 * s);
        }
      }
    }
    } else {
    // ------------------------------------------------ MMA issuer (warp kMmaWarp: 25 for 16-bit types, 17 for f32; the next two warps idle)
    if (warp == kMmaWarp && lane == 0) {
      const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 0, 0, kTileM, NT);
      uint32_t kidx = 0;
      int ms = 0;
      uint32_t mph = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!mbar_wait(acce0 + 8 * ab, ((it >> 1) & 1) ^ 1, a.err, &abort_flag)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + (uint32_t)(ab * NT);
        const bool mbias = NS == 1 && a.mma_bias;
        if (mbias)   // D = 1 x bias^T over a K = 16 slice: the accumulator starts at the bias
          umma_f16(dt, nosw_desc(sbias_a, 128, 256),
                   nosw_desc(sbias_b + (uint32_t)(tile % P.nCoT) * (uint32_t)NT * 32u, 128, 256), idesc, 0u);
        for (int kc = 0; kc < P.nK; ++kc, ++kidx) {
          const int s = ms;
          const uint32_t ph = mph;
          if (++ms == S) { ms = 0; mph ^= 1u; }
          if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
          DCN_TS(512 + 2 * kidx);
          tc_fence_after();
          const uint32_t at = sbase + s * stageBytes;
          const uint32_t bt = at + NS * kATile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sw128_desc(at + kk * 32, 16, 1024);
            const uint64_t bd = sw128_desc(bt + kk * 32, 16, 1024);
            if (!DCN_SKIP(4)) umma_f16(dt, ad, bd, idesc, (mbias || (kc | kk) != 0) ? 1u : 0u);
            if constexpr (NS == 2) {
              const uint64_t adl = sw128_desc(at + kATile + kk * 32, 16, 1024);
              const uint64_t bdl = sw128_desc(bt + bTile + kk * 32, 16, 1024);
              umma_f16(dt, ad, bdl, idesc, 1);
              umma_f16(dt, adl, bd, idesc, 1);
            }
          }
          umma_commit(empty0 + 8 * s);
          DCN_TS(513 + 2 * kidx);
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * ab);
      }
      // drain: every issued MMA has retired before TMEM is released
      umma_commit(drain);
      mbar_wait_drain(drain, 0, a.err);
    }
  }

  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace

int launch_forward(const FwdArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  if (P.Co > kMaxCo) return DCN_E_UNSUPPORTED;
  const int NS = P.nsplit;
  const size_t stageBytes = (size_t)NS * (128 * 128 + (size_t)P.NT * 128);
  // two geometry windows built by the epilogue warps when every (tap, group) of
  // a tile fits one window and two stages still fit, else one built by the producers
  const size_t geoWin = (size_t)kGeoTaps * kTileM * (sizeof(float4) + sizeof(int));
  // the bias goes into the MMA for 16-bit types with up to two Co tiles: its A
  // and B slices (128 x 16 and nCoT x NT x 16 elements) after the fp32 bias copy
  const int mma_bias = NS == 1 && P.nCoT <= 2 && a.bias != nullptr;
  const size_t biasBytes =
      (size_t)P.nCoT * P.NT * sizeof(float) + (mma_bias ? 128 + (128 + (size_t)P.nCoT * P.NT) * 32 : 0);
  int NB = P.K2 * P.dg <= kGeoTaps ? 2 : 1;
  if (NB == 2 && (kFwdSmemBudget - 1024 - 2 * geoWin - biasBytes) / stageBytes < 2) NB = 1;
  const size_t geoBytes = NB * geoWin + biasBytes;
  int S = (int)((kFwdSmemBudget - 1024 - geoBytes) / stageBytes);
  if (S > kMaxStages) S = kMaxStages;
#ifdef DCN_STUDY
  static const int study_stages = [] {   // study switch DCN_FWD_STAGES: fewer stages, more L1
    const char* e = getenv("DCN_FWD_STAGES");
    return e ? atoi(e) : 0;
  }();
  if (study_stages >= 2 && study_stages < S) S = study_stages;
#endif
  if (S < 2) return DCN_E_UNSUPPORTED;
  FwdArgs args = a;
  args.stages = S;
  args.geo_bufs = NB;
  args.mma_bias = mma_bias;
  const size_t smem = 1024 + (size_t)S * stageBytes + geoBytes;
#ifdef DCN_STUDY
  static const int study_carve = [] {   // study switch DCN_FWD_CARVE: shared-memory carveout (%)
    const char* e = getenv("DCN_FWD_CARVE");
    if (e != nullptr) {
      const int pc = atoi(e);
      cudaFuncSetAttribute(dcn_fwd_kernel<__nv_bfloat16, 16>, cudaFuncAttributePreferredSharedMemoryCarveout, pc);
      cudaFuncSetAttribute(dcn_fwd_kernel<__half, 16>, cudaFuncAttributePreferredSharedMemoryCarveout, pc);
      return pc;
    }
    return -1;
  }();
  (void)study_carve;
#endif
  const int nTiles = P.nPT * P.nCoT;
  int grid = nTiles < a.num_sms ? nTiles : a.num_sms;
  if (grid <= 0) return DCN_OK;
  cudaError_t e;
  switch (P.dtype) {
    case DCN_F32:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<float, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      e = launch_k(dcn_fwd_kernel<float, 8>, dim3(grid), dim3(FwdLayout<8>::kThreads), smem, stream, args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<__half, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      e = launch_k(dcn_fwd_kernel<__half, 16>, dim3(grid), dim3(FwdLayout<16>::kThreads), smem, stream, args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<__nv_bfloat16, 16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      e = launch_k(dcn_fwd_kernel<__nv_bfloat16, 16>, dim3(grid), dim3(FwdLayout<16>::kThreads), smem, stream, args);
      break;
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
