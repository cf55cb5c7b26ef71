// Backward of DCNv2, data side, part 2, tile path: the same results as
// dcn_bwd_scatter.cu (grad_offset / grad_mask by the reference's coordinate
// kernel, com.cu:431-501; grad_input by its col2im scatter, com.cu:553-609; the
// sampled columns of the re-im2col, com.cu:637-706), with the grad_input
// scatter done on the tensor cores.
//
// Why: the scatter of gcol * mask * corner weight into grad_input is 4 corners x
// C fp32 adds per (pixel, tap), 1.2 GB of reductions for the README layer.  As
// L2 reductions (red.global) it is bound by the L2's rate of sector reduction
// operations: the same kernel with half-sector reductions (the channel order
// without the packed permutation) takes 406 instead of 252 us.  Here the adds
// happen in TMEM: for an output tile of 8 x 8 pixels, every sample's (pixel,
// tap) 4 corners lie (up to a margin) in a 16 x 16 window of input pixels, and
//
//   gx_window[256 window pixels, 64 ch] += A[256, 64 samples] . gcol[64 samples, 64 ch]
//
// with A the (sparse) bilinear interpolation matrix: column k holds the corner
// weights x mask of sample k at the rows of its corners.  One K step = the 64
// pixels of the tile for one tap.  After the taps, the window is added to the
// fp32 grad_input accumulator by TMA reductions of whole 128-byte rows, about
// 9x fewer sector reductions than per-sample scattering.  Corners outside the
// window go to red.global directly.
//
// Operands: the window of the packed input and each tap's gcol rows arrive as
// TMA tiles (x window 16 x 16 px x 64 ch, gcol 8 x 8 px x 64 ch, 128-byte
// swizzle); A is written into shared memory by the SIMT warps (4 entries per
// sample, K-major SW128); entries are cleared by the lane that wrote them when
// the stage comes round again, so A never needs a bulk clear.  The SIMT warps
// also read the corners (from the window, or global memory outside it) and the
// gcol slices (from the TMA tile) to form the per-sample sums S_c = gcol .
// corner_c for grad_offset / grad_mask, and the sampled columns for the weight
// gradient, exactly as the plain kernel does.  Each K step is two phases for a
// SIMT warp: the A entries (all the MMA waits for), then the gathers.
//
// CTA roles (768 threads, one CTA per SM, persistent over (tile, group) units,
// 64-channel blocks cb inside a unit):
//   warps 0-15  SIMT, two groups of 8 warps taking alternate taps: sample
//               k = 8 * (warp % 8) + lane / 4 of a K step, 4 lanes per sample
//               (two 16-byte slices of 8 channels each)
//   warps 16-19 epilogue: TMEM (window x 64 channels, fp32) -> staging in shared
//               memory -> TMA reduction (add) into the grad_input accumulator
//   warp 20     TMA: x windows (2-slot ring), gcol tiles (3-slot ring)
//   warp 21     TMEM owner and tcgen05.mma issuer (M = 128 window pixels x 2,
//               N = 64 channels, K = 64 samples per tap); warps 22-23 idle
// Used for 16-bit types when the whole backward is one pixel chunk, the image
// is at least 16 x 16 (output 8 x 8), K2 <= 16 and an 8 x 8 tile's samples span
// at most 11 input rows and columns before offsets (stride 1 with a 3 x 3
// kernel, for instance); otherwise the plain kernel runs.
#include "dcn_common.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kTH = 8, kTW = 8;           // output tile
constexpr int kWH = 16, kWW = 16;         // input window
constexpr int kWin = kWH * kWW;           // 256 window pixels (2 M tiles)
constexpr int kSimtWarps = 16;
constexpr int kEpiWarp0 = 16;
constexpr int kTmaWarp = 20, kMmaWarp = 21;
constexpr int kThreads = 24 * 32;
constexpr int kXS = 2, kAS = 2, kBS = 3;  // ring depths: x windows, A stages, gcol tiles
constexpr int kGS = 2;                    // K2 <= 8 * kGS = 16 taps (geometry table size)
constexpr uint32_t kXBytes = kWin * 128;  // 32 KB
constexpr uint32_t kABytes = kWin * 128;  // 32 KB: 2 M tiles x 128 rows x 128 B
constexpr uint32_t kBBytes = 64 * 128;    // 8 KB
constexpr uint32_t kStgBytes = 2 * 128 * 128;  // flush staging: 128 window pixels x 64 fp32 (two halves)
constexpr uint32_t kNoEntry = 0xffffffffu;

// per-stage global-timer stamps of CTA 0 (study builds with DCN_DEBUG_TS only)
#define DCN_TS(slot) \
  do { if (DCN_STUDY_ON && a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

__device__ __forceinline__ void sts_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// 4-D tiled TMA load (no multicast), completion as tx bytes on an mbarrier.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// 4-D tiled TMA reduction (add) of a shared-memory box into global memory.
// Coordinates are never negative here (the window is kept inside the image).
__device__ __forceinline__ void tma_reduce_add_4d(const void* tmap, uint32_t src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
          tmap),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// named barrier of the four epilogue warps
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// {a.x * b.x + c.x, a.y * b.y + c.y}: the sm_100 packed f32x2 FMA through the
// CUDA builtin (operands stay in register pairs; inline PTX packing them with
// mov.b64 cost extra moves)
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int i) {
  float r = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k)
    if (k == i) r = v[k];
  return r;
}

// Window origin along one axis: the tile's sample bases span
// [base0, base0 + span]; the window (size n) holds corner rows base0 + floor(o)
// .. base0 + span + floor(o) + 1 for offsets o in [-m, m) with m = (n - 1 -
// span) / 2, and is kept inside the image (so no TMA reduction starts at a
// negative coordinate).
__device__ __forceinline__ int window_origin(int base0, int span, int n, int extent) {
  int r0 = base0 - (n - 1 - span) / 2;
  if (r0 > extent - n) r0 = extent - n;
  if (r0 < 0) r0 = 0;
  return r0;
}

struct Unit {
  int b, ho0, wo0, g;
};

__device__ __forceinline__ Unit unit_of(int u, const Plan& P, int nTx, int nTy) {
  Unit r;
  r.g = u % P.dg;
  u /= P.dg;
  const int tx = u % nTx;
  u /= nTx;
  const int ty = u % nTy;
  r.b = u / nTy;
  r.ho0 = ty * kTH;
  r.wo0 = tx * kTW;
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) dcn_bwd_scatter_tc_kernel(const __grid_constant__ BwdDataArgs a) {
  const Plan& P = a.plan;
  const int nTx = (P.Wo + kTW - 1) / kTW, nTy = (P.Ho + kTH - 1) / kTH;
  const int nUnits = P.B * nTy * nTx * P.dg;
  const int K2 = P.K2, nCB = P.nCB;
  const int span_h = (kTH - 1) * P.sh + (P.kh - 1) * P.dh;
  const int span_w = (kTW - 1) * P.sw + (P.kw - 1) * P.dw;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * (kXS + kAS + kBS) + 5];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t xring = sbase;
  const uint32_t aring = xring + kXS * kXBytes;
  const uint32_t bring = aring + kAS * kABytes;
  const uint32_t stg = bring + kBS * kBBytes;
  // per-warp sample geometry of the current unit: 4 * K2 entries of 32 bytes
  const uint32_t geo = stg + kStgBytes;
  const uint32_t geo_warp_bytes = (uint32_t)(8 * ((K2 + 1) / 2)) * 32u;
  float* sbuf = reinterpret_cast<float*>(smem_raw + (geo + kSimtWarps * geo_warp_bytes - smem_u32(smem_raw)));
  const uint32_t xfull0 = smem_u32(&bars[0]), xempty0 = xfull0 + 8 * kXS;
  const uint32_t afull0 = xempty0 + 8 * kXS, aempty0 = afull0 + 8 * kAS;
  const uint32_t bfull0 = aempty0 + 8 * kAS, bempty0 = bfull0 + 8 * kBS;
  const uint32_t tfull0 = bempty0 + 8 * kBS, tempty0 = tfull0 + 16, drain = tempty0 + 16;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kXS; ++i) {
      mbar_init(xfull0 + 8 * i, 1);
      mbar_init(xempty0 + 8 * i, kSimtWarps);
    }
    for (int i = 0; i < kAS; ++i) {
      mbar_init(afull0 + 8 * i, kSimtWarps / 2);   // one group of 8 warps per A stage
      mbar_init(aempty0 + 8 * i, 1);
    }
    for (int i = 0; i < kBS; ++i) {
      mbar_init(bfull0 + 8 * i, 1);
      mbar_init(bempty0 + 8 * i, kSimtWarps / 2 + 1);   // the step's SIMT group reads it too, then the MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull0 + 8 * i, 1);
      mbar_init(tempty0 + 8 * i, 4);
    }
    mbar_init(drain, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // A stages start out zero; afterwards every entry is cleared by its writer
  for (uint32_t o = (uint32_t)tid * 16u; o < kAS * kABytes; o += kThreads * 16u)
    sts_v4(aring + o, make_uint4(0u, 0u, 0u, 0u));
  fence_proxy_async_smem();
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_slot), 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  pdl_wait();

  // registers by warpgroup (launch pool 768 x 80): SIMT 4 x 128 x 104 +
  // epilogue 128 x 40 + TMA / MMA 128 x 24 = 61440
  if (warp < kSimtWarps) {
    regs_inc<104>();
    // ------------------------------------------------ SIMT: samples, A entries
    // Two groups of 8 warps take the taps in turn: group G the taps t with
    // (t + par) % 2 == G, par = 0, or for nCB == 1 the CTA's unit count % 2 so
    // that an odd K2 balances over two units (with several channel blocks a tap
    // stays with one group, whose lanes accumulate its S sums over the blocks).
    // A stage G belongs to group G.  In a step, warp wg of the group handles
    // samples 8 wg .. 8 wg + 7, 4 lanes per sample, each lane 16 channels
    // (16-byte slices 2 q4 and 2 q4 + 1 of the 64-channel block).
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    T* __restrict__ goff = reinterpret_cast<T*>(a.goffset);
    T* __restrict__ gmsk = reinterpret_cast<T*>(a.gmask);
    const int grp = warp >> 3, wg = warp & 7;
    const int lp = lane >> 2, q4 = lane & 3;
    const int k = 8 * wg + lp;                   // sample (pixel of the tile) of this lane group
    const int kr = k >> 3, kc = k & 7;
    const int HW = P.H * P.W;
    const int nblk = P.NC / kChunk, natoms = P.nU * nblk;
    const uint32_t astage = aring + (uint32_t)grp * kABytes;   // this group's A stage
    uint32_t rem = kNoEntry;                     // the A entry this lane wrote last time
    int xs = 0;
    uint32_t xph = 0, aph = 0;
    bool ok = true;
    int n = 0;                                   // global K step counter (both groups; B slot n % kBS)
    int uit = 0;                                 // units done by this CTA
    // Global writes of a K step (its sampled columns and, for lane q4 == 0, the
    // grad_offset / grad_mask values) are issued after the group's NEXT step's A
    // entries have been fenced and published, so the proxy fence before that
    // publication does not wait for them.
    uint4* dcol = nullptr;
    uint4 vcol0 = make_uint4(0u, 0u, 0u, 0u), vcol1 = vcol0;
    T* doff = nullptr;
    T* dmsk = nullptr;
    int doffs = 0;
    T vh = Elem<T>::from_f(0.f), vw = vh, vm = vh;
    auto flush_deferred = [&]() {
      if (dcol != nullptr) {
        dcol[0] = vcol0;
        dcol[1] = vcol1;
      }
      if (doff != nullptr) {
        doff[0] = vh;
        doff[doffs] = vw;
        *dmsk = vm;
      }
      dcol = nullptr;
      doff = nullptr;
    };
    // geometry table of this warp for the current unit: its 8 samples x the
    // taps of its group, entries of 32 bytes
    const uint32_t gtab = geo + (uint32_t)warp * geo_warp_bytes;
    for (int u = blockIdx.x; u < nUnits && ok; u += gridDim.x, ++uit) {
      const Unit un = unit_of(u, P, nTx, nTy);
      const int par = nCB == 1 ? (uit & 1) : 0;
      const int t0 = (grp + par) & 1;            // first tap of this group
      const int ho = un.ho0 + kr, wo = un.wo0 + kc;
      const bool pv = ho < P.Ho && wo < P.Wo;
      const int p = ho * P.Wo + wo;
      const int pix = un.b * P.HoWo + p;         // flat pixel (one chunk: pix0 == 0)
      const int r0 = window_origin(un.ho0 * P.sh - P.ph, span_h, kWH, P.H);
      const int c0 = window_origin(un.wo0 * P.sw - P.pw, span_w, kWW, P.W);
      {
        // entry j = (sample 8 wg + j % 8, tap t0 + 2 (j / 8)) by lane j % 32
        const int nE = 8 * ((K2 - t0 + 1) / 2);
        for (int j0 = 0; j0 < nE; j0 += 32) {
          const int j = j0 + lane;
          const int ke = 8 * wg + (j & 7), te = t0 + 2 * (j >> 3);
          const int hoe = un.ho0 + (ke >> 3), woe = un.wo0 + (ke & 7);
          const bool pve = j < nE && hoe < P.Ho && woe < P.Wo;
          uint32_t rh = 0u, rw = 0u, rm = 0u;
          if (pve) {
            const int pe = hoe * P.Wo + woe;
            const int ob = un.b * P.off_bs + (un.g * 2 * K2 + 2 * te) * P.off_cs + pe * P.off_ps;
            rh = ldg_raw<T>(off + ob);
            rw = ldg_raw<T>(off + ob + P.off_cs);
            rm = ldg_raw<T>(msk + un.b * P.msk_bs + (un.g * K2 + te) * P.msk_cs + pe * P.msk_ps);
          }
          if (j < nE) {
            const int ie = te / P.kw, je = te - ie * P.kw;
            const float h = (float)(hoe * P.sh - P.ph + ie * P.dh) + raw_to_f<T>(rh);
            const float w = (float)(woe * P.sw - P.pw + je * P.dw) + raw_to_f<T>(rw);
            float mv = raw_to_f<T>(rm);
            if (P.mask_logit) mv = 1.f / (1.f + __expf(-mv));   // sigmoid of a predictor logit
            const float hf = floorf(h), wf = floorf(w);
            const int hl = (int)hf, wl = (int)wf;
            uint32_t cv = 0u;
            if (pve && (h > -1.f) && (w > -1.f) && (h < (float)P.H) && (w < (float)P.W)) {
              const bool rr0 = hl >= 0, rr1 = hl + 1 <= P.H - 1, cc0 = wl >= 0, cc1 = wl + 1 <= P.W - 1;
              cv = (rr0 && cc0 ? 1u : 0u) | (rr0 && cc1 ? 2u : 0u) | (rr1 && cc0 ? 4u : 0u) | (rr1 && cc1 ? 8u : 0u);
            }
            uint32_t wpk[2] = {0u, 0u};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int wr = hl + (c >> 1) - r0, wc = wl + (c & 1) - c0;
              const int wp = ((cv >> c) & 1u) && wr >= 0 && wr < kWH && wc >= 0 && wc < kWW ? wr * kWW + wc : -1;
              wpk[c >> 1] |= ((uint32_t)wp & 0xffffu) << (16 * (c & 1));
            }
            const uint32_t ea = gtab + (uint32_t)j * 32u;
            sts_v4(ea, make_uint4(wpk[0], wpk[1], cv, (uint32_t)(un.b * HW + hl * P.W + wl)));
            sts_v4(ea + 16u, make_uint4(__float_as_uint(h - hf), __float_as_uint(w - wf),
                                        __float_as_uint(pve ? mv : 0.f), 0u));
          }
        }
        __syncwarp();
      }
      for (int cb = 0; cb < nCB && ok; ++cb) {
        if (!mbar_wait_warp(xfull0 + 8 * xs, xph, a.err, &abort_flag)) { ok = false; break; }
        const uint32_t xwin = xring + xs * kXBytes;
        for (int t = 0; t < K2; ++t, ++n) {
          if (((t + par) & 1) != grp) continue;
          const int bs = n % kBS;
          const uint32_t bph = (uint32_t)(n / kBS) & 1u;
          const int nch = (int)((uint32_t)n >> 1);
          if (warp == 0 && nch < 260) DCN_TS(3 * nch);
          // phase 1 (feeds the MMA): this sample's A entries
          if (!mbar_wait_warp(aempty0 + 8 * grp, aph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          if (rem != kNoEntry) sts_u16(rem, 0);   // clear what this lane wrote last time round
          const uint32_t ea = gtab + (uint32_t)(8 * ((t - t0) >> 1) + lp) * 32u;
          const uint4 e0 = lds_v4(ea), e1 = lds_v4(ea + 16u);
          const uint32_t cval = e0.z;
          const int gi0 = (int)e0.w;
          const float lh = __uint_as_float(e1.x), lw = __uint_as_float(e1.y), m = __uint_as_float(e1.z);
          const float hh = 1.f - lh, hw = 1.f - lw;
          const float bw[4] = {(cval & 1u) ? hh * hw : 0.f, (cval & 2u) ? hh * lw : 0.f,
                               (cval & 4u) ? lh * hw : 0.f, (cval & 8u) ? lh * lw : 0.f};
          int wpix[4];
#pragma unroll
          for (int c = 0; c < 4; ++c)
            wpix[c] = (int)(int16_t)(((c < 2 ? e0.x : e0.y) >> (16 * (c & 1))) & 0xffffu);
          // A entry of corner q4: row = window pixel, column = sample
          rem = kNoEntry;
          if (!DCN_SKIP(1 << 17)) {
            float bq = 0.f;
            int wp = -1;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (c == q4) { bq = bw[c]; wp = wpix[c]; }
            const float wcm = bq * m;
            if (wp >= 0 && wcm != 0.f) {
              const int mt = wp >> 7, rr = wp & 127;
              rem = astage + (uint32_t)mt * 16384u + (uint32_t)rr * 128u +
                    (uint32_t)(((k >> 3) ^ (rr & 7)) << 4) + (uint32_t)(k & 7) * 2u;
              uint16_t hv;
              if constexpr (OpOf<T>::kBF16) hv = __bfloat16_as_ushort(__float2bfloat16_rn(wcm));
              else hv = __half_as_ushort(__float2half_rn(wcm));
              sts_u16(rem, hv);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(afull0 + 8 * grp);
          aph ^= 1u;
          flush_deferred();
          if (warp == 0 && nch < 260) DCN_TS(3 * nch + 1);
          // phase 2: corners and gcol -> S sums, sampled columns, out-of-window scatter
          if (!mbar_wait_warp(bfull0 + 8 * bs, bph, a.err, &abort_flag)) { ok = false; break; }
          const uint32_t bstage = bring + bs * kBBytes;
          const int cofs = un.g * P.Cgp + cb * kChunk;
          // the lane's two 8-channel slices one after the other (registers)
          float S[4] = {0.f, 0.f, 0.f, 0.f};
          uint4 vcs[2];
          float gcs[2][8];
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            if (DCN_SKIP(1 << 16)) { vcs[jj] = make_uint4(0u, 0u, 0u, 0u); continue; }
            const int sl = 2 * q4 + jj;
            uint4 raw[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if (wpix[c] >= 0) {
                raw[c] = lds_v4(xwin + (uint32_t)wpix[c] * 128u + (uint32_t)((sl ^ (wpix[c] & 7)) << 4));
              } else if ((cval >> c) & 1u) {
                const int gi = gi0 + (c >> 1) * P.W + (c & 1);
                raw[c] = ldg_nc_v4(xt + (size_t)(unsigned)(gi * P.CS + cofs + sl * 8));
              } else {
                raw[c] = make_uint4(0u, 0u, 0u, 0u);
              }
            }
            unpack8<T>(lds_v4(bstage + (uint32_t)k * 128u + (uint32_t)((sl ^ (k & 7)) << 4)), gcs[jj]);
            // packed f32x2 arithmetic: two channels per instruction
            float2 col2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float wcm = bw[c] * m;
              float v[8];
              unpack8<T>(raw[c], v);
              float2 sp = make_float2(0.f, 0.f);
#pragma unroll
              for (int e = 0; e < 8; e += 2) {
                const float2 ve = make_float2(v[e], v[e + 1]);
                sp = fma2(make_float2(gcs[jj][e], gcs[jj][e + 1]), ve, sp);
                col2[e >> 1] = fma2(ve, make_float2(wcm, wcm), col2[e >> 1]);
              }
              S[c] += sp.x + sp.y;
            }
            constexpr int kBF = OpOf<T>::kBF16;
            vcs[jj] = make_uint4(pack2<kBF>(col2[0].x, col2[0].y), pack2<kBF>(col2[1].x, col2[1].y),
                                 pack2<kBF>(col2[2].x, col2[2].y), pack2<kBF>(col2[3].x, col2[3].y));
          }
          // sampled columns for the weight gradient (B tiles of dcn_bwd_weight)
          if (pv && a.cols != nullptr && !DCN_SKIP(1 << 18)) {
            const int crow = pix & 63;
            const int cch = cb / nblk, cblk = cb - cch * nblk;
            const int atom = ((t * P.dg + un.g) * P.nCC + cch) * nblk + cblk;
            uint8_t* rowp = a.cols + ((size_t)(unsigned)(pix >> 6) * P.nsplit * natoms + atom) * 8192u + crow * 128;
            // slices 2 q4 and 2 q4 + 1 of the swizzled row are the two chunks of
            // one 32-byte pair ((2 q4) ^ r and (2 q4 + 1) ^ r differ in bit 0):
            // odd rows hold them in swapped order
            const bool odd = (crow & 1) != 0;
            vcol0 = odd ? vcs[1] : vcs[0];
            vcol1 = odd ? vcs[0] : vcs[1];
            dcol = reinterpret_cast<uint4*>(rowp + ((((2 * q4) ^ (crow & 7)) & ~1) << 4));
          }
          // corners outside the window: straight into the accumulator
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (wpix[c] < 0 && ((cval >> c) & 1u)) {
              const float sk = bw[c] * m;
              const int gi = gi0 + (c >> 1) * P.W + (c & 1);
              float* dst = a.gx_nhwc + (size_t)(unsigned)(gi * P.CS + cofs);
#pragma unroll
              for (int jj = 0; jj < 2; ++jj) {
                const int sl = 2 * q4 + jj;
                red_add_v4(dst + slice_lo(sl), gcs[jj][0] * sk, gcs[jj][1] * sk, gcs[jj][2] * sk,
                           gcs[jj][3] * sk);
                red_add_v4(dst + slice_hi(sl), gcs[jj][4] * sk, gcs[jj][5] * sk, gcs[jj][6] * sk,
                           gcs[jj][7] * sk);
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bempty0 + 8 * bs);
          if (warp == 0 && nch < 260) DCN_TS(3 * nch + 2);
          // per-sample sums over the 4 lanes' channels
          if (DCN_SKIP(1 << 19)) continue;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            S[c] += __shfl_xor_sync(0xffffffffu, S[c], 1);
            S[c] += __shfl_xor_sync(0xffffffffu, S[c], 2);
          }
          if (q4 == 0 && pv) {
            if (nCB > 1) {
              float* sb = sbuf + ((size_t)t * 64 + k) * 4;
#pragma unroll
              for (int c = 0; c < 4; ++c) sb[c] = cb == 0 ? S[c] : sb[c] + S[c];
              if (cb == nCB - 1) {
#pragma unroll
                for (int c = 0; c < 4; ++c) S[c] = sb[c];
              }
            }
            if (cb == nCB - 1) {
              const float am = bw[0] * S[0] + bw[1] * S[1] + bw[2] * S[2] + bw[3] * S[3];
              const float ah = hw * (S[2] - S[0]) + lw * (S[3] - S[1]);
              const float aw = hh * (S[1] - S[0]) + lh * (S[3] - S[2]);
              const int ob = un.b * P.off_bs + (un.g * 2 * K2 + 2 * t) * P.off_cs + p * P.off_ps;
              doff = goff + ob;
              doffs = P.off_cs;
              dmsk = gmsk + un.b * P.msk_bs + (un.g * K2 + t) * P.msk_cs + p * P.msk_ps;
              vh = Elem<T>::from_f(ah * m);
              vw = Elem<T>::from_f(aw * m);
              vm = Elem<T>::from_f(P.mask_logit ? am * m * (1.f - m) : am);
            }
          }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(xempty0 + 8 * xs);
        if (++xs == kXS) { xs = 0; xph ^= 1u; }
      }
    }
    flush_deferred();
  } else if (warp < kTmaWarp) {
    regs_dec<40>();
    // ------------------------------------------------ epilogue: window -> grad_input accumulator
    const int qd = warp & 3;                     // TMEM lane quarter
    // CTA 0 first zeroes the sampled columns of the pixels past the end of the
    // last 64-pixel block (the weight gradient reads whole blocks)
    if (blockIdx.x == 0 && a.cols != nullptr && (P.totalP & 63) != 0) {
      const int natoms = P.nU * (P.NC / kChunk);
      const int lastb = (int)(P.totalP >> 6), r0p = (int)(P.totalP & 63);
      const int nrow = (64 - r0p) * P.nsplit * natoms;
      for (int idx = (warp - kEpiWarp0) * 32 + lane; idx < nrow * 8; idx += 128) {
        const int row = idx >> 3, ch = idx & 7;
        const int atom = row / (64 - r0p), rr = r0p + row % (64 - r0p);
        *reinterpret_cast<uint4*>(a.cols + ((size_t)lastb * P.nsplit * natoms + atom) * 8192u + rr * 128 + ch * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
    }
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < nUnits && ok; u += gridDim.x) {
      const Unit un = unit_of(u, P, nTx, nTy);
      const int r0 = window_origin(un.ho0 * P.sh - P.ph, span_h, kWH, P.H);
      const int c0 = window_origin(un.wo0 * P.sw - P.pw, span_w, kWW, P.W);
      for (int cb = 0; cb < nCB; ++cb, ++it) {
        const int ab = it & 1;
        if (!mbar_wait_warp(tfull0 + 8 * ab, (it >> 1) & 1, a.err, &abort_flag)) { ok = false; break; }
        if (warp == kEpiWarp0 && it < 10) DCN_TS(1002 + 2 * it);
        tc_fence_after();
#pragma unroll 1
        for (int mt = 0; mt < 2; ++mt) {
          // M tile mt = window rows 8 mt .. 8 mt + 7: TMEM -> staging (two
          // 32-channel halves, 128-byte rows, logical channel order, 128-byte
          // swizzle) -> one TMA reduction (add) per half into the accumulator
          const int r = qd * 32 + lane;
          const uint32_t tb = tmem_base + ((uint32_t)(qd * 32) << 16) + (uint32_t)(ab * 128 + mt * 64);
#pragma unroll 1
          for (int quarter = 0; quarter < 4; ++quarter) {
            float v[16];
            tmem_ld16(tb + quarter * 16, v);
#pragma unroll
            for (int j4 = 0; j4 < 2; ++j4) {
              const int jq = quarter * 2 + j4;   // physical 8-channel slice of these columns
              const int llo = slice_lo(jq), lhi = slice_hi(jq);
              sts_v4(stg + (uint32_t)(llo >> 5) * 16384u + (uint32_t)r * 128u +
                         (uint32_t)((((llo & 31) >> 2) ^ (r & 7)) << 4),
                     make_uint4(__float_as_uint(v[8 * j4]), __float_as_uint(v[8 * j4 + 1]),
                                __float_as_uint(v[8 * j4 + 2]), __float_as_uint(v[8 * j4 + 3])));
              sts_v4(stg + (uint32_t)(lhi >> 5) * 16384u + (uint32_t)r * 128u +
                         (uint32_t)((((lhi & 31) >> 2) ^ (r & 7)) << 4),
                     make_uint4(__float_as_uint(v[8 * j4 + 4]), __float_as_uint(v[8 * j4 + 5]),
                                __float_as_uint(v[8 * j4 + 6]), __float_as_uint(v[8 * j4 + 7])));
            }
          }
          fence_proxy_async_smem();
          epi_bar();
          if (warp == kEpiWarp0 && lane == 0) {
            const int cx = un.g * P.Cgp + cb * kChunk;
            tma_reduce_add_4d(&a.rmap, stg, cx, c0, r0 + mt * 8, un.b);
            tma_reduce_add_4d(&a.rmap, stg + 16384u, cx + 32, c0, r0 + mt * 8, un.b);
            bulk_commit();
            bulk_wait_read();
          }
          epi_bar();
        }
        if (warp == kEpiWarp0 && it < 10) DCN_TS(1003 + 2 * it);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * ab);
      }
    }
  } else {
    regs_dec<24>();
    if (warp == kTmaWarp) {
      // ---------------------------------------------- TMA: x windows and gcol tiles
      if (lane == 0) {
        int xs = 0, bs = 0;
        uint32_t xph = 0, bph = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < nUnits && ok; u += gridDim.x) {
          const Unit un = unit_of(u, P, nTx, nTy);
          const int r0 = window_origin(un.ho0 * P.sh - P.ph, span_h, kWH, P.H);
          const int c0 = window_origin(un.wo0 * P.sw - P.pw, span_w, kWW, P.W);
          for (int cb = 0; cb < nCB && ok; ++cb) {
            if (!mbar_wait(xempty0 + 8 * xs, xph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(xfull0 + 8 * xs, kXBytes);
            tma_load_4d(xring + xs * kXBytes, &a.xmap, un.g * P.Cgp + cb * kChunk, c0, r0, un.b, xfull0 + 8 * xs);
            if (++xs == kXS) { xs = 0; xph ^= 1u; }
            for (int t = 0; t < K2; ++t) {
              if (!mbar_wait(bempty0 + 8 * bs, bph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
              mbar_arrive_expect_tx(bfull0 + 8 * bs, kBBytes);
              tma_load_4d(bring + bs * kBBytes, &a.cmap, (t * P.dg + un.g) * P.Cgp + cb * kChunk, un.wo0, un.ho0,
                          un.b, bfull0 + 8 * bs);
              if (++bs == kBS) { bs = 0; bph ^= 1u; }
            }
          }
        }
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------- MMA issuer
      if (lane == 0) {
        constexpr int kBF = OpOf<T>::kBF16;
        const uint32_t idesc = make_idesc(kBF, 0, 1, 128, 64);   // A K-major, B MN-major
        int bs = 0, it = 0, mch = 0, uit = 0;
        uint32_t aph2 = 0, bph = 0;              // bit s: phase of A stage s
        bool ok = true;
        for (int u = blockIdx.x; u < nUnits && ok; u += gridDim.x, ++uit) {
          const int par = nCB == 1 ? (uit & 1) : 0;
          for (int cb = 0; cb < nCB && ok; ++cb, ++it) {
            const int ab = it & 1;
            if (!mbar_wait(tempty0 + 8 * ab, ((it >> 1) & 1) ^ 1, a.err, &abort_flag)) { ok = false; break; }
            tc_fence_after();
            for (int t = 0; t < K2; ++t, ++mch) {
              const int as_ = (t + par) & 1;       // the SIMT group (and A stage) of this tap
              const uint32_t aph = (aph2 >> as_) & 1u;
              if (!mbar_wait(afull0 + 8 * as_, aph, a.err, &abort_flag)) { ok = false; break; }
              if (!mbar_wait(bfull0 + 8 * bs, bph, a.err, &abort_flag)) { ok = false; break; }
              if (mch < 100) DCN_TS(800 + 2 * mch);
              tc_fence_after();
              const uint32_t astage = aring + as_ * kABytes, bstage = bring + bs * kBBytes;
#pragma unroll
              for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                  const uint64_t ad = sw128_desc(astage + mt * 16384u + kk * 32u, 16, 1024);
                  const uint64_t bd = sw128_desc(bstage + kk * 2048u, 8192, 1024);
                  umma_f16(tmem_base + (uint32_t)(ab * 128 + mt * 64), ad, bd, idesc, (t | kk) != 0);
                }
              }
              umma_commit(aempty0 + 8 * as_);
              umma_commit(bempty0 + 8 * bs);
              if (mch < 100) DCN_TS(801 + 2 * mch);
              aph2 ^= 1u << as_;
              if (++bs == kBS) { bs = 0; bph ^= 1u; }
            }
            if (!ok) break;
            umma_commit(tfull0 + 8 * ab);
          }
        }
        umma_commit(drain);
        mbar_wait_drain(drain, 0, a.err);
      }
    }
  }
  if (warp == kEpiWarp0 && lane == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace

size_t backward_scatter_tc_smem(const Plan& P) {
  return 1024 + (size_t)kXS * kXBytes + (size_t)kAS * kABytes + (size_t)kBS * kBBytes + kStgBytes +
         (size_t)kSimtWarps * 8 * ((P.K2 + 1) / 2) * 32 + (P.nCB > 1 ? (size_t)P.K2 * 64 * 4 * sizeof(float) : 0);
}

bool backward_scatter_tc_eligible(const Plan& P) {
  if (P.esz != 2 || P.gcol_chunk < P.totalP || P.totalP <= 0 || P.K2 > 8 * kGS) return false;
  // every TMA box inside the tensor's extent (no box larger than the tensor),
  // and a window margin of at least 1.5 px
  if (P.H < kWH || P.W < kWW || P.Ho < kTH || P.Wo < kTW) return false;
  if ((kTH - 1) * P.sh + (P.kh - 1) * P.dh > kWH - 5) return false;
  if ((kTW - 1) * P.sw + (P.kw - 1) * P.dw > kWW - 5) return false;
  return backward_scatter_tc_smem(P) <= kBwdSmemLimit;
}

int launch_backward_scatter_tc(const BwdDataArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const long long nUnits = (long long)P.B * ((P.Ho + kTH - 1) / kTH) * ((P.Wo + kTW - 1) / kTW) * P.dg;
  if (nUnits <= 0) return DCN_OK;
  const int grid = (int)(nUnits < a.num_sms ? nUnits : a.num_sms);
  const size_t smem = backward_scatter_tc_smem(P);
  cudaError_t e;
  if (P.dtype == DCN_F16) {
    e = cudaFuncSetAttribute(dcn_bwd_scatter_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e == cudaSuccess)
      e = launch_k(dcn_bwd_scatter_tc_kernel<__half>, dim3(grid), dim3(kThreads), smem, stream, a);
  } else {
    e = cudaFuncSetAttribute(dcn_bwd_scatter_tc_kernel<__nv_bfloat16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = launch_k(dcn_bwd_scatter_tc_kernel<__nv_bfloat16>, dim3(grid), dim3(kThreads), smem, stream, a);
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
