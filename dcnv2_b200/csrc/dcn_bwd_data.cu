// Backward of DCNv2 with respect to the data-side inputs (input, offset, mask),
// as one persistent warp-specialised kernel.  Replaces, per batch, the
// reference's cuBLAS  columns = W^T . grad_out  (com.cu:789-793), the coordinate
// kernel (com.cu:431-501) and the col2im scatter (com.cu:553-609):
//
//   gcol[pixel, (t,g,c)] = sum_co grad_out[b, co, pixel] * W[co, g*Cg + c, t]
//       -- tcgen05 GEMM, M = 128 pixels, N = a channel chunk of one (tap, group),
//          K = Co; the result stays in TMEM and never reaches HBM
//   grad_mask[b, g*T+t, p]     = sum_c gcol * bilinear(x_c)
//   grad_offset[b, 2(gT+t)+d, p] = mask * sum_c gcol * d bilinear(x_c) / d(h|w)
//   grad_input[b, c, corner]  += gcol * mask * corner weight    (fp32 vector red.add)
//
// CTA roles (448 threads):
//   warp 0      bulk copies of pre-packed grad_out chunks (128 pixels x 64 Co,
//               K-major SW128) into an smem ring, once per tile when all Co chunks fit
//               (warps 1-3 idle)
//   warps 4-11  epilogue: gcol TMEM -> smem transpose, then 8 lanes per pixel
//               gather the 4 bilinear corner lines, reduce and scatter
//   warp 12     bulk-copy producer of the pre-packed W^T tile (K-major SW128)
//   warp 13     TMEM owner and tcgen05.mma issuer
// The accumulator is double-buffered in TMEM (unit u in buffer u & 1) so the
// heavy epilogue of one (tap, group) overlaps the GEMM of the next.
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_gout.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

#define DCN_TS(slot) \
  do { if (a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

constexpr int kThreads = 512;  // 4 warpgroups
constexpr int kAWarps = 4;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kTmaWarp = 12;
constexpr int kMmaWarp = 13;

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    dcn_bwd_data_kernel(const __grid_constant__ BwdDataArgs a) {
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;
  const Plan& P = a.plan;
  const int NC = P.NC;
  const uint32_t bTile = (uint32_t)NC * 128u;
  const uint32_t stageBytes = NS * bTile;          // one W^T stage (B operand)
  const uint32_t aSlot = NS * kATile;              // one grad_out chunk (A operand)
  const int S = a.stages;
  const int RA = a.a_slots;
  // A chunks (128 pixels x 64 Co) are loaded once per tile and reused by every
  // unit when the ring holds all Co chunks (resident), else re-streamed per unit
  const bool resident = RA >= P.nKo;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 7];
  __shared__ __align__(8) uint64_t abars[2 * kMaxASlots];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 2]);
  const uint32_t trf = smem_u32(&bars[2 * kMaxStages + 4]);  // transpose buffer filled
  const uint32_t tre = smem_u32(&bars[2 * kMaxStages + 5]);  // transpose buffer consumed
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 6]);
  const uint32_t afull0 = smem_u32(&abars[0]);
  const uint32_t aempty0 = smem_u32(&abars[kMaxASlots]);
  const uint32_t abase = sbase + (uint32_t)S * stageBytes;   // A ring after the B stages

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int r = 0; r < RA; ++r) {
      mbar_init(afull0 + 8 * r, 1);
      mbar_init(aempty0 + 8 * r, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, kEpiWarps);
    }
    mbar_init(trf, kEpiWarps);
    mbar_init(tre, kEpiWarps);
    mbar_init(drain, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * NC)) tmem_cols <<= 1;
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_slot), tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  const int nTiles = P.nPT;
  if (warp == kMmaWarp) DCN_TS(1000);
  const int HoWo = P.HoWo;

  // Roles by warpgroup.  setmaxnreg sits at the top of each warpgroup's branch
  // (one instruction per warpgroup): the two epilogue warpgroups grow to 200
  // registers, the loader/idle and control warpgroups shrink to 56.
  if (warp >= kEpiWarp0 && warp < kTmaWarp) {
    regs_inc<200>();
    // ------------------------------------------------ epilogue
    // Per unit (tap t, group g, channel chunk cch) and per pass of CB channels:
    //  A) TMEM -> smem transpose buffer (thread = pixel row); after the last pass
    //     the TMEM buffer goes back to the MMA warp;
    //  B) 8 lanes per pixel, each on 8 channels of the pixel's corner lines:
    //     gather the 4 corners, reduce bilinear / d/dh / d/dw against gcol, and
    //     scatter gcol * mask * corner weight with vector red.add.
    // Geometry: lane r < 16 of epilogue warp e owns row 16e + r (offsets
    // prefetched one (tap, group) ahead) and broadcasts it to the gather lanes.
    using GS = GatherShape<T>;
    constexpr int LPP = GS::kLPP, PPI = GS::kPPI, LD = GS::kLD;
    constexpr int ITER = 16 / PPI;                // pixels per lane and pass
    constexpr int BATCH = sizeof(T) == 4 ? 2 : 4;
    const int ew = warp - kEpiWarp0;              // 0..7
    const int q4 = warp & 3;                      // TMEM lane quarter
    const int lp = lane / LPP, q = lane % LPP;
    const int CB = a.tb_ch;                       // channels per pass (64 or 128)
    const int npass = NC / CB;
    const uint32_t tbuf = abase + (uint32_t)RA * aSlot;  // [128][CB] fp32, chunk-swizzled
    const uint32_t rowB = (uint32_t)CB * 4u;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    T* __restrict__ goff = reinterpret_cast<T*>(a.goffset);
    T* __restrict__ gmsk = reinterpret_cast<T*>(a.gmask);
    const int HW = P.H * P.W;
    const int nTG = P.K2 * P.dg;
    uint32_t ucnt = 0, trcnt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      // this lane's geometry row
      const int mpix = tile * kTileM + ew * 16 + (lane & 15);
      const bool mpv = mpix < P.totalP;
      const int mb = mpv ? (int)(mpix / HoWo) : 0;
      const int mp = mpv ? (int)(mpix - mb * HoWo) : 0;
      const int mho = mp / P.Wo, mwo = mp - mho * P.Wo;
      uint32_t rh = 0, rw = 0, rm = 0;  // raw prefetched offset / mask bits
      auto fetch_raw = [&](int tg) {
        if (!mpv) return;
        const int t = tg / P.dg, g = tg - t * P.dg;
        const int ob = ((mb * P.dg + g) * 2 * P.K2 + 2 * t) * HoWo + mp;
        rh = ldg_raw<T>(off + (ob));
        rw = ldg_raw<T>(off + (ob + HoWo));
        rm = ldg_raw<T>(msk + (((mb * P.dg + g) * P.K2 + t) * HoWo + mp));
      };
      fetch_raw(0);
      // grad_offset / grad_mask bases (offset[b][0][p], mask[b][0][p]) of this lane's
      // pixels, -1 for padding rows
      int wob[ITER], wmb[ITER];
#pragma unroll
      for (int it = 0; it < ITER; ++it) {
        const int pix = tile * kTileM + ew * 16 + it * PPI + lp;
        wob[it] = wmb[it] = -1;
        if (pix < P.totalP) {
          const int b = pix / HoWo, p = pix - b * HoWo;
          wob[it] = b * P.dg * 2 * P.K2 * HoWo + p;
          wmb[it] = b * P.dg * P.K2 * HoWo + p;
        }
      }
      float racc[ITER][3];
      int gidx[ITER];
      float glh[ITER], glw[ITER], gm[ITER];
      uint32_t gval[ITER];
      // this lane's row geometry for (tap, group) tg from the prefetched raw values
      // (and the prefetch of tg + 1)
      int mi = 0;
      float mlh = 0.f, mlw = 0.f, mm = 0.f;
      uint32_t mval = 0u;
      auto compute_mine = [&](int tg) {
        const int t = tg / P.dg;
        const int i = t / P.kw, j = t - i * P.kw;
        mi = 0;
        mlh = mlw = mm = 0.f;
        mval = 0u;
        if (mpv) {
          const float h = (float)(mho * P.sh - P.ph + i * P.dh) + raw_to_f<T>(rh);
          const float w = (float)(mwo * P.sw - P.pw + j * P.dw) + raw_to_f<T>(rw);
          mm = raw_to_f<T>(rm);
          const float hf = floorf(h), wf = floorf(w);
          const int hl = (int)hf, wl = (int)wf;
          mlh = h - hf;
          mlw = w - wf;
          if ((h > -1.f) && (w > -1.f) && (h < (float)P.H) && (w < (float)P.W) && !(a.dbg & 1)) {
            const bool r0 = hl >= 0, r1 = hl + 1 <= P.H - 1, c0 = wl >= 0, c1 = wl + 1 <= P.W - 1;
            mval = (r0 && c0 ? 1u : 0u) | (r0 && c1 ? 2u : 0u) | (r1 && c0 ? 4u : 0u) |
                   (r1 && c1 ? 8u : 0u);
            mi = mb * HW + hl * P.W + wl;
          }
        }
        if (tg + 1 < nTG) fetch_raw(tg + 1);
      };
      compute_mine(0);
      for (int u = 0; u < P.nU && ok; ++u, ++ucnt) {
        const int tg = u / P.nCC;
        const int cch = u - tg * P.nCC;
        const int t = tg / P.dg, g = tg - t * P.dg;
        if (cch == 0) {
          if (tg > 0) compute_mine(tg);
#pragma unroll
          for (int it = 0; it < ITER; ++it) {
            const int src = it * PPI + lp;
            racc[it][0] = racc[it][1] = racc[it][2] = 0.f;
            gidx[it] = __shfl_sync(0xffffffffu, mi, src);
            glh[it] = __shfl_sync(0xffffffffu, mlh, src);
            glw[it] = __shfl_sync(0xffffffffu, mlw, src);
            gm[it] = __shfl_sync(0xffffffffu, mm, src);
            gval[it] = __shfl_sync(0xffffffffu, mval, src);
          }
        }
        if (ew == 0) DCN_TS(4 * ucnt);
        const int ab = ucnt & 1;
        if (!mbar_wait(accf0 + 8 * ab, (ucnt >> 1) & 1, a.err, &abort_flag)) { ok = false; break; }
        if (ew == 0) DCN_TS(4 * ucnt + 1);
        tc_fence_after();
        for (int pass = 0; pass < npass && ok; ++pass, ++trcnt) {
          const int c0ch = cch * NC + pass * CB;  // first channel (within the group) of the pass
          int cend = P.Cgp - c0ch;
          if (cend > CB) cend = CB;
          // ---- A: TMEM -> transpose buffer
          if (!mbar_wait(tre, (trcnt & 1) ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          {
            const int row = q4 * 32 + lane;
            const uint32_t tb =
                tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(ab * NC + pass * CB);
            const int half = ew >> 2;
            const uint32_t rbase = tbuf + (uint32_t)row * rowB;
            const uint32_t sw = (uint32_t)(row & 7);
            for (int c0 = half * (CB / 2); c0 < (half + 1) * (CB / 2); c0 += 16) {
              float v[16];
              tmem_ld16(tb + c0, v);
              const uint32_t ck = (uint32_t)(c0 >> 2);  // 16-byte chunk index
#pragma unroll
              for (int k = 0; k < 4; ++k)
                sts_v4(rbase + (((ck + k) ^ sw) << 4),
                       make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                  __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3])));
            }
          }
          if (pass == npass - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce0 + 8 * ab);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(trf);
          if (!mbar_wait(trf, trcnt & 1, a.err, &abort_flag)) { ok = false; break; }
          if (ew == 0) DCN_TS(4 * ucnt + 2);
          // ---- B: gather, reduce, scatter (all corner loads of a batch in flight)
          const int d[4] = {0, 1, P.W, P.W + 1};
          for (int cs = 0; cs < cend; cs += kChunk) {
            // lane q owns packed slice q = logical channels [4q, 4q+4) and
            // [32+4q, 32+4q+4) of the 64-channel block (perm_logical): one 16-byte
            // load per corner from the packed input, and each red.add instruction
            // of a pixel's 8 lanes fills whole 32-byte sectors of grad_input
            const int ch = cs + q * 8;                      // packed position in the pass
            const int cofs = g * P.Cgp + c0ch + ch;         // packed input
            const int lofs = g * P.Cgp + c0ch + cs + 4 * q;  // grad_input (logical order)
#pragma unroll
            for (int i0 = 0; i0 < ITER; i0 += BATCH) {
              uint4 raw[BATCH][4][LD];
              float gc[BATCH][8];
#pragma unroll
              for (int k = 0; k < BATCH; ++k) {
                const int it = i0 + k;
                const int row = ew * 16 + it * PPI + lp;
                const uint32_t rbase = tbuf + (uint32_t)row * rowB;
                const uint32_t ck = (uint32_t)(ch >> 2), sw = (uint32_t)(row & 7);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  uint4 r4;
                  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                               : "=r"(r4.x), "=r"(r4.y), "=r"(r4.z), "=r"(r4.w)
                               : "r"(rbase + (((ck + h) ^ sw) << 4)));
                  gc[k][4 * h + 0] = __uint_as_float(r4.x);
                  gc[k][4 * h + 1] = __uint_as_float(r4.y);
                  gc[k][4 * h + 2] = __uint_as_float(r4.z);
                  gc[k][4 * h + 3] = __uint_as_float(r4.w);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                  for (int l = 0; l < LD; ++l)
                    raw[k][c][l] = (gval[it] & (1u << c))
                                       ? ldg_nc_v4(xt + (size_t)(unsigned)((gidx[it] + d[c]) * P.CS + cofs) + l * (8 / LD))
                                       : make_uint4(0u, 0u, 0u, 0u);
              }
#pragma unroll
              for (int k = 0; k < BATCH; ++k) {
                const int it = i0 + k;
                if (gval[it] == 0u) continue;
                // S_c = sum_e gcol_e * corner_c[e]; bilinear and its h/w derivatives
                // are linear in the corners, so the three channel sums follow from S
                float S[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  float vv[8];
                  unpack_slice<T>(raw[k][c], vv);
                  float acc = 0.f;
#pragma unroll
                  for (int e = 0; e < 8; ++e) acc = fmaf(gc[k][e], vv[e], acc);
                  S[c] = acc;
                }
                const float lh = glh[it], lw = glw[it], hh = 1.f - lh, hw = 1.f - lw;
                const float bw[4] = {(gval[it] & 1u) ? hh * hw : 0.f, (gval[it] & 2u) ? hh * lw : 0.f,
                                     (gval[it] & 4u) ? lh * hw : 0.f, (gval[it] & 8u) ? lh * lw : 0.f};
                const float am = bw[0] * S[0] + bw[1] * S[1] + bw[2] * S[2] + bw[3] * S[3];
                const float ah = hw * (S[2] - S[0]) + lw * (S[3] - S[1]);
                const float aw = hh * (S[1] - S[0]) + lh * (S[3] - S[2]);
                racc[it][0] += am;
                racc[it][1] += ah;
                racc[it][2] += aw;
                const float m = gm[it];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  if ((gval[it] & (1u << c)) && !(a.dbg & 2)) {
                    const float sk = bw[c] * m;
                    float* dst = a.gx_nhwc + (size_t)(unsigned)((gidx[it] + d[c]) * P.CS + lofs);
                    red_add_v4(dst, gc[k][0] * sk, gc[k][1] * sk, gc[k][2] * sk, gc[k][3] * sk);
                    red_add_v4(dst + 32, gc[k][4] * sk, gc[k][5] * sk, gc[k][6] * sk, gc[k][7] * sk);
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(tre);
          if (ew == 0) DCN_TS(4 * ucnt + 3);
        }
        if (!ok) break;
        if (ew == 0) DCN_TS(400 + 2 * ucnt);
        if (cch == P.nCC - 1) {
          // reduce each pixel's per-lane partials; write grad_offset / grad_mask
#pragma unroll
          for (int it = 0; it < ITER; ++it) {
            float r0 = racc[it][0], r1 = racc[it][1], r2 = racc[it][2];
#pragma unroll
            for (int sh = 1; sh < LPP; sh <<= 1) {
              r0 += __shfl_xor_sync(0xffffffffu, r0, sh);
              r1 += __shfl_xor_sync(0xffffffffu, r1, sh);
              r2 += __shfl_xor_sync(0xffffffffu, r2, sh);
            }
            if (q == 0 && wob[it] >= 0) {
              const int oo = wob[it] + (g * P.K2 + t) * 2 * HoWo;
              goff[oo] = Elem<T>::from_f(r1 * gm[it]);
              goff[oo + HoWo] = Elem<T>::from_f(r2 * gm[it]);
              gmsk[wmb[it] + (g * P.K2 + t) * HoWo] = Elem<T>::from_f(r0);
            }
          }
        }
      }
    }
  } else {
    regs_dec<56>();
    if (warp < kAWarps) {
    // ------------------------------------------------ grad_out chunk loader
    // One thread bulk-copies the two pre-packed 64-pixel blocks of each Co chunk
    // (K-major, 128-byte swizzle; f32: hi and lo) into the A ring.
    if (warp == 0 && lane == 0) {
      uint32_t aseq = 0;
      bool ok = true;
      const int nload = resident ? P.nKo : P.nU * P.nKo;  // chunk loads per tile
      const uint32_t blk = NS * 8192u;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        for (int l = 0; l < nload; ++l, ++aseq) {
          const int ko = l % P.nKo;
          const int r = aseq % RA;
          const uint32_t ph = (aseq / RA) & 1u;
          if (!mbar_wait(aempty0 + 8 * r, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          const uint32_t at = abase + (uint32_t)r * aSlot;
          const int pb0 = tile * 2;
          const int nb = (pb0 + 1 < P.nPB) ? 2 : 1;
          mbar_arrive_expect_tx(afull0 + 8 * r, (uint32_t)nb * blk);
          for (int h = 0; h < nb; ++h) {
            const uint8_t* src = a.gpk + ((size_t)(pb0 + h) * P.nKo + ko) * blk;
            bulk_g2s(at + h * 8192u, src, 8192u, afull0 + 8 * r);
            if constexpr (NS == 2) bulk_g2s(at + kATile + h * 8192u, src + 8192, 8192u, afull0 + 8 * r);
          }
        }
      }
    }
    } else if (warp == kTmaWarp) {
    // ------------------------------------------------ W^T tiles (bulk copy)
    if (lane == 0) {
      uint32_t kidx = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        for (int u = 0; u < P.nU && ok; ++u) {
          for (int ko = 0; ko < P.nKo; ++ko, ++kidx) {
            const int s = kidx % S;
            const uint32_t ph = (kidx / S) & 1u;
            if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
            const uint32_t bt = sbase + s * stageBytes;
            mbar_arrive_expect_tx(full0 + 8 * s, NS * bTile);
            bulk_g2s(bt, a.wpk + (size_t)(u * P.nKo + ko) * P.wd_tile_bytes, NS * bTile,
                     full0 + 8 * s);
          }
        }
      }
    }
    } else {
    // ------------------------------------------------ MMA issuer
    if (warp == kMmaWarp && lane == 0) {
      const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 0, 0, kTileM, NC);
      uint32_t kidx = 0, ucnt = 0, aseq0 = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        for (int u = 0; u < P.nU && ok; ++u, ++ucnt) {
          const int ab = ucnt & 1;
          if (!mbar_wait(acce0 + 8 * ab, ((ucnt >> 1) & 1) ^ 1, a.err, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dt = tmem_base + (uint32_t)(ab * NC);
          for (int ko = 0; ko < P.nKo; ++ko, ++kidx) {
            const uint32_t aseq = aseq0 + (resident ? ko : u * P.nKo + ko);
            const int r = aseq % RA;
            if ((!resident || u == 0) &&
                !mbar_wait(afull0 + 8 * r, (aseq / RA) & 1u, a.err, &abort_flag)) { ok = false; break; }
            const int s = kidx % S;
            const uint32_t ph = (kidx / S) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t at = abase + (uint32_t)r * aSlot;
            const uint32_t bt = sbase + s * stageBytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sw128_desc(at + kk * 32, 16, 1024);
              const uint64_t bd = sw128_desc(bt + kk * 32, 16, 1024);
              if (!(a.dbg & 4)) umma_f16(dt, ad, bd, idesc, (ko | kk) != 0);
              if constexpr (NS == 2) {
                const uint64_t adl = sw128_desc(at + kATile + kk * 32, 16, 1024);
                const uint64_t bdl = sw128_desc(bt + bTile + kk * 32, 16, 1024);
                umma_f16(dt, ad, bdl, idesc, 1);
                umma_f16(dt, adl, bd, idesc, 1);
              }
            }
            umma_commit(empty0 + 8 * s);
            DCN_TS(600 + ucnt);
            if (!resident || u == P.nU - 1) umma_commit(aempty0 + 8 * r);
          }
          if (!ok) break;
          umma_commit(accf0 + 8 * ab);
        }
        aseq0 += resident ? P.nKo : P.nU * P.nKo;
      }
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

int launch_backward_data(const BwdDataArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const size_t bStage = (size_t)P.nsplit * P.NC * 128;     // W^T stage
  const size_t aSlot = (size_t)P.nsplit * 128 * 128;       // grad_out chunk
  const size_t avail = kBwdSmemLimit - 1024;
  // Preference: A double-buffered across tiles (2 x nKo slots), then resident
  // (nKo slots), then streamed (2 slots); transpose buffer of 128 channels, then
  // 64; W^T ring of up to 4 stages, at least 2.
  int CB = 0, S = 0, RA = 0;
  const int cbs[2] = {P.NC < 128 ? P.NC : 128, 64};
  const int ras[3] = {2 * P.nKo, P.nKo, 2};
  for (int ri = 0; ri < 3 && !RA; ++ri) {
    for (int ci = 0; ci < 2 && !RA; ++ci) {
      const int ra = ras[ri] > kMaxASlots ? -1 : ras[ri];
      if (ra < 0) continue;
      const size_t fixed = (size_t)ra * aSlot + (size_t)128 * 4 * cbs[ci];
      if (fixed + 2 * bStage > avail) continue;
      int s = (int)((avail - fixed) / bStage);
      if (s > 4) s = 4;
      RA = ra;
      CB = cbs[ci];
      S = s;
    }
  }
  if (!RA) return DCN_E_UNSUPPORTED;
  const size_t tbytes = (size_t)128 * 4 * CB;
  BwdDataArgs args = a;
  args.stages = S;
  args.tb_ch = CB;
  args.a_slots = RA;
  const size_t smem = 1024 + (size_t)S * bStage + (size_t)RA * aSlot + tbytes;
  int grid = P.nPT < a.num_sms ? P.nPT : a.num_sms;
  if (grid <= 0) return DCN_OK;
  cudaError_t e = cudaSuccess;
  switch (P.dtype) {
    case DCN_F32:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<float>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) dcn_bwd_data_kernel<float><<<grid, kThreads, smem, stream>>>(args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) dcn_bwd_data_kernel<__half><<<grid, kThreads, smem, stream>>>(args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        dcn_bwd_data_kernel<__nv_bfloat16><<<grid, kThreads, smem, stream>>>(args);
      break;
  }
  if (e != cudaSuccess) return DCN_E_CUDA;
  return cudaGetLastError() == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
