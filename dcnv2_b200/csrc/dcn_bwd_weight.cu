// Backward of DCNv2 with respect to weight and bias.  Replaces, per batch, the
// reference's re-im2col (com.cu:637-706) and its cuBLAS products
// grad_weight += grad_out . columns^T and grad_bias += grad_out . 1
// (com.cu:818-835) with one tcgen05 GEMM whose B operand is gathered on the fly:
//
//   gW[co, (t,g,c)] = sum_pixels grad_out[b, co, p] * mask * bilinear(x_c, pos + offset)
//       M = 128 Co rows (per M tile), N = channels of a set of (tap, group, chunk)
//       units, K = pixels (64 per pipeline stage); both co tiles and units are
//       kept in TMEM at once so every gathered column feeds all of them.
//
// The pixel reduction is split over CTAs; each CTA adds its fp32 partial into a
// zeroed fp32 buffer with vector red.add.  grad_bias is summed while grad_output
// is packed (pack_gout_kernel).
//
// CTA roles (416 threads):
//   warps 0-7   column gather producers (B operand, MN-major SW128), coalesced
//               corner-line loads as in the forward
//   warp 8      bulk copies of pre-packed grad_out blocks (A operand, MN-major
//               SW128); warps 8-11 then run the TMEM -> global epilogue
//   warp 12     TMEM owner and tcgen05.mma issuer (warps 13-15 idle)
// setmaxnreg gives the gather warps 168 registers, the grad_out warps 120.
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_gout.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

#define DCN_TS(slot) \
  do { if (a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

constexpr int kThreads = 512;  // 4 warpgroups; warps 13-15 idle
constexpr int kBWarps = 8;
constexpr int kAWarp0 = 8;
constexpr int kAWarps = 4;
constexpr int kMmaWarp = 12;
constexpr int kMaxMT = 4;

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    dcn_bwd_weight_kernel(const __grid_constant__ BwdWeightArgs a) {
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;
  const Plan& P = a.plan;
  const int NC = P.NC;
  const int mpc = P.wg_mt_per_cta, ups = P.wg_units_per_set;
  const uint32_t aBytes = (uint32_t)mpc * kATile;            // one (hi or lo) A block
  const uint32_t bBytes = (uint32_t)ups * NC * 128u;         // one (hi or lo) B block
  const uint32_t stageBytes = NS * (aBytes + bBytes);
  const int S = a.stages;

  // work item
  const int split = blockIdx.x % P.wg_nsplit_px;
  const int rest = blockIdx.x / P.wg_nsplit_px;
  const int set = rest % P.wg_nsets;
  const int cg = rest / P.wg_nsets;
  const int per = (P.wg_ksteps + P.wg_nsplit_px - 1) / P.wg_nsplit_px;
  const int ks0 = split * per;
  const int ks1 = min(P.wg_ksteps, ks0 + per);
  const int mt0 = cg * mpc;
  const int mcount = min(mpc, P.nMT - mt0);
  const int u0 = set * ups;
  const int ucount = min(ups, P.nU - u0);
  if (ks1 <= ks0 || mcount <= 0 || ucount <= 0) return;  // uniform for the CTA
  const int ntot = ucount * NC;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 2];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 1]);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, kBWarps + 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accf, 1);
    mbar_init(drain, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(mpc * ups * NC)) tmem_cols <<= 1;
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&tmem_slot), tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  const int HoWo = P.HoWo;
  if (warp == 0) DCN_TS(1000);

  // register split per warpgroup (one setmaxnreg per warpgroup)
  if ((warp >> 2) < 2) {
    regs_inc<168>();
  } else if ((warp >> 2) == 2) {
    regs_dec<120>();
  } else {
    regs_dec<56>();
  }

  if (warp < kBWarps) {
    // ------------------------------------------------ column gather (B operand)
    // Warp w owns pixel rows w*8 .. w*8+7 of every K step.  Lane L computes the
    // sampling geometry of (unit L/8, row L%8) (and L+32 when there are more than
    // four units), with the offsets prefetched one K step ahead; the gather runs
    // 4 rows at a time with 8 lanes per row and packed blends.
    using GS = GatherShape<T>;
    constexpr int LPP = GS::kLPP, CPL = GS::kCPL, PPI = GS::kPPI;
    constexpr int BATCH = sizeof(T) == 4 ? 2 : 4;
    const int lp = lane / LPP, q = lane % LPP;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    const int HW = P.H * P.W;
    const int nblk = NC / kChunk;
    const int ngeo = ucount * 8;                 // geometries per warp and K step
    const int niter = ucount * nblk * 2;         // 4-row gather iterations per K step
    uint32_t rh[2] = {0, 0}, rw[2] = {0, 0}, rm[2] = {0, 0};  // raw prefetched bits
    auto fetch_raw = [&](int ks) {
#pragma unroll
      for (int sl = 0; sl < 2; ++sl) {
        const int item = lane + 32 * sl;
        if (item < ngeo) {
          const int pix = ks * 64 + warp * 8 + (item & 7);
          if (pix < P.totalP) {
            const int u = u0 + (item >> 3);
            const int tg = u / P.nCC, t = tg / P.dg, g = tg - t * P.dg;
            const int b = (int)(pix / HoWo), p = (int)(pix - b * HoWo);
            const int ob = ((b * P.dg + g) * 2 * P.K2 + 2 * t) * HoWo + p;
            rh[sl] = ldg_raw<T>(off + (ob));
            rw[sl] = ldg_raw<T>(off + (ob + HoWo));
            rm[sl] = ldg_raw<T>(msk + (((b * P.dg + g) * P.K2 + t) * HoWo + p));
          }
        }
      }
    };
    fetch_raw(ks0);
    for (int ks = ks0; ks < ks1; ++ks) {
      const uint32_t kidx = ks - ks0;
      const int s = kidx % S;
      const uint32_t ph = (kidx / S) & 1u;
      PixGeo mine[2];
#pragma unroll
      for (int sl = 0; sl < 2; ++sl) {
        mine[sl] = zero_pixgeo();
        const int item = lane + 32 * sl;
        const int pix = ks * 64 + warp * 8 + (item & 7);
        if (item < ngeo && pix < P.totalP && !(a.dbg & 1)) {
          const int u = u0 + (item >> 3);
          const int tg = u / P.nCC, t = tg / P.dg;
          const int i = t / P.kw, jj = t - i * P.kw;
          const int b = (int)(pix / HoWo), p = (int)(pix - b * HoWo);
          const int ho = p / P.Wo, wo = p - ho * P.Wo;
          const float hs = (float)(ho * P.sh - P.ph + i * P.dh) + raw_to_f<T>(rh[sl]);
          const float ws = (float)(wo * P.sw - P.pw + jj * P.dw) + raw_to_f<T>(rw[sl]);
          mine[sl] = make_pixgeo(b * HW, hs, ws, raw_to_f<T>(rm[sl]), P.H, P.W);
        }
      }
      if (ks + 1 < ks1) fetch_raw(ks + 1);
      if (warp == 0) DCN_TS(4 * kidx);
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) break;
      if (warp == 0) DCN_TS(4 * kidx + 1);
      const uint32_t bt = sbase + s * stageBytes + NS * aBytes;
      for (int i0 = 0; i0 < niter; i0 += BATCH) {
        uint4 v[BATCH][4][GS::kLD];
        PixGeo gg[BATCH];
        int row[BATCH], atom[BATCH];
#pragma unroll
        for (int k = 0; k < BATCH; ++k) {
          const int itr = i0 + k;
          row[k] = -1;
          atom[k] = 0;
          gg[k] = zero_pixgeo();
          if (itr < niter) {                     // warp-uniform
            const int half = itr & 1, r2 = itr >> 1;
            const int blk = r2 % nblk, j = r2 / nblk;
            const int item = j * 8 + half * 4 + lp;
            const PixGeo src = (item >> 5) ? mine[1] : mine[0];  // slot is warp-uniform
            gg[k] = shfl_pixgeo(src, item & 31);
            const int u = u0 + j;
            const int tg = u / P.nCC, cch = u - tg * P.nCC;
            const int g = tg % P.dg;
            const int cc = cch * NC + blk * kChunk;
            if (cc >= P.Cgp) gg[k] = zero_pixgeo();
            row[k] = warp * 8 + half * 4 + lp;
            atom[k] = j * nblk + blk;
            load_corners_px<T>(xt, gg[k], P.W, P.CS, g * P.Cgp + cc + q * CPL, v[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < BATCH; ++k)
          if (row[k] >= 0) blend_store<T>(v[k], gg[k], bt + (uint32_t)atom[k] * 8192u, bBytes, row[k], q);
      }
      if (warp == 0) DCN_TS(4 * kidx + 2);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + 8 * s);
    }
  } else if (warp < kAWarp0 + kAWarps) {
    // ------------------------------------------------ grad_out tiles (A operand)
    // One thread bulk-copies, per K step and M tile, the two pre-packed blocks
    // (64 pixels x 64 Co each) that form the MN-major SW128 A tile.
    bool ok = true;
    if (warp == kAWarp0 && lane == 0) {
      const uint32_t blk = NS * 8192u;
      for (int ks = ks0; ks < ks1; ++ks) {
        const uint32_t kidx = ks - ks0;
        const int s = kidx % S;
        const uint32_t ph = (kidx / S) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
        DCN_TS(256 + 2 * kidx);
        const uint32_t at = sbase + s * stageBytes;
        uint32_t bytes = 0;
        for (int m = 0; m < mcount; ++m)
          for (int h = 0; h < 2; ++h)
            if (2 * (mt0 + m) + h < P.nKo) bytes += blk;
        mbar_arrive_expect_tx(full0 + 8 * s, bytes);
        for (int m = 0; m < mcount; ++m) {
          for (int h = 0; h < 2; ++h) {
            const int ko = 2 * (mt0 + m) + h;
            if (ko >= P.nKo) continue;
            const uint8_t* src = a.gpk + ((size_t)ks * P.nKo + ko) * blk;
            bulk_g2s(at + m * kATile + h * 8192u, src, 8192u, full0 + 8 * s);
            if constexpr (NS == 2)
              bulk_g2s(at + aBytes + m * kATile + h * 8192u, src + 8192, 8192u, full0 + 8 * s);
          }
        }
      }
    }
    __syncwarp();
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    // ------------------------------------------------ epilogue: TMEM -> fp32 red.add
    if (ok && mbar_wait(accf, 0, a.err, &abort_flag)) {
      if (warp == kAWarp0) DCN_TS(1001);
      tc_fence_after();
      const int q = warp & 3;
      for (int m = 0; m < mcount; ++m) {
        const int co = (mt0 + m) * 128 + q * 32 + lane;
        for (int j = 0; j < ucount; ++j) {
          const int u = u0 + j;
          const int tg = u / P.nCC, cch = u - tg * P.nCC;
          int cend = P.Cgp - cch * NC;
          if (cend > NC) cend = NC;
          const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((m * ups + j) * NC);
          float* dst = a.gw + ((size_t)co * P.K2 * P.dg + tg) * P.Cgp + cch * NC;
          for (int c0 = 0; c0 < cend; c0 += 8) {
            float v[8];
            tmem_ld8(tb + c0, v);
            if (co < P.Co) {
              // packed columns c0..c0+7 are logical channels blk+4q' .. and blk+32+4q' ..
              const int lc = (c0 & ~63) + 4 * ((c0 & 63) >> 3);
              red_add_v4(dst + lc, v[0], v[1], v[2], v[3]);
              red_add_v4(dst + lc + 32, v[4], v[5], v[6], v[7]);
            }
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ MMA issuer
    if (warp == kMmaWarp && lane == 0) {
      bool ok = true;
      for (int ks = ks0; ks < ks1; ++ks) {
        const uint32_t kidx = ks - ks0;
        const int s = kidx % S;
        const uint32_t ph = (kidx / S) & 1u;
        if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
        DCN_TS(512 + 2 * kidx);
        tc_fence_after();
        const uint32_t at = sbase + s * stageBytes;
        const uint32_t bt = at + NS * aBytes;
        for (int m = 0; m < mcount; ++m) {
          for (int n0 = 0; n0 < ntot; n0 += 256) {
            const int N = min(256, ntot - n0);
            const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 1, 1, kTileM, N);
            const uint32_t dt = tmem_base + (uint32_t)(m * ups * NC + n0);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sw128_desc(at + m * kATile + kk * 2048, 8192, 1024);
              const uint64_t bd = sw128_desc(bt + (uint32_t)(n0 >> 6) * 8192u + kk * 2048, 8192, 1024);
              if (!(a.dbg & 4)) umma_f16(dt, ad, bd, idesc, (ks > ks0 || kk > 0) ? 1u : 0u);
              if constexpr (NS == 2) {
                const uint64_t adl = sw128_desc(at + aBytes + m * kATile + kk * 2048, 8192, 1024);
                const uint64_t bdl =
                    sw128_desc(bt + bBytes + (uint32_t)(n0 >> 6) * 8192u + kk * 2048, 8192, 1024);
                umma_f16(dt, ad, bdl, idesc, 1);
                umma_f16(dt, adl, bd, idesc, 1);
              }
            }
          }
        }
        umma_commit(empty0 + 8 * s);
        DCN_TS(513 + 2 * kidx);
      }
      if (ok) umma_commit(accf);
      umma_commit(drain);
      mbar_wait_drain(drain, 0, a.err);
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

int launch_backward_weight(const BwdWeightArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  if (P.wg_mt_per_cta > kMaxMT || P.wg_units_per_set > 8) return DCN_E_UNSUPPORTED;
  const size_t stageBytes =
      (size_t)P.nsplit * ((size_t)P.wg_mt_per_cta * 128 * 128 +
                          (size_t)P.wg_units_per_set * P.NC * 128);
  int S = (int)((kBwdSmemBudget - 1024) / stageBytes);
  if (S > kMaxStages) S = kMaxStages;
  if (S < 2) return DCN_E_UNSUPPORTED;
  BwdWeightArgs args = a;
  args.stages = S;
  const size_t smem = 1024 + (size_t)S * stageBytes;
  const int grid = P.wg_ncg * P.wg_nsets * P.wg_nsplit_px;
  if (grid <= 0) return DCN_OK;
  cudaError_t e = cudaSuccess;
  switch (P.dtype) {
    case DCN_F32:
      e = cudaFuncSetAttribute(dcn_bwd_weight_kernel<float>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) dcn_bwd_weight_kernel<float><<<grid, kThreads, smem, stream>>>(args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_bwd_weight_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) dcn_bwd_weight_kernel<__half><<<grid, kThreads, smem, stream>>>(args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_bwd_weight_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        dcn_bwd_weight_kernel<__nv_bfloat16><<<grid, kThreads, smem, stream>>>(args);
      break;
  }
  if (e != cudaSuccess) return DCN_E_CUDA;
  return cudaGetLastError() == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
