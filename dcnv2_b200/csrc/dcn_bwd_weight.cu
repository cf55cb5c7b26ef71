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
// zeroed fp32 buffer with vector red.add, and grad_bias is summed by the
// grad_out loaders of the unit-set-0 CTAs.
//
// CTA roles (416 threads):
//   warps 0-7   column gather producers (B operand, MN-major SW128), coalesced
//               corner-line loads as in the forward
//   warps 8-11  grad_out tile producers (A operand, K-major SW128) + bias sums,
//               then the TMEM -> global epilogue
//   warp 12     TMEM owner and tcgen05.mma issuer
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_gout.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kThreads = 416;
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
      mbar_init(full0 + 8 * s, kBWarps + kAWarps);
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

  if (warp < kBWarps) {
    // ------------------------------------------------ column gather (B operand)
    // Work items: (unit j, 64-channel block, group of 4 pixels), 8 lanes per
    // pixel (whole corner lines per warp-wide load); BATCH items in flight.
    using GS = GatherShape<T>;
    constexpr int LPP = GS::kLPP, CPL = GS::kCPL, PPI = GS::kPPI;
    constexpr int BATCH = sizeof(T) == 4 ? 2 : 4;
    const int lp = lane / LPP, q = lane % LPP;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    const size_t img = (size_t)P.H * P.W * P.CS;
    const int nblk = NC / kChunk;
    const int npg = 64 / PPI;
    const int items = ucount * nblk * npg;
    for (int ks = ks0; ks < ks1; ++ks) {
      const uint32_t kidx = ks - ks0;
      const int s = kidx % S;
      const uint32_t ph = (kidx / S) & 1u;
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) break;
      const uint32_t bt = sbase + s * stageBytes + NS * aBytes;
      for (int it0 = warp; it0 < items; it0 += kBWarps * BATCH) {
        Geo geo[BATCH];
        int xo[BATCH], row[BATCH], atom[BATCH];
        size_t xb[BATCH];
#pragma unroll
        for (int k = 0; k < BATCH; ++k) {
          const int it = it0 + k * kBWarps;
          geo[k] = zero_geo();
          xb[k] = 0;
          xo[k] = 0;
          row[k] = -1;
          atom[k] = 0;
          if (it < items) {
            const int pg = it % npg;
            const int r2 = it / npg;
            const int blk = r2 % nblk, j = r2 / nblk;
            const int u = u0 + j;
            const int tg = u / P.nCC, cch = u - tg * P.nCC;
            const int t = tg / P.dg, g = tg - t * P.dg;
            const int cc = cch * NC + blk * kChunk;
            const int px = pg * PPI + lp;
            row[k] = px;
            atom[k] = j * nblk + blk;
            const long long pix = (long long)ks * 64 + px;
            if (pix < P.totalP && cc < P.Cgp) {
              const int b = (int)(pix / HoWo);
              const int p = (int)(pix - (long long)b * HoWo);
              const int ho = p / P.Wo, wo = p - ho * P.Wo;
              const int i = t / P.kw, jj = t - i * P.kw;
              const size_t ob = ((size_t)b * P.dg + g) * 2 * P.K2;
              const float hs = (float)(ho * P.sh - P.ph + i * P.dh) + ldf(off + (ob + 2 * t) * HoWo + p);
              const float ws = (float)(wo * P.sw - P.pw + jj * P.dw) + ldf(off + (ob + 2 * t + 1) * HoWo + p);
              const float m = ldf(msk + (((size_t)b * P.dg + g) * P.K2 + t) * HoWo + p);
              geo[k] = make_geo(hs, ws, m, P.H, P.W);
              if (a.dbg & 1) geo[k] = zero_geo();
              xb[k] = (size_t)b * img;
              xo[k] = g * P.Cgp + cc + q * CPL;
            }
          }
        }
        uint4 v[BATCH][4][GS::kLD];
#pragma unroll
        for (int k = 0; k < BATCH; ++k) load_corners<T>(xt + xb[k] + xo[k], geo[k], P.W, P.CS, v[k]);
#pragma unroll
        for (int k = 0; k < BATCH; ++k) {
          if (row[k] >= 0) {
            float sl[8];
            blend_corners<T>(v[k], geo[k], sl);
            store_slice<T>(bt + (uint32_t)atom[k] * 8192u, bBytes, row[k], q, sl);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + 8 * s);
    }
  } else if (warp < kAWarp0 + kAWarps) {
    // ------------------------------------------------ grad_out tiles (A operand) + bias
    const int i = tid - kAWarp0 * 32;  // 0..127
    const T* __restrict__ gout = reinterpret_cast<const T*>(a.gout);
    const bool vec = a.vec_gout && (HoWo % 8 == 0);
    const bool do_bias = (a.gb != nullptr) && set == 0;
    float bsum[kMaxMT][8];
#pragma unroll
    for (int m = 0; m < kMaxMT; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) bsum[m][j] = 0.f;
    bool ok = true;
    for (int ks = ks0; ks < ks1; ++ks) {
      const uint32_t kidx = ks - ks0;
      const int s = kidx % S;
      const uint32_t ph = (kidx / S) & 1u;
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
      const uint32_t at = sbase + s * stageBytes;
#pragma unroll
      for (int m = 0; m < kMaxMT; ++m) {
        if (m < mcount) {
          const int c = i & 7;
          if (vec) {
            // all 8 chunks of this thread in flight before any is consumed
            GoutRaw<T> raw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              gout_raw_load<T>(gout, P, (long long)ks * 64 + c * 8, (mt0 + m) * 128 + (i >> 3) + 16 * j, raw[j]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float v[8];
              gout_raw_to_f<T>(raw[j], v);
              if (do_bias) bsum[m][j] += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
              store8_op<T>(at + m * kATile + sw128_off((i >> 3) + 16 * j, c), aBytes, v);
            }
          } else {
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {
              const int r = (i >> 3) + 16 * j;
              float v[8];
              load8_gout<T>(gout, P, (long long)ks * 64 + c * 8, (mt0 + m) * 128 + r, false, v);
              if (do_bias) bsum[m][j] += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
              store8_op<T>(at + m * kATile + sw128_off(r, c), aBytes, v);
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(full0 + 8 * s);
    }
    if (do_bias && ok) {
#pragma unroll
      for (int m = 0; m < kMaxMT; ++m) {
        if (m < mcount) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float v = bsum[m][j];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            const int co = (mt0 + m) * 128 + (i >> 3) + 16 * j;
            if ((i & 7) == 0 && co < P.Co) atomicAdd(a.gb + co, v);
          }
        }
      }
    }
    // ------------------------------------------------ epilogue: TMEM -> fp32 red.add
    if (ok && mbar_wait(accf, 0, a.err, &abort_flag)) {
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
              red_add_v4(dst + c0, v[0], v[1], v[2], v[3]);
              red_add_v4(dst + c0 + 4, v[4], v[5], v[6], v[7]);
            }
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int ks = ks0; ks < ks1; ++ks) {
        const uint32_t kidx = ks - ks0;
        const int s = kidx % S;
        const uint32_t ph = (kidx / S) & 1u;
        if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t at = sbase + s * stageBytes;
        const uint32_t bt = at + NS * aBytes;
        for (int m = 0; m < mcount; ++m) {
          for (int n0 = 0; n0 < ntot; n0 += 256) {
            const int N = min(256, ntot - n0);
            const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 0, 1, kTileM, N);
            const uint32_t dt = tmem_base + (uint32_t)(m * ups * NC + n0);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sw128_desc(at + m * kATile + kk * 32, 16, 1024);
              const uint64_t bd = sw128_desc(bt + (uint32_t)(n0 >> 6) * 8192u + kk * 2048, 8192, 1024);
              if (!(a.dbg & 4)) umma_f16(dt, ad, bd, idesc, (ks > ks0 || kk > 0) ? 1u : 0u);
              if constexpr (NS == 2) {
                const uint64_t adl = sw128_desc(at + aBytes + m * kATile + kk * 32, 16, 1024);
                const uint64_t bdl =
                    sw128_desc(bt + bBytes + (uint32_t)(n0 >> 6) * 8192u + kk * 2048, 8192, 1024);
                umma_f16(dt, ad, bdl, idesc, 1);
                umma_f16(dt, adl, bd, idesc, 1);
              }
            }
          }
        }
        umma_commit(empty0 + 8 * s);
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
  if (P.wg_mt_per_cta > kMaxMT) return DCN_E_UNSUPPORTED;
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
