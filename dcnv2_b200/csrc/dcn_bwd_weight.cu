// Backward of DCNv2 with respect to weight.  Replaces, per batch, the
// reference's re-im2col (com.cu:637-706) and its cuBLAS product
// grad_weight += grad_out . columns^T (com.cu:818-822) with one tcgen05 GEMM
// over the whole pixel chunk:
//
//   gW[co, (t,g,c)] = sum_pixels grad_out[b, co, p] * column[p, (t,g,c)]
//       M = 128 Co rows (per M tile), N = channels of a set of (tap, group, chunk)
//       units, K = pixels (64 per pipeline stage); all of a CTA's Co tiles and
//       units are kept in TMEM at once.
//
// The B operand (sampled columns) arrives as MN-major SW128 blocks of 64 pixels
// written by the backward scatter kernel, which already holds every bilinear
// corner.  The A operand is read from grad_output itself by TMA for 16-bit
// types (64 pixels x 64 Co boxes, K-major) or arrives as MN-major blocks
// pre-packed by pack_gout_kernel (f32 as bf16 hi/lo, and shapes whose 64-pixel
// blocks straddle images).  The
// kernel is therefore a plain streaming GEMM: one thread bulk-copies both
// operands into a ring of stages, one thread issues the MMAs, and at the end
// four warps add the fp32 partial sums into a zeroed fp32 buffer with vector
// red.add (the pixel reduction is split over CTAs).  grad_bias is summed by the
// epilogue warps from the A tiles while the GEMM runs (direct reads), else while
// grad_output is packed.
//
// CTA roles (192 threads):
//   warps 0-3   epilogue: TMEM -> fp32 red.add into gW (warp w reads TMEM lanes 32w..32w+31)
//   warp 4      bulk copies of the A (grad_out) and B (column) blocks
//   warp 5      TMEM owner and tcgen05.mma issuer
#include "dcn_common.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

#define DCN_TS(slot) \
  do { if (DCN_STUDY_ON && a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

constexpr int kThreads = 192;
constexpr int kLoadWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kMaxMT = 4;

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    dcn_bwd_weight_kernel(const __grid_constant__ BwdWeightArgs a) {
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;
  const Plan& P = a.plan;
  const int NC = P.NC;
  const int nblk = NC / kChunk;
  const int natoms = P.nU * nblk;
  const int mpc = P.wg_mt_per_cta, ups = P.wg_units_per_set;
  const uint32_t aBytes = (uint32_t)mpc * kATile;            // one (hi or lo) A block
  const uint32_t bBytes = (uint32_t)ups * NC * 128u;         // one (hi or lo) B block
  const uint32_t stageBytes = NS * (aBytes + bBytes);
  const int S = a.stages;

  // work item: (Co group, unit set, pixel split) over the chunk's 64-pixel blocks
  const int split = blockIdx.x % P.wg_nsplit_px;
  const int rest = blockIdx.x / P.wg_nsplit_px;
  const int set = rest % P.wg_nsets;
  const int cg = rest / P.wg_nsets;
  const int per = (a.nks + P.wg_nsplit_px - 1) / P.wg_nsplit_px;
  const int kl0 = split * per;
  const int kl1 = min(a.nks, kl0 + per);
  const int mt0 = cg * mpc;
  const int mcount = min(mpc, P.nMT - mt0);
  const int u0 = set * ups;
  const int ucount = min(ups, P.nU - u0);
  if (kl1 <= kl0 || mcount <= 0 || ucount <= 0) return;  // uniform for the CTA
  const int ntot = ucount * NC;
  // grad_output read directly (16-bit): A tiles are K-major (pixels contiguous
  // per Co row), and the CTAs of unit set 0 also sum grad_bias from them
  const bool gdirect = NS == 1 && a.gdirect == kGoutNchw;
  const bool gnhwc = NS == 1 && a.gdirect == kGoutNhwc;
  const bool bias = (gdirect || gnhwc) && a.gb != nullptr && set == 0;

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
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, bias ? 1 + 4 : 1);  // MMA commit (+ the 4 bias-summing warps)
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
  pdl_wait();
  if (warp == 0) DCN_TS(1000);

  if (warp == kLoadWarp) {
    // ------------------------------------------------ operand loads (one thread)
    // Per K step and M tile, the two pre-packed grad_out blocks (64 pixels x 64
    // Co each) form the A tile; the unit set's column blocks are contiguous in
    // the chunk's column buffer and form the B tile in one copy (per hi/lo).
    if (lane == 0) {
      const uint32_t blk = NS * 8192u;
      const int nPBi = P.HoWo / 64;               // 64-pixel blocks per image (gdirect)
      int ls = 0;                                   // ring stage and its phase
      uint32_t lph = 0;
      for (int kl = kl0; kl < kl1; ++kl) {
        const uint32_t kidx = kl - kl0;
        const int s = ls;
        const uint32_t ph = lph;
        if (++ls == S) { ls = 0; lph ^= 1u; }
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) break;
        DCN_TS(256 + 2 * kidx);
        const uint32_t at = sbase + s * stageBytes;
        const uint32_t bt = at + NS * aBytes;
        const uint32_t bcopy = (uint32_t)ucount * nblk * 8192u;
        uint32_t bytes = NS * bcopy;
        for (int m = 0; m < mcount; ++m)
          for (int h = 0; h < 2; ++h)
            if (2 * (mt0 + m) + h < P.nKo) bytes += blk;
        mbar_arrive_expect_tx(full0 + 8 * s, bytes);
        const int ks = a.ks0 + kl;
        const int kb = gdirect ? ks / nPBi : 0;
        for (int m = 0; m < mcount; ++m) {
          for (int h = 0; h < 2; ++h) {
            const int ko = 2 * (mt0 + m) + h;
            if (ko >= P.nKo) continue;
            if (gdirect) {
              // Co rows ko*64 .. +63 of 64-pixel block ks (Co past the end reads zeros)
              tma_load_3d(at + m * kATile + h * 8192u, &a.gmap, (ks - kb * nPBi) * 64, ko * 64, kb,
                          full0 + 8 * s);
              continue;
            }
            if (gnhwc) {
              // channels-last: the packed block's layout straight from grad_output
              tma_load_3d(at + m * kATile + h * 8192u, &a.gmap, ko * 64, ks * 64, 0, full0 + 8 * s);
              continue;
            }
            const uint8_t* src = a.gpk + ((size_t)ks * P.nKo + ko) * blk;
            bulk_g2s(at + m * kATile + h * 8192u, src, 8192u, full0 + 8 * s);
            if constexpr (NS == 2)
              bulk_g2s(at + aBytes + m * kATile + h * 8192u, src + 8192, 8192u, full0 + 8 * s);
          }
        }
        const uint8_t* csrc = a.cols + ((size_t)kl * NS * natoms + (size_t)u0 * nblk) * 8192u;
        bulk_g2s(bt, csrc, bcopy, full0 + 8 * s);
        if constexpr (NS == 2) bulk_g2s(bt + bBytes, csrc + (size_t)natoms * 8192u, bcopy, full0 + 8 * s);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      int ms = 0;                                   // ring stage and its phase
      uint32_t mph = 0;
      for (int kl = kl0; kl < kl1; ++kl) {
        const uint32_t kidx = kl - kl0;
        const int s = ms;
        const uint32_t ph = mph;
        if (++ms == S) { ms = 0; mph ^= 1u; }
        if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
        DCN_TS(512 + 2 * kidx);
        tc_fence_after();
        const uint32_t at = sbase + s * stageBytes;
        const uint32_t bt = at + NS * aBytes;
        for (int m = 0; m < mcount; ++m) {
          for (int n0 = 0; n0 < ntot; n0 += 256) {
            const int N = min(256, ntot - n0);
            const uint32_t idesc = make_idesc(OpOf<T>::kBF16, gdirect ? 0 : 1, 1, kTileM, N);
            const uint32_t dt = tmem_base + (uint32_t)(m * ups * NC + n0);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = gdirect ? sw128_desc(at + m * kATile + kk * 32, 16, 1024)
                                          : sw128_desc(at + m * kATile + kk * 2048, 8192, 1024);
              const uint64_t bd = sw128_desc(bt + (uint32_t)(n0 >> 6) * 8192u + kk * 2048, 8192, 1024);
              if (!DCN_SKIP(4)) umma_f16(dt, ad, bd, idesc, (kl > kl0 || kk > 0) ? 1u : 0u);
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
  } else {
    if (bias) {
      // ---------------------------------------------- grad_bias from the A tiles
      // Thread tid owns Co row tid of every M tile: per stage it adds the 64
      // pixels of its 128-byte row (chunk order is irrelevant to the sum; lane
      // i starts at chunk i % 8 so that eight rows hit eight bank groups).
      // Channels-last tiles hold 64 pixel rows of 64 Co per half: thread tid
      // sums the Co pair 2 * (tid & 31) of half (tid >> 5) & 1 over rows
      // 32 * (tid >> 6) .. +31 (a warp reads one 128-byte row per load).
      float bsum[kMaxMT], bsum1[kMaxMT];
#pragma unroll
      for (int m = 0; m < kMaxMT; ++m) bsum[m] = bsum1[m] = 0.f;
      const int nh = (tid >> 5) & 1, np = tid & 31, nr0 = 32 * (tid >> 6);
      const uint32_t ncol = (uint32_t)((2 * np) & 7) * 2u;
      const int nchunk = (2 * np) >> 3;
      int bs = 0;
      uint32_t bph = 0;
      bool ok = true;
      for (int kl = kl0; kl < kl1; ++kl) {
        const int s = bs;
        const uint32_t ph = bph;
        if (++bs == S) { bs = 0; bph ^= 1u; }
        if (!mbar_wait_warp(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
        const uint32_t at = sbase + s * stageBytes;
        if (gnhwc) {
#pragma unroll
          for (int m = 0; m < kMaxMT; ++m) {
            if (m < mcount) {
              const uint32_t hb = at + m * kATile + (uint32_t)nh * 8192u + ncol;
              float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr) {
                const int r = nr0 + rr;
                const uint32_t w = lds_u32(hb + (uint32_t)r * 128u + (uint32_t)((nchunk ^ (r & 7)) << 4));
                a0 += raw_to_f<T>(w & 0xffffu);
                a1 += raw_to_f<T>(w >> 16);
              }
              bsum[m] += a0;
              bsum1[m] += a1;
            }
          }
        } else {
#pragma unroll
        for (int m = 0; m < kMaxMT; ++m) {
          if (m < mcount) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 w = lds_v4(at + m * kATile + tid * 128u + (uint32_t)(((j + tid) & 7) << 4));
              acc += sum8<T>(w);
            }
            bsum[m] += acc;
          }
        }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
      }
      if (ok) {
        for (int m = 0; m < mcount; ++m) {
          if (gnhwc) {
            const int co = (mt0 + m) * 128 + nh * 64 + 2 * np;
            if (co < P.Co) atomicAdd(a.gb + co, bsum[m]);
            if (co + 1 < P.Co) atomicAdd(a.gb + co + 1, bsum1[m]);
          } else {
            const int co = (mt0 + m) * 128 + tid;
            if (co < P.Co) atomicAdd(a.gb + co, bsum[m]);
          }
        }
      }
    }
    // ------------------------------------------------ epilogue: TMEM -> fp32 red.add
    if (mbar_wait_warp(accf, 0, a.err, &abort_flag)) {
      if (warp == 0) DCN_TS(1001);
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
              const int blk = c0 & ~63, qs = (c0 & 63) >> 3;
              red_add_v4(dst + blk + slice_lo(qs), v[0], v[1], v[2], v[3]);
              red_add_v4(dst + blk + slice_hi(qs), v[4], v[5], v[6], v[7]);
            }
          }
        }
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

int launch_backward_weight(const BwdWeightArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  if (P.wg_mt_per_cta > kMaxMT || P.wg_units_per_set > 8) return DCN_E_UNSUPPORTED;
  const size_t stageBytes =
      (size_t)P.nsplit * ((size_t)P.wg_mt_per_cta * 128 * 128 +
                          (size_t)P.wg_units_per_set * P.NC * 128);
  // as many stages as the shared memory holds (the work split needs two)
  int S = (int)((kBwdSmemLimit - 1024) / stageBytes);
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
      if (e == cudaSuccess) e = launch_k(dcn_bwd_weight_kernel<float>, dim3(grid), dim3(kThreads), smem, stream, args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_bwd_weight_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch_k(dcn_bwd_weight_kernel<__half>, dim3(grid), dim3(kThreads), smem, stream, args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_bwd_weight_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        e = launch_k(dcn_bwd_weight_kernel<__nv_bfloat16>, dim3(grid), dim3(kThreads), smem, stream, args);
      break;
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
