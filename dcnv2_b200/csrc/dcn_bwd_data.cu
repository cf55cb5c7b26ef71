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
//   warps 0-3   A producers: grad_out tile (128 pixels x 64 Co) -> smem, MN-major SW128
//   warps 4-11  epilogue: two threads per pixel row (channel halves) read gcol from
//               TMEM, gather the 4 bilinear corners, reduce and scatter
//   warp 12     bulk-copy producer of the pre-packed W^T tile (K-major SW128)
//   warp 13     TMEM owner and tcgen05.mma issuer
// The accumulator is double-buffered in TMEM (unit u in buffer u & 1) so the
// heavy epilogue of one (tap, group) overlaps the GEMM of the next.
#include "dcn_common.cuh"
#include "dcn_gout.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kThreads = 448;
constexpr int kAWarps = 4;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kTmaWarp = 12;
constexpr int kMmaWarp = 13;

template <typename T>
__device__ __forceinline__ void load_corner8(const T* __restrict__ src, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const uint4 a = ldg_nc_v4(src), c = ldg_nc_v4(src + 4);
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
    v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
    v[4] = __uint_as_float(c.x); v[5] = __uint_as_float(c.y);
    v[6] = __uint_as_float(c.z); v[7] = __uint_as_float(c.w);
  } else {
    unpack8<T>(ldg_nc_v4(src), v);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    dcn_bwd_data_kernel(const __grid_constant__ BwdDataArgs a) {
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;
  const Plan& P = a.plan;
  const int NC = P.NC;
  const uint32_t bTile = (uint32_t)NC * 128u;
  const uint32_t stageBytes = NS * (kATile + bTile);
  const int S = a.stages;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 9];
  __shared__ float red[2][128][3];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 2]);
  const uint32_t redf0 = smem_u32(&bars[2 * kMaxStages + 4]);  // partials written
  const uint32_t rede0 = smem_u32(&bars[2 * kMaxStages + 6]);  // partials consumed
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 8]);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, kAWarps + 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, kEpiWarps);
      mbar_init(redf0 + 8 * i, kEpiWarps / 2);
      mbar_init(rede0 + 8 * i, kEpiWarps / 2);
    }
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
  const int HoWo = P.HoWo;
  const bool vec = a.vec_gout && (HoWo % 8 == 0);

  if (warp < kAWarps) {
    // ------------------------------------------------ grad_out tile producer
    const T* __restrict__ gout = reinterpret_cast<const T*>(a.gout);
    uint32_t kidx = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      for (int u = 0; u < P.nU && ok; ++u) {
        for (int ko = 0; ko < P.nKo; ++ko, ++kidx) {
          const int s = kidx % S;
          const uint32_t ph = (kidx / S) & 1u;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          const uint32_t at = sbase + s * stageBytes;
#pragma unroll 2
          for (int j = 0; j < 8; ++j) {
            const int idx = tid + 128 * j;
            const int pg = idx & 15, k = idx >> 4;
            float v[8];
            load8_gout<T>(gout, P, (long long)tile * kTileM + pg * 8, ko * kChunk + k, vec, v);
            // MN-major: row = co (K), 64-pixel atoms 8192 B apart
            const uint32_t off = (uint32_t)(pg >> 3) * 8192u + sw128_off(k, pg & 7);
            store8_op<T>(at + off, kATile, v);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(full0 + 8 * s);
        }
      }
    }
  } else if (warp < kTmaWarp) {
    // ------------------------------------------------ epilogue
    const int ew = warp - kEpiWarp0;
    const int q = warp & 3;           // TMEM lane quarter
    const int chalf = ew >> 2;        // channel half
    const int row = q * 32 + lane;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    T* __restrict__ goff = reinterpret_cast<T*>(a.goffset);
    T* __restrict__ gmsk = reinterpret_cast<T*>(a.gmask);
    uint32_t ucnt = 0, tgcnt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      const long long pix = (long long)tile * kTileM + row;
      const bool pv = pix < P.totalP;
      const int b = pv ? (int)(pix / HoWo) : 0;
      const int p = pv ? (int)(pix - (long long)b * HoWo) : 0;
      const int ho = p / P.Wo, wo = p - ho * P.Wo;
      const size_t xbase = (size_t)b * P.H * P.W;
      float am = 0.f, ah = 0.f, aw = 0.f;
      float bw[4] = {0.f, 0.f, 0.f, 0.f};
      float hh = 0.f, hw = 0.f, lh = 0.f, lw = 0.f, m = 0.f;
      int cidx[4] = {0, 0, 0, 0};
      uint32_t cval = 0;
      for (int u = 0; u < P.nU; ++u, ++ucnt) {
        const int tg = u / P.nCC;
        const int cch = u - tg * P.nCC;
        const int t = tg / P.dg, g = tg - t * P.dg;
        if (cch == 0) {
          float hs = 0.f, ws = 0.f;
          m = 0.f;
          if (pv) {
            const int i = t / P.kw, j = t - i * P.kw;
            const size_t ob = ((size_t)b * P.dg + g) * 2 * P.K2;
            hs = (float)(ho * P.sh - P.ph + i * P.dh) + ldf(off + (ob + 2 * t) * HoWo + p);
            ws = (float)(wo * P.sw - P.pw + j * P.dw) + ldf(off + (ob + 2 * t + 1) * HoWo + p);
            m = ldf(msk + (((size_t)b * P.dg + g) * P.K2 + t) * HoWo + p);
          }
          const Sample smp = make_sample(hs, ws, 1.f, P.H, P.W);
          cval = pv ? smp.cvalid : 0u;
          lh = smp.lh; lw = smp.lw; hh = 1.f - lh; hw = 1.f - lw;
          bw[0] = (cval & 1u) ? hh * hw : 0.f;
          bw[1] = (cval & 2u) ? hh * lw : 0.f;
          bw[2] = (cval & 4u) ? lh * hw : 0.f;
          bw[3] = (cval & 8u) ? lh * lw : 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) cidx[i] = smp.cidx[i];
        }
        const int ab = ucnt & 1;
        if (!mbar_wait(accf0 + 8 * ab, (ucnt >> 1) & 1, a.err, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * NC);
        const int cbase = cch * NC;                 // first channel of this chunk
        int cend = P.Cgp - cbase;                   // channels present in this chunk
        if (cend > NC) cend = NC;
        const int c_lo = chalf * (NC / 2);
        int c_hi = c_lo + NC / 2;
        if (c_hi > cend) c_hi = cend;
        const size_t gofs = (size_t)g * P.Cgp + cbase;
        for (int c0 = c_lo; c0 < c_hi; c0 += 8) {
          float gc[8];
          tmem_ld8(tb + c0, gc);
          if (cval != 0u) {
            float v[4][8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (cval & (1u << i)) {
                load_corner8<T>(xt + (xbase + cidx[i]) * P.CS + gofs + c0, v[i]);
              } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float bil = bw[0] * v[0][e] + bw[1] * v[1][e] + bw[2] * v[2][e] + bw[3] * v[3][e];
              const float dh = hw * (v[2][e] - v[0][e]) + lw * (v[3][e] - v[1][e]);
              const float dw = hh * (v[1][e] - v[0][e]) + lh * (v[3][e] - v[2][e]);
              am = fmaf(gc[e], bil, am);
              ah = fmaf(gc[e], dh, ah);
              aw = fmaf(gc[e], dw, aw);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (cval & (1u << i)) {
                const float s = bw[i] * m;
                float* dst = a.gx_nhwc + (xbase + cidx[i]) * P.CS + gofs + c0;
                red_add_v4(dst, gc[0] * s, gc[1] * s, gc[2] * s, gc[3] * s);
                red_add_v4(dst + 4, gc[4] * s, gc[5] * s, gc[6] * s, gc[7] * s);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce0 + 8 * ab);
        if (cch == P.nCC - 1) {
          // combine the two channel halves of this (tap, group) through smem
          const int rb = tgcnt & 1;
          const uint32_t rph = (tgcnt >> 1) & 1;
          if (chalf == 1) {
            if (!mbar_wait(rede0 + 8 * rb, rph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
            red[rb][row][0] = am;
            red[rb][row][1] = ah;
            red[rb][row][2] = aw;
            __syncwarp();
            if (lane == 0) mbar_arrive(redf0 + 8 * rb);
          } else {
            if (!mbar_wait(redf0 + 8 * rb, rph, a.err, &abort_flag)) { ok = false; break; }
            const float tm = am + red[rb][row][0];
            const float th = ah + red[rb][row][1];
            const float tw = aw + red[rb][row][2];
            __syncwarp();
            if (lane == 0) mbar_arrive(rede0 + 8 * rb);
            if (pv) {
              const size_t gb = (size_t)b * P.dg + g;
              goff[((gb * P.K2 + t) * 2 + 0) * HoWo + p] = Elem<T>::from_f(th * m);
              goff[((gb * P.K2 + t) * 2 + 1) * HoWo + p] = Elem<T>::from_f(tw * m);
              gmsk[(gb * P.K2 + t) * HoWo + p] = Elem<T>::from_f(tm);
            }
          }
          ++tgcnt;
          am = ah = aw = 0.f;
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
            const uint32_t bt = sbase + s * stageBytes + NS * kATile;
            mbar_arrive_expect_tx(full0 + 8 * s, NS * bTile);
            bulk_g2s(bt, a.wpk + (size_t)(u * P.nKo + ko) * P.wd_tile_bytes, NS * bTile,
                     full0 + 8 * s);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 1, 0, kTileM, NC);
      uint32_t kidx = 0, ucnt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        for (int u = 0; u < P.nU && ok; ++u, ++ucnt) {
          const int ab = ucnt & 1;
          if (!mbar_wait(acce0 + 8 * ab, ((ucnt >> 1) & 1) ^ 1, a.err, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dt = tmem_base + (uint32_t)(ab * NC);
          for (int ko = 0; ko < P.nKo; ++ko, ++kidx) {
            const int s = kidx % S;
            const uint32_t ph = (kidx / S) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t at = sbase + s * stageBytes;
            const uint32_t bt = at + NS * kATile;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sw128_desc(at + kk * 2048, 8192, 1024);
              const uint64_t bd = sw128_desc(bt + kk * 32, 16, 1024);
              umma_f16(dt, ad, bd, idesc, (ko | kk) != 0);
              if constexpr (NS == 2) {
                const uint64_t adl = sw128_desc(at + kATile + kk * 2048, 8192, 1024);
                const uint64_t bdl = sw128_desc(bt + bTile + kk * 32, 16, 1024);
                umma_f16(dt, ad, bdl, idesc, 1);
                umma_f16(dt, adl, bd, idesc, 1);
              }
            }
            umma_commit(empty0 + 8 * s);
          }
          if (!ok) break;
          umma_commit(accf0 + 8 * ab);
        }
      }
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

int launch_backward_data(const BwdDataArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const size_t stageBytes = (size_t)P.nsplit * (128 * 128 + (size_t)P.NC * 128);
  int S = (int)((kBwdSmemBudget - 1024) / stageBytes);
  if (S > kMaxStages) S = kMaxStages;
  if (S < 2) return DCN_E_UNSUPPORTED;
  BwdDataArgs args = a;
  args.stages = S;
  const size_t smem = 1024 + (size_t)S * stageBytes;
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
