// Forward DCNv2 as one fused, persistent, warp-specialised implicit GEMM on
// tcgen05 tensor cores (replaces the reference's im2col + WMMA GEMM pair,
// com.cu:151-195 and com.cu:46-117, and never materialises the columns).
//
//   D[pixel, co] = sum_{t, g, c} A[pixel, (t,g,c)] * Wt[co, (t,g,c)]
//   A[pixel, (t,g,c)] = mask * bilinear(x_nhwc[b, :, :, g, c], pos(pixel, t) + offset)
//
// CTA roles (448 threads):
//   warps 0-7  gather producers: one pixel row and 32 channels per thread; build
//              the A tile (128 pixels x 64 channels, K-major, 128B swizzle) in smem
//   warps 8-11 epilogue: TMEM -> registers, + bias, NCHW store
//   warp 12    bulk-copy (TMA) producer of the pre-packed weight tile
//   warp 13    TMEM owner and single-thread tcgen05.mma issuer
// A/B stages form an mbarrier ring; the accumulator is double-buffered in TMEM so
// the epilogue of tile i overlaps the main loop of tile i+1.
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kFwdThreads = 448;
constexpr int kProdThreads = 256;
constexpr int kEpiWarp0 = 8;
constexpr int kTmaWarp = 12;
constexpr int kMmaWarp = 13;

template <typename T>
__global__ void __launch_bounds__(kFwdThreads, 1)
    dcn_fwd_kernel(const __grid_constant__ FwdArgs a) {
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;  // 128 rows x 128 B
  const Plan& P = a.plan;
  const int NT = P.NT;
  const uint32_t bTile = (uint32_t)NT * 128u;
  const uint32_t stageBytes = NS * (kATile + bTile);
  const int S = a.stages;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 5];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 2]);
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 4]);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, kProdThreads / 32 + 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 4);
    }
    mbar_init(drain, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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

  if (warp < kProdThreads / 32) {
    // ------------------------------------------------ gather producers
    const int r = tid & 127, half = tid >> 7;
    const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
    const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
    const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
    uint32_t kidx = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      const int pt = tile / P.nCoT;
      const long long pix = (long long)pt * kTileM + r;
      const bool pv = pix < P.totalP;
      const int b = pv ? (int)(pix / HoWo) : 0;
      const int p = pv ? (int)(pix - (long long)b * HoWo) : 0;
      const int ho = p / P.Wo, wo = p - ho * P.Wo;
      const T* xb = xt + (size_t)b * P.H * P.W * P.CS;
      Sample smp;
      for (int kc = 0; kc < P.nK; ++kc, ++kidx) {
        const int t = kc / (P.dg * P.nCB);
        const int rem = kc - t * (P.dg * P.nCB);
        const int g = rem / P.nCB;
        const int cb = rem - g * P.nCB;
        if (cb == 0) {
          float hs = 0.f, ws = 0.f, m = 0.f;
          if (pv) {
            const int i = t / P.kw, j = t - i * P.kw;
            const size_t ob = ((size_t)b * P.dg + g) * 2 * P.K2;
            hs = (float)(ho * P.sh - P.ph + i * P.dh) + ldf(off + (ob + 2 * t) * HoWo + p);
            ws = (float)(wo * P.sw - P.pw + j * P.dw) + ldf(off + (ob + 2 * t + 1) * HoWo + p);
            m = ldf(msk + (((size_t)b * P.dg + g) * P.K2 + t) * HoWo + p);
          }
          smp = make_sample(hs, ws, m, P.H, P.W);
          if (!pv) smp.cw[0] = smp.cw[1] = smp.cw[2] = smp.cw[3] = 0.f;
        }
        float acc[32];
        gather32<T>(xb, smp, g * P.Cgp + cb * kChunk + half * 32, P.CS, acc);
        const int s = kidx % S;
        const uint32_t ph = (kidx / S) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
        const uint32_t atile = sbase + s * stageBytes;
        store_row32<T>(atile, kATile, r, half * 4, acc);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(full0 + 8 * s);
      }
    }
  } else if (warp < kTmaWarp) {
    // ------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    T* __restrict__ y = reinterpret_cast<T*>(a.out);
    const T* __restrict__ bias = reinterpret_cast<const T*>(a.bias);
    int it = 0;
    for (int tile = blockIdx.x; tile < nTiles; tile += gridDim.x, ++it) {
      const int pt = tile / P.nCoT, ct = tile - pt * P.nCoT;
      const int ab = it & 1;
      if (!mbar_wait(accf0 + 8 * ab, (it >> 1) & 1, a.err, &abort_flag)) break;
      tc_fence_after();
      const long long pix = (long long)pt * kTileM + row;
      const bool pv = pix < P.totalP;
      const int b = pv ? (int)(pix / HoWo) : 0;
      const int p = pv ? (int)(pix - (long long)b * HoWo) : 0;
      T* yb = y + (size_t)b * P.Co * HoWo + p;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * NT);
      for (int c0 = 0; c0 < NT; c0 += 8) {
        float v[8];
        tmem_ld8(tbase + c0, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int co = ct * NT + c0 + j;
          if (pv && co < P.Co) {
            const float bv = (bias != nullptr) ? ldf(bias + co) : 0.f;
            yb[(size_t)co * HoWo] = Elem<T>::from_f(v[j] + bv);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * ab);
    }
  } else if (warp == kTmaWarp) {
    // ------------------------------------------------ weight tiles (bulk copy)
    if (lane == 0) {
      uint32_t kidx = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        const int ct = tile % P.nCoT;
        const uint8_t* wsrc = a.wpk + (size_t)ct * P.nK * P.wf_tile_bytes;
        for (int kc = 0; kc < P.nK; ++kc, ++kidx) {
          const int s = kidx % S;
          const uint32_t ph = (kidx / S) & 1u;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          const uint32_t btile = sbase + s * stageBytes + NS * kATile;
          mbar_arrive_expect_tx(full0 + 8 * s, NS * bTile);
          bulk_g2s(btile, wsrc + (size_t)kc * P.wf_tile_bytes, NS * bTile, full0 + 8 * s);
        }
      }
    }
  } else {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(OpOf<T>::kBF16, 0, 0, kTileM, NT);
      uint32_t kidx = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x, ++it) {
        const int ab = it & 1;
        if (!mbar_wait(acce0 + 8 * ab, ((it >> 1) & 1) ^ 1, a.err, &abort_flag)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + (uint32_t)(ab * NT);
        for (int kc = 0; kc < P.nK; ++kc, ++kidx) {
          const int s = kidx % S;
          const uint32_t ph = (kidx / S) & 1u;
          if (!mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t at = sbase + s * stageBytes;
          const uint32_t bt = at + NS * kATile;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = sw128_desc(at + kk * 32, 16, 1024);
            const uint64_t bd = sw128_desc(bt + kk * 32, 16, 1024);
            umma_f16(dt, ad, bd, idesc, (kc | kk) != 0);
            if constexpr (NS == 2) {
              const uint64_t adl = sw128_desc(at + kATile + kk * 32, 16, 1024);
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
      // drain: every issued MMA has retired before TMEM is released
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

int launch_forward(const FwdArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const int NS = P.nsplit;
  const size_t stageBytes = (size_t)NS * (128 * 128 + (size_t)P.NT * 128);
  int S = (int)((kFwdSmemBudget - 1024) / stageBytes);
  if (S > kMaxStages) S = kMaxStages;
  if (S < 2) return DCN_E_UNSUPPORTED;
  FwdArgs args = a;
  args.stages = S;
  const size_t smem = 1024 + (size_t)S * stageBytes;
  const int nTiles = P.nPT * P.nCoT;
  int grid = nTiles < a.num_sms ? nTiles : a.num_sms;
  if (grid <= 0) return DCN_OK;
  cudaError_t e;
  switch (P.dtype) {
    case DCN_F32:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      dcn_fwd_kernel<float><<<grid, kFwdThreads, smem, stream>>>(args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      dcn_fwd_kernel<__half><<<grid, kFwdThreads, smem, stream>>>(args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_fwd_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return DCN_E_CUDA;
      dcn_fwd_kernel<__nv_bfloat16><<<grid, kFwdThreads, smem, stream>>>(args);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
