// Backward of DCNv2, data side, part 1: the column gradients
//
//   gcol[pixel, (t,g,c)] = sum_co grad_out[b, co, pixel] * W[co, g*Cg + c, t]
//
// (the reference's per-batch cuBLAS  columns = W^T . grad_out, com.cu:789-793)
// as one persistent warp-specialised tcgen05 GEMM: M = 128 pixels, N = a
// channel chunk of one (tap, group), K = Co.  gcol rows are written as
// [pixel][tap][group][Cgp] (packed channel order; bf16/f16 for 16-bit inputs,
// f32 for f32 inputs) for the scatter kernel (dcn_bwd_scatter.cu), which turns
// them into grad_input, grad_offset and grad_mask at full occupancy.
//
// CTA roles (512 threads):
//   warp 0      bulk copies of pre-packed grad_out chunks (128 pixels x 64 Co,
//               K-major SW128) into an smem ring, once per tile when all Co
//               chunks fit (warps 1-3 idle)
//   warps 4-11  epilogue: TMEM -> registers -> 16-byte global stores
//   warp 12     bulk-copy producer of the pre-packed W^T tile (K-major SW128)
//   warp 13     TMEM owner and tcgen05.mma issuer (warps 14-15 idle)
// The accumulator is double-buffered in TMEM so the epilogue of one unit
// overlaps the GEMM of the next.
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
  const int NC = P.gNC;                            // columns of one unit (<= 256)
  const uint32_t bTile = (uint32_t)NC * 128u;
  const uint32_t stageBytes = NS * bTile;          // one W^T stage (B operand)
  const uint32_t aSlot = NS * kATile;              // one grad_out chunk (A operand)
  const int S = a.stages;
  const int RA = a.a_slots;
  // A chunks (128 pixels x 64 Co) are loaded once per tile and reused by every
  // unit when the ring holds all Co chunks (resident), else re-streamed per unit
  const bool resident = RA >= P.nKo;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages + 5];
  __shared__ __align__(8) uint64_t abars[2 * kMaxASlots];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = smem_u32(&bars[0]);
  const uint32_t empty0 = smem_u32(&bars[kMaxStages]);
  const uint32_t accf0 = smem_u32(&bars[2 * kMaxStages]);
  const uint32_t acce0 = smem_u32(&bars[2 * kMaxStages + 2]);
  const uint32_t drain = smem_u32(&bars[2 * kMaxStages + 4]);
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

  const int nTiles = (a.npix + kTileM - 1) / kTileM;   // tiles of this pixel chunk
  const int pend = a.pix0 + a.npix;
  if (warp == kMmaWarp) DCN_TS(1000);
  const int HoWo = P.HoWo;

  // Roles by warpgroup.  setmaxnreg sits at the top of each warpgroup's branch
  // (one instruction per warpgroup): the two epilogue warpgroups grow to 200
  // registers, the loader/idle and control warpgroups shrink to 56.
  if (warp >= kEpiWarp0 && warp < kTmaWarp) {
    regs_inc<200>();
    // ------------------------------------------------ epilogue: gcol TMEM -> global
    // Warp e reads TMEM lane quarter e % 4 (its 32 pixel rows) and half of the
    // unit's columns; every thread writes whole 16-byte runs of its pixel's row.
    using G = typename std::conditional<std::is_same<T, float>::value, float, T>::type;
    constexpr int EPV = 16 / (int)sizeof(G);
    const int ew = warp - kEpiWarp0;              // 0..7
    const int q4 = warp & 3;                      // TMEM lane quarter
    const int half = ew >> 2;
    const int row = q4 * 32 + lane;
    const int rowlen = P.K2 * P.dg * P.Cgp;       // gcol row: [tap][group][Cgp]
    G* __restrict__ gcol = reinterpret_cast<G*>(a.gcol);
    uint32_t ucnt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
      const int pix = a.pix0 + tile * kTileM + row;
      const bool pv = pix < pend;
      for (int u = 0; u < P.gnU && ok; ++u, ++ucnt) {
        const int set = u / P.nCC;
        const int cch = u - set * P.nCC;
        int cend = P.Cgp - cch * P.NC;           // channels of the chunk present
        if (cend > P.NC) cend = P.NC;
        const int ab = ucnt & 1;
        if (ew == 0) DCN_TS(4 * ucnt);
        if (!mbar_wait(accf0 + 8 * ab, (ucnt >> 1) & 1, a.err, &abort_flag)) { ok = false; break; }
        if (ew == 0) DCN_TS(4 * ucnt + 1);
        tc_fence_after();
        const uint32_t tb = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(ab * NC);
        G* drow = gcol + (size_t)(unsigned)(pix - a.pix0) * rowlen + cch * P.NC;
        const int c_lo = half * (NC / 2), c_hi = c_lo + NC / 2;
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
          // column c0 = j*NC + within: (tap, group) set*gT + j, channel within
          const int j = c0 / P.NC, within = c0 - j * P.NC;
          const int tg = set * P.gT + j;
          float v[16];
          tmem_ld16(tb + c0, v);
          G* dst = drow + tg * P.Cgp + within - c0;
          if (pv && tg < P.K2 * P.dg && within < cend && !(a.dbg & 2)) {
#pragma unroll
            for (int k = 0; k < 16 / EPV; ++k) {
              alignas(16) G o[EPV];
#pragma unroll
              for (int e = 0; e < EPV; ++e) o[e] = Elem<G>::from_f(v[k * EPV + e]);
              *reinterpret_cast<uint4*>(dst + c0 + k * EPV) = *reinterpret_cast<const uint4*>(o);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce0 + 8 * ab);
        if (ew == 0) DCN_TS(4 * ucnt + 3);
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
      const int nload = resident ? P.nKo : P.gnU * P.nKo;  // chunk loads per tile
      const uint32_t blk = NS * 8192u;
      for (int tile = blockIdx.x; tile < nTiles && ok; tile += gridDim.x) {
        for (int l = 0; l < nload; ++l, ++aseq) {
          const int ko = l % P.nKo;
          const int r = aseq % RA;
          const uint32_t ph = (aseq / RA) & 1u;
          if (!mbar_wait(aempty0 + 8 * r, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
          const uint32_t at = abase + (uint32_t)r * aSlot;
          const int pb0 = a.pix0 / 64 + tile * 2;
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
        for (int u = 0; u < P.gnU && ok; ++u) {
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
        for (int u = 0; u < P.gnU && ok; ++u, ++ucnt) {
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
            DCN_TS(700 + 4 * ucnt + (ko & 3));
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
            if (!resident || u == P.gnU - 1) umma_commit(aempty0 + 8 * r);
          }
          if (!ok) break;
          umma_commit(accf0 + 8 * ab);
        }
        aseq0 += resident ? P.nKo : P.gnU * P.nKo;
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
  const size_t bStage = (size_t)P.nsplit * P.gNC * 128;    // W^T stage
  const size_t aSlot = (size_t)P.nsplit * 128 * 128;       // grad_out chunk
  const size_t avail = kBwdSmemLimit - 1024;
  // Preference: A double-buffered across tiles (2 x nKo slots), then resident
  // (nKo slots), then streamed (2 slots); W^T ring of up to 12 stages, at least 2.
  int S = 0, RA = 0;
  const int ras[3] = {2 * P.nKo, P.nKo, 2};
  for (int ri = 0; ri < 3 && !RA; ++ri) {
    const int ra = ras[ri];
    if (ra > kMaxASlots) continue;
    const size_t fixed = (size_t)ra * aSlot;
    if (fixed + 2 * bStage > avail) continue;
    int s = (int)((avail - fixed) / bStage);
    if (s > 12) s = 12;
    RA = ra;
    S = s;
  }
  if (!RA) return DCN_E_UNSUPPORTED;
  BwdDataArgs args = a;
  args.stages = S;
  args.a_slots = RA;
  const size_t smem = 1024 + (size_t)S * bStage + (size_t)RA * aSlot;
  const int ntiles = (a.npix + kTileM - 1) / kTileM;
  int grid = ntiles < a.num_sms ? ntiles : a.num_sms;
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
