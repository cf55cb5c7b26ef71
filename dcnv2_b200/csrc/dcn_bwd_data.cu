// Backward of DCNv2, data side, part 1: the column gradients
//
//   gcol[pixel, (t,g,c)] = sum_co grad_out[b, co, pixel] * W[co, g*Cg + c, t]
//
// (the reference's per-batch cuBLAS  columns = W^T . grad_out, com.cu:789-793)
// as one persistent warp-specialised tcgen05 GEMM: M = 128 pixels, N = one unit
// of gNC columns (gT (tap, group)s x NC channels), K = Co.  gcol rows are written
// as [pixel][tap][group][Cgp] (packed channel order; bf16/f16 for 16-bit inputs,
// f32 for f32 inputs) for the scatter kernel (dcn_bwd_scatter.cu).
//
// Each CTA owns one unit and a strided set of pixel tiles: the unit's W^T tiles
// are loaded once and stay in shared memory when they fit (else they stream
// through a ring per tile), and the grad_out chunks of each tile stream through
// an A ring; CTAs of different units visit the same tiles at about the same
// time, so the grad_out reads of the other units hit L2.
//
// CTA roles (512 threads):
//   warp 0      copies of grad_out chunks (128 pixels x 64 Co, SW128) into the
//               A ring (warps 1-3 idle): TMA tiles read from grad_output itself
//               (16-bit types; MN-major) or bulk copies of pre-packed blocks
//               (K-major; f32 as bf16 hi/lo)
//   warps 4-11  epilogue: TMEM -> registers -> shared-memory transpose -> global
//               stores of whole 64- or 128-byte row segments
//   warp 12     bulk copies of the unit's pre-packed W^T tiles (K-major SW128)
//   warp 13     TMEM owner and tcgen05.mma issuer (warps 14-15 idle)
// The accumulator is double-buffered in TMEM so the epilogue of one tile
// overlaps the GEMM of the next.
#include "dcn_common.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

#define DCN_TS(slot) \
  do { if (DCN_STUDY_ON && a.ts && blockIdx.x == 0 && lane == 0 && (slot) < 1024) a.ts[(slot)] = globaltimer(); } while (0)

constexpr int kThreads = 512;  // 4 warpgroups
constexpr int kAWarps = 4;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;
constexpr int kTmaWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kStageRowBytes = 128;                          // transpose buffer row (one warp row)
constexpr int kStageBytes = kEpiWarps * 32 * kStageRowBytes;  // 32 KB

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    dcn_bwd_data_kernel(const __grid_constant__ BwdDataArgs a) {
  using G = typename std::conditional<std::is_same<T, float>::value, float, T>::type;
  constexpr int NS = OpOf<T>::kSplit ? 2 : 1;
  constexpr uint32_t kATile = 128 * 128;
  const Plan& P = a.plan;
  const int NC = P.gNC;                            // columns of one unit (<= 256)
  const uint32_t bTile = (uint32_t)NC * 128u;
  const uint32_t stageBytes = NS * bTile;          // one W^T tile (B operand)
  const uint32_t aSlot = NS * kATile;              // one grad_out chunk (A operand)
  const int S = a.stages;
  const int RA = a.a_slots;
  const bool wres = S >= P.nKo;                    // W^T of the unit resident in smem

  // work: unit u, tiles r, r + cpu, ...
  const int nTiles = (a.npix + kTileM - 1) / kTileM;
  const int cpu = gridDim.x / P.gnU;               // CTAs per unit
  const int u = blockIdx.x % P.gnU;
  const int r0 = blockIdx.x / P.gnU;
  const int set = u / P.nCC;
  const int cch = u - set * P.nCC;

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
  const uint32_t abase = sbase + (uint32_t)S * stageBytes;   // A ring after the W^T stages
  const uint32_t xbase = abase + (uint32_t)RA * aSlot;       // transpose buffer after the A ring

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
  pdl_wait();
  const int pend = a.pix0 + a.npix;
  if (warp == kMmaWarp) DCN_TS(1000);

  // Roles by warpgroup.  setmaxnreg sits at the top of each warpgroup's branch
  // (one instruction per warpgroup): the two epilogue warpgroups grow to 200
  // registers, the loader/idle and control warpgroups shrink to 56.
  if (warp >= kEpiWarp0 && warp < kTmaWarp) {
    regs_inc<200>();
    // ------------------------------------------------ epilogue: gcol TMEM -> global
    // Warp e reads TMEM lane quarter e % 4 (its 32 pixel rows) and every other
    // block of BC columns (BC x sizeof(G) = 64 or 128 bytes per row).  A block
    // goes through the warp's slice of the transpose buffer (16-byte chunks
    // XOR-swizzled by row, conflict-free both ways) and leaves as whole row
    // segments: 128 / (BC x sizeof(G)) ... 8 rows per store instruction.
    constexpr int BC = 32;                                  // columns per block
    constexpr int RB = BC * (int)sizeof(G);                 // bytes per row of a block
    constexpr int NCH = RB / 16;                            // 16-byte chunks per row
    constexpr int RPI = 32 / NCH;                           // rows per store instruction
    const int ew = warp - kEpiWarp0;              // 0..7
    const int q4 = warp & 3;                      // TMEM lane quarter
    const int half = ew >> 2;
    const int rowlen = P.K2 * P.dg * P.Cgp;       // gcol row: [tap][group][Cgp]
    G* __restrict__ gcol = reinterpret_cast<G*>(a.gcol);
    const uint32_t xw = xbase + (uint32_t)ew * 32u * kStageRowBytes;
    auto swz = [&](int row, int c) {              // physical 16-byte chunk of (row, c)
      return NCH == 8 ? (c ^ (row & 7)) : (c ^ ((row >> 1) & 3));
    };
    int cend = P.Cgp - cch * P.NC;                // channels of the chunk present
    if (cend > P.NC) cend = P.NC;
    uint32_t it = 0;
    bool ok = true;
    for (int tile = r0; tile < nTiles && ok; tile += cpu, ++it) {
      const int ab = it & 1;
      if (ew == 0) DCN_TS(4 * it);
      if (!mbar_wait_warp(accf0 + 8 * ab, (it >> 1) & 1, a.err, &abort_flag)) { ok = false; break; }
      if (ew == 0) DCN_TS(4 * it + 1);
      tc_fence_after();
      const uint32_t tb = tmem_base + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(ab * NC);
      const int nblk = NC / BC;
      const int nmine = (nblk - half + 1) / 2;    // blocks half, half + 2, ...
      for (int bi = 0; bi < nmine; ++bi) {
        const int c0 = (half + 2 * bi) * BC;
        float v[32];
        tmem_ld32(tb + c0, v);
        if (bi == nmine - 1) {
          // every TMEM column of this warp is in registers: release the buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acce0 + 8 * ab);
        }
        // registers -> transpose buffer (row = lane)
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint4 w;
          if constexpr (sizeof(G) == 4) {
            w = make_uint4(__float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]),
                           __float_as_uint(v[4 * c + 2]), __float_as_uint(v[4 * c + 3]));
          } else {
            constexpr int kBF = std::is_same<G, __nv_bfloat16>::value ? 1 : 0;
            w = make_uint4(pack2<kBF>(v[8 * c], v[8 * c + 1]), pack2<kBF>(v[8 * c + 2], v[8 * c + 3]),
                           pack2<kBF>(v[8 * c + 4], v[8 * c + 5]), pack2<kBF>(v[8 * c + 6], v[8 * c + 7]));
          }
          sts_v4(xw + lane * RB + swz(lane, c) * 16, w);
        }
        __syncwarp();
        // transpose buffer -> global, RPI rows per instruction
        const int j = c0 / P.NC, within = c0 - j * P.NC;
        const int tg = set * P.gT + j;
        if (tg < P.K2 * P.dg && within < cend && !DCN_SKIP(2)) {
#pragma unroll
          for (int i = 0; i < 32 / RPI; ++i) {
            const int row = i * RPI + lane / NCH, c = lane % NCH;
            const int pix = a.pix0 + tile * kTileM + q4 * 32 + row;
            const uint4 w = lds_v4(xw + row * RB + swz(row, c) * 16);
            if (pix < pend) {
              G* dst = gcol + (size_t)(unsigned)(pix - a.pix0) * rowlen + tg * P.Cgp + cch * P.NC +
                       within + c * (16 / (int)sizeof(G));
              *reinterpret_cast<uint4*>(dst) = w;
            }
          }
        }
        __syncwarp();
      }
      if (nmine == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce0 + 8 * ab);
      }
      if (ew == 0) DCN_TS(4 * it + 3);
    }
  } else {
    regs_dec<56>();
    if (warp < kAWarps) {
      // ---------------------------------------------- grad_out chunk loader
      // One thread copies the two 64-pixel blocks of each Co chunk into the A
      // ring: pre-packed blocks (K-major, 128-byte swizzle; f32: hi and lo) by
      // bulk copy, or TMA boxes of 16-bit grad_output.
      if (warp == 0 && lane == 0) {
        int r = 0;                                  // A ring slot and its phase
        uint32_t ph = 0;
        bool ok = true;
        const uint32_t blk = NS * 8192u;
        const bool gdirect = NS == 1 && a.gdirect == kGoutNchw;
        const bool gnhwc = NS == 1 && a.gdirect == kGoutNhwc;
        const int nPBi = P.HoWo / 64;              // 64-pixel blocks per image (gdirect)
        for (int tile = r0; tile < nTiles && ok; tile += cpu) {
          for (int ko = 0; ko < P.nKo; ++ko, (++r == RA ? (r = 0, ph ^= 1u) : 0u)) {
            if (!mbar_wait(aempty0 + 8 * r, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
            const uint32_t at = abase + (uint32_t)r * aSlot;
            const int pb0 = a.pix0 / 64 + tile * 2;
            const int nb = (pb0 + 1 < P.nPB) ? 2 : 1;
            mbar_arrive_expect_tx(afull0 + 8 * r, (uint32_t)nb * blk);
            for (int h = 0; h < nb; ++h) {
              if (gdirect) {
                // 64 pixels x 64 Co straight from grad_output (one image: HoWo % 64 == 0);
                // pixels contiguous, so the tile is MN-major; Co past the end reads zeros
                const int pbi = pb0 + h, b = pbi / nPBi;
                tma_load_3d(at + h * 8192u, &a.gmap, (pbi - b * nPBi) * 64, ko * 64, b, afull0 + 8 * r);
              } else if (gnhwc) {
                // channels-last: 64 Co of 64 consecutive pixels, the packed block's layout
                tma_load_3d(at + h * 8192u, &a.gmap, ko * 64, (pb0 + h) * 64, 0, afull0 + 8 * r);
              } else {
                const uint8_t* src = a.gpk + ((size_t)(pb0 + h) * P.nKo + ko) * blk;
                bulk_g2s(at + h * 8192u, src, 8192u, afull0 + 8 * r);
                if constexpr (NS == 2) bulk_g2s(at + kATile + h * 8192u, src + 8192, 8192u, afull0 + 8 * r);
              }
            }
          }
        }
      }
    } else if (warp == kTmaWarp) {
      // ---------------------------------------------- W^T tiles of the unit
      if (lane == 0) {
        int ws = 0;                                 // W^T ring stage and its phase
        uint32_t wph = 0;
        bool ok = true;
        for (int tile = r0; tile < nTiles && ok; tile += cpu) {
          for (int ko = 0; ko < P.nKo; ++ko) {
            const int s = wres ? ko : ws;
            const uint32_t ph = wres ? 0u : wph;
            if (++ws == S) { ws = 0; wph ^= 1u; }
            if (wres && tile != r0) break;        // resident: loaded once
            if (!wres && !mbar_wait(empty0 + 8 * s, ph ^ 1u, a.err, &abort_flag)) { ok = false; break; }
            const uint32_t bt = sbase + s * stageBytes;
            mbar_arrive_expect_tx(full0 + 8 * s, NS * bTile);
            bulk_g2s(bt, a.wpk + (size_t)(u * P.nKo + ko) * P.wd_tile_bytes, NS * bTile,
                     full0 + 8 * s);
          }
          if (wres) break;
        }
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------- MMA issuer
      if (lane == 0) {
        // A: packed grad_out chunks are K-major (Co contiguous per pixel row);
        // tiles read from grad_output directly are MN-major (pixels contiguous
        // per Co row, the two 64-pixel halves 8 KB apart)
        const bool gdirect = NS == 1 && a.gdirect == kGoutNchw;
        const uint32_t idesc = make_idesc(OpOf<T>::kBF16, gdirect ? 1 : 0, 0, kTileM, NC);
        uint32_t it = 0;
        int ar = 0, ms = 0;                         // A slot / W^T stage and their phases
        uint32_t aph = 0, mph = 0;
        bool ok = true;
        for (int tile = r0; tile < nTiles && ok; tile += cpu, ++it) {
          const int ab = it & 1;
          if (!mbar_wait(acce0 + 8 * ab, ((it >> 1) & 1) ^ 1, a.err, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t dt = tmem_base + (uint32_t)(ab * NC);
          for (int ko = 0; ko < P.nKo; ++ko) {
            const int r = ar;
            const uint32_t rph = aph;
            if (++ar == RA) { ar = 0; aph ^= 1u; }
            const int s = wres ? ko : ms;
            const uint32_t ph = wres ? 0u : mph;
            if (++ms == S) { ms = 0; mph ^= 1u; }
            if (!mbar_wait(afull0 + 8 * r, rph, a.err, &abort_flag)) { ok = false; break; }
            if ((!wres || it == 0) && !mbar_wait(full0 + 8 * s, ph, a.err, &abort_flag)) { ok = false; break; }
            DCN_TS(700 + 4 * it + (ko & 3));
            tc_fence_after();
            const uint32_t at = abase + (uint32_t)r * aSlot;
            const uint32_t bt = sbase + s * stageBytes;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = gdirect ? sw128_desc(at + kk * 2048, 8192, 1024)
                                          : sw128_desc(at + kk * 32, 16, 1024);
              const uint64_t bd = sw128_desc(bt + kk * 32, 16, 1024);
              if (!DCN_SKIP(4)) umma_f16(dt, ad, bd, idesc, (ko | kk) != 0);
              if constexpr (NS == 2) {
                const uint64_t adl = sw128_desc(at + kATile + kk * 32, 16, 1024);
                const uint64_t bdl = sw128_desc(bt + bTile + kk * 32, 16, 1024);
                umma_f16(dt, ad, bdl, idesc, 1);
                umma_f16(dt, adl, bd, idesc, 1);
              }
            }
            if (!wres) umma_commit(empty0 + 8 * s);
            umma_commit(aempty0 + 8 * r);
          }
          if (!ok) break;
          umma_commit(accf0 + 8 * ab);
          DCN_TS(600 + it);
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
  const size_t bStage = (size_t)P.nsplit * P.gNC * 128;    // W^T tile
  const size_t aSlot = (size_t)P.nsplit * 128 * 128;       // grad_out chunk
  const size_t avail = kBwdSmemLimit - 1024 - kStageBytes;
  // W^T of the unit resident (nKo tiles) with the rest as A ring, else a W^T
  // ring of at least 2 stages beside 2 A slots
  int S = 0, RA = 0;
  if (P.nKo <= kMaxStages && (size_t)P.nKo * bStage + 2 * aSlot <= avail) {
    S = P.nKo;
    RA = (int)((avail - (size_t)S * bStage) / aSlot);
  } else {
    RA = 2;
    if (2 * aSlot + 2 * bStage > avail) return DCN_E_UNSUPPORTED;
    S = (int)((avail - 2 * aSlot) / bStage);
    if (S > kMaxStages) S = kMaxStages;
    if (S >= P.nKo) S = P.nKo - 1;               // keep the streaming mode (S < nKo)
    if (S < 2) return DCN_E_UNSUPPORTED;
  }
  if (RA > kMaxASlots) RA = kMaxASlots;
  BwdDataArgs args = a;
  args.stages = S;
  args.a_slots = RA;
  const size_t smem = 1024 + (size_t)S * bStage + (size_t)RA * aSlot + kStageBytes;
  const int ntiles = (a.npix + kTileM - 1) / kTileM;
  // CTAs per unit: every unit gets the same number, at most one per tile
  int cpu = a.num_sms / P.gnU;
  if (cpu < 1) cpu = 1;
  if (cpu > ntiles) cpu = ntiles;
  const long long grid = (long long)cpu * P.gnU;
  if (ntiles <= 0) return DCN_OK;
  if (grid > (1LL << 30)) return DCN_E_UNSUPPORTED;
  cudaError_t e = cudaSuccess;
  switch (P.dtype) {
    case DCN_F32:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<float>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch_k(dcn_bwd_data_kernel<float>, dim3((int)grid), dim3(kThreads), smem, stream, args);
      break;
    case DCN_F16:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<__half>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) e = launch_k(dcn_bwd_data_kernel<__half>, dim3((int)grid), dim3(kThreads), smem, stream, args);
      break;
    default:
      e = cudaFuncSetAttribute(dcn_bwd_data_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess)
        e = launch_k(dcn_bwd_data_kernel<__nv_bfloat16>, dim3((int)grid), dim3(kThreads), smem, stream, args);
      break;
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
