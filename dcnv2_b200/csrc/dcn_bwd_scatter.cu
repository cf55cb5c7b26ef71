// Backward of DCNv2, data side, part 2: from the column gradients gcol
// (dcn_bwd_data.cu) to the gradients of input, offset and mask.  Follows the
// reference's coordinate kernel (com.cu:431-501, weights com.cu:388-429) and
// col2im scatter (com.cu:553-609, weights com.cu:526-550):
//
//   grad_mask[b, g*T+t, p]       = sum_c gcol * bilinear(x_c)
//   grad_offset[b, 2(g*T+t)+d, p] = mask * sum_c gcol * d bilinear(x_c) / d(h | w)
//   grad_input[b, c, corner]    += gcol * mask * corner weight   (fp32 red.add)
//
// A plain SIMT kernel run at high occupancy so the load and reduction latencies
// are hidden by many warps.  A warp handles 32 pixels of one (tap, group): each
// lane computes the sampling geometry of one pixel, then 8 sub-iterations take
// 4 pixels at a time, the 8 lanes of a pixel owning one 16-byte slice (8
// channels, packed order) of the pixel's gcol row and of each bilinear corner
// line; the per-pixel sums return to the owner lane for coalesced stores.  bilinear and its two
// derivatives are linear in the four corners, so each lane only forms
// S_c = sum_e gcol_e * corner_c[e]; the three channel sums follow from S and
// are reduced over the 8 lanes with shuffles.  The scatter writes grad_input in
// logical channel order (lane q: channels 4q..4q+3 and 32+4q..32+4q+3 of the
// block), so each red.add instruction of a pixel fills whole 32-byte sectors.
//
// The same corner loads also give the sampled column mask * bilinear(x_c) of
// every (pixel, tap, channel): the kernel writes it, rounded to the operand type
// (a bf16 hi/lo pair for f32), in the layout of the weight-gradient GEMM's B
// tiles, so that GEMM streams it with bulk copies instead of gathering it again
// (the reference re-runs im2col for it, com.cu:637-706).  Pixels past the end
// of the chunk up to its last 64-pixel block get zero columns.
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kThreads = 256;

// {a.x * b.x + c.x, a.y * b.y + c.y}: the sm_100 packed f32x2 FMA through the
// CUDA builtin (operands stay in register pairs; inline PTX packing them with
// mov.b64 cost extra moves)
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// 2 x f32 packed multiply (sm_100): {a.x * s, a.y * s}
__device__ __forceinline__ float2 mul2(float2 a, float s) { return __fmul2_rn(a, make_float2(s, s)); }

template <typename T>
__global__ void __launch_bounds__(kThreads, 3) dcn_bwd_scatter_kernel(const __grid_constant__ BwdDataArgs a) {
  using G = typename std::conditional<std::is_same<T, float>::value, float, T>::type;
  constexpr int LD = GatherShape<T>::kLD;
  pdl_wait();
  const Plan& P = a.plan;
  const int lane = threadIdx.x & 31;
  const int lp = lane >> 3, q = lane & 7;
  const int HoWo = P.HoWo, HW = P.H * P.W;
  const int nTG = P.K2 * P.dg;
  const int rowlen = nTG * P.Cgp;
  const int pend = a.pix0 + a.npix;
  const int ngrp = (a.npix + 63) / 64 * 2;      // 32-pixel groups covering the chunk's 64-pixel blocks
  const int nblk = P.NC / kChunk;
  const int natoms = P.nU * nblk;               // 8 KB column blocks per 64 pixels (one of hi/lo)
  const int nitems = ngrp * nTG;                // warp items: (32-pixel group, tap-group)
  const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
  const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
  const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
  const G* __restrict__ gcol = reinterpret_cast<const G*>(a.gcol);
  T* __restrict__ goff = reinterpret_cast<T*>(a.goffset);
  T* __restrict__ gmsk = reinterpret_cast<T*>(a.gmask);
  const int warp0 = (int)((blockIdx.x * kThreads + threadIdx.x) >> 5);
  const int nwarps = (int)((gridDim.x * kThreads) >> 5);

  for (int item = warp0; item < nitems; item += nwarps) {
    const int grp = fdiv(item, P.fd_ntg);
    const int tg = item - grp * nTG;
    const int t = fdiv(tg, P.fd_dg), g = tg - t * P.dg;
    // ---- geometry of pixel (group base + lane), computed once per lane
    const int mpix = a.pix0 + grp * 32 + lane;
    const bool mpv = mpix < pend;
    const int mb = mpv ? fdiv(mpix, P.fd_howo) : 0;
    const int mp = mpv ? mpix - mb * HoWo : 0;
    const int obase = mb * P.off_bs + (g * 2 * P.K2 + 2 * t) * P.off_cs + mp * P.off_ps;
    const int mbase = mb * P.msk_bs + (g * P.K2 + t) * P.msk_cs + mp * P.msk_ps;
    float mlh = 0.f, mlw = 0.f, mm = 0.f;
    int mgidx = 0;
    uint32_t mval = 0u;
    if (mpv) {
      const int i = fdiv(t, P.fd_kw), j = t - i * P.kw;
      const int ho = fdiv(mp, P.fd_wo), wo = mp - ho * P.Wo;
      const float h = (float)(ho * P.sh - P.ph + i * P.dh) + ldf(off + obase);
      const float w = (float)(wo * P.sw - P.pw + j * P.dw) + ldf(off + obase + P.off_cs);
      mm = ldf(msk + mbase);
      if (P.mask_logit) mm = 1.f / (1.f + __expf(-mm));   // sigmoid of a predictor logit
      const float hf = floorf(h), wf = floorf(w);
      const int hl = (int)hf, wl = (int)wf;
      mlh = h - hf;
      mlw = w - wf;
      if ((h > -1.f) && (w > -1.f) && (h < (float)P.H) && (w < (float)P.W) && !DCN_SKIP(1)) {
        const bool r0 = hl >= 0, r1 = hl + 1 <= P.H - 1, c0 = wl >= 0, c1 = wl + 1 <= P.W - 1;
        mval = (r0 && c0 ? 1u : 0u) | (r0 && c1 ? 2u : 0u) | (r1 && c0 ? 4u : 0u) |
               (r1 && c1 ? 8u : 0u);
        mgidx = mb * HW + hl * P.W + wl;
      }
    }
    const int d[4] = {0, 1, P.W, P.W + 1};
    float om = 0.f, oh = 0.f, ow = 0.f;   // results of this lane's own pixel
    // ---- 8 sub-iterations of 4 pixels, 8 lanes per pixel
#pragma unroll 1
    for (int sub = 0; sub < 8; ++sub) {
      const int src = sub * 4 + lp;
      const int gidx = __shfl_sync(0xffffffffu, mgidx, src);
      const float lh = __shfl_sync(0xffffffffu, mlh, src);
      const float lw = __shfl_sync(0xffffffffu, mlw, src);
      const float m = __shfl_sync(0xffffffffu, mm, src);
      const uint32_t cval = __shfl_sync(0xffffffffu, mval, src);
      const int pix = a.pix0 + grp * 32 + src;
      const float hh = 1.f - lh, hw = 1.f - lw;
      const float bw[4] = {(cval & 1u) ? hh * hw : 0.f, (cval & 2u) ? hh * lw : 0.f,
                           (cval & 4u) ? lh * hw : 0.f, (cval & 8u) ? lh * lw : 0.f};
      float S[4] = {0.f, 0.f, 0.f, 0.f};
      const G* grow = gcol + (size_t)(unsigned)(pix - a.pix0) * rowlen + tg * P.Cgp + q * 8;
      const float wc[4] = {bw[0] * m, bw[1] * m, bw[2] * m, bw[3] * m};
      const int pl = pix - a.pix0, crow = pl & 63;
      uint8_t* cdst = a.cols == nullptr ? nullptr
                      : a.cols + ((size_t)(unsigned)(pl >> 6) * P.nsplit * natoms) * 8192u +
                            crow * 128 + ((q ^ (crow & 7)) << 4);
      int cch = 0, cblk = 0;                       // channel chunk of the unit, 64-block inside it
      for (int cb = 0; cb < P.nCB; ++cb, (++cblk == nblk ? (cblk = 0, ++cch) : 0)) {
        float col[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (cval != 0u) {
          const int cofs = g * P.Cgp + cb * kChunk;
          uint4 graw[sizeof(G) / 2];
#pragma unroll
          for (int l = 0; l < (int)(sizeof(G) / 2); ++l) graw[l] = ldg_nc_v4(grow + cb * kChunk + l * 4);
          uint4 raw[4][LD];
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int l = 0; l < LD; ++l)
              raw[c][l] = (cval & (1u << c))
                              ? ldg_nc_v4(xt + (size_t)(unsigned)((gidx + d[c]) * P.CS + cofs + q * 8) + l * (8 / LD))
                              : make_uint4(0u, 0u, 0u, 0u);
          float gc[8];
          if constexpr (sizeof(G) == 4) {
            gc[0] = __uint_as_float(graw[0].x); gc[1] = __uint_as_float(graw[0].y);
            gc[2] = __uint_as_float(graw[0].z); gc[3] = __uint_as_float(graw[0].w);
            gc[4] = __uint_as_float(graw[LD - 1].x); gc[5] = __uint_as_float(graw[LD - 1].y);
            gc[6] = __uint_as_float(graw[LD - 1].z); gc[7] = __uint_as_float(graw[LD - 1].w);
          } else {
            unpack8<G>(graw[0], gc);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float v[8];
            unpack_slice<T>(raw[c], v);
            float2 sp = make_float2(0.f, 0.f);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float2 ve = make_float2(v[e], v[e + 1]);
              sp = fma2(make_float2(gc[e], gc[e + 1]), ve, sp);
              const float2 ce = fma2(ve, make_float2(wc[c], wc[c]), make_float2(col[e], col[e + 1]));
              col[e] = ce.x;
              col[e + 1] = ce.y;
            }
            S[c] += sp.x + sp.y;
          }
          if (!DCN_SKIP(2)) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if (cval & (1u << c)) {
                const float sk = wc[c];
                float* dst = a.gx_nhwc + (size_t)(unsigned)((gidx + d[c]) * P.CS + cofs);
                const float2 s0 = mul2(make_float2(gc[0], gc[1]), sk);
                const float2 s1 = mul2(make_float2(gc[2], gc[3]), sk);
                const float2 s2 = mul2(make_float2(gc[4], gc[5]), sk);
                const float2 s3 = mul2(make_float2(gc[6], gc[7]), sk);
                red_add_v4(dst + slice_lo(q), s0.x, s0.y, s1.x, s1.y);
                red_add_v4(dst + slice_hi(q), s2.x, s2.y, s3.x, s3.y);
              }
            }
          }
        }
        if (cdst != nullptr) {
          // column block of (unit tg * nCC + channel chunk, 64-channel block inside it)
          const int atom = (tg * P.nCC + cch) * nblk + cblk;
          uint8_t* dst = cdst + (size_t)atom * 8192u;
          if constexpr (OpOf<T>::kSplit) {
            uint4 hi, lo;
            split2(col[0], col[1], hi.x, lo.x);
            split2(col[2], col[3], hi.y, lo.y);
            split2(col[4], col[5], hi.z, lo.z);
            split2(col[6], col[7], hi.w, lo.w);
            *reinterpret_cast<uint4*>(dst) = hi;
            *reinterpret_cast<uint4*>(dst + (size_t)natoms * 8192u) = lo;
          } else {
            constexpr int kBF = OpOf<T>::kBF16;
            uint4 u;
            u.x = pack2<kBF>(col[0], col[1]);
            u.y = pack2<kBF>(col[2], col[3]);
            u.z = pack2<kBF>(col[4], col[5]);
            u.w = pack2<kBF>(col[6], col[7]);
            *reinterpret_cast<uint4*>(dst) = u;
          }
        }
      }
      float am = bw[0] * S[0] + bw[1] * S[1] + bw[2] * S[2] + bw[3] * S[3];
      float ah = hw * (S[2] - S[0]) + lw * (S[3] - S[1]);
      float aw = hh * (S[1] - S[0]) + lh * (S[3] - S[2]);
#pragma unroll
      for (int sh = 1; sh < 8; sh <<= 1) {
        am += __shfl_xor_sync(0xffffffffu, am, sh);
        ah += __shfl_xor_sync(0xffffffffu, ah, sh);
        aw += __shfl_xor_sync(0xffffffffu, aw, sh);
      }
      // hand the sums of pixel src to its owner lane (held by lane 8 * (owner - 4*sub))
      const int from = 8 * ((lane - sub * 4) & 3);
      const float tm = __shfl_sync(0xffffffffu, am, from);
      const float th = __shfl_sync(0xffffffffu, ah, from);
      const float tw = __shfl_sync(0xffffffffu, aw, from);
      if ((lane >> 2) == sub) {
        om = tm;
        oh = th;
        ow = tw;
      }
    }
    if (mpv) {
      goff[obase] = Elem<T>::from_f(oh * mm);
      goff[obase + P.off_cs] = Elem<T>::from_f(ow * mm);
      // with logits: d/dx sigmoid(x) = s (1 - s)
      gmsk[mbase] = Elem<T>::from_f(P.mask_logit ? om * mm * (1.f - mm) : om);
    }
  }
}

}  // namespace

int launch_backward_scatter(const BwdDataArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const long long nitems = (long long)(a.npix + 63) / 64 * 2 * (P.K2 * P.dg);
  long long blocks = (nitems + 7) / 8;
  const long long cap = (long long)a.num_sms * 16;
  if (blocks > cap) blocks = cap;
  if (blocks <= 0) return DCN_OK;
  cudaError_t e;
  switch (P.dtype) {
    case DCN_F32:
      e = launch_k(dcn_bwd_scatter_kernel<float>, dim3((int)blocks), dim3(kThreads), 0, stream, a);
      break;
    case DCN_F16:
      e = launch_k(dcn_bwd_scatter_kernel<__half>, dim3((int)blocks), dim3(kThreads), 0, stream, a);
      break;
    default:
      e = launch_k(dcn_bwd_scatter_kernel<__nv_bfloat16>, dim3((int)blocks), dim3(kThreads), 0, stream, a);
      break;
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
