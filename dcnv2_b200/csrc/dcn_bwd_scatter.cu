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
// are hidden by many warps.  A warp handles 4 pixels of one (tap, group); the
// 8 lanes of a pixel own one 16-byte slice (8 channels, packed order) of the
// pixel's gcol row and of each bilinear corner line.  bilinear and its two
// derivatives are linear in the four corners, so each lane only forms
// S_c = sum_e gcol_e * corner_c[e]; the three channel sums follow from S and
// are reduced over the 8 lanes with shuffles.  The scatter writes grad_input in
// logical channel order (lane q: channels 4q..4q+3 and 32+4q..32+4q+3 of the
// block), so each red.add instruction of a pixel fills whole 32-byte sectors.
#include "dcn_common.cuh"
#include "dcn_gather.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int kThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads) dcn_bwd_scatter_kernel(const __grid_constant__ BwdDataArgs a) {
  using G = typename std::conditional<std::is_same<T, float>::value, float, T>::type;
  constexpr int LD = GatherShape<T>::kLD;
  const Plan& P = a.plan;
  const int lane = threadIdx.x & 31;
  const int lp = lane >> 3, q = lane & 7;
  const int HoWo = P.HoWo, HW = P.H * P.W;
  const int nTG = P.K2 * P.dg;
  const int rowlen = nTG * P.Cgp;
  const int npg = (a.npix + 3) / 4;
  const int pend = a.pix0 + a.npix;
  const int nitems = npg * nTG;                 // < 2^31 (the plan bounds B*Ho*Wo*K2*dg)
  const T* __restrict__ xt = reinterpret_cast<const T*>(a.xt);
  const T* __restrict__ off = reinterpret_cast<const T*>(a.offset);
  const T* __restrict__ msk = reinterpret_cast<const T*>(a.mask);
  const G* __restrict__ gcol = reinterpret_cast<const G*>(a.gcol);
  T* __restrict__ goff = reinterpret_cast<T*>(a.goffset);
  T* __restrict__ gmsk = reinterpret_cast<T*>(a.gmask);
  const int warp0 = (int)((blockIdx.x * kThreads + threadIdx.x) >> 5);
  const int nwarps = (int)((gridDim.x * kThreads) >> 5);

  for (int item = warp0; item < nitems; item += nwarps) {
    const int pg = item / nTG;
    const int tg = item - pg * nTG;
    const int t = tg / P.dg, g = tg - t * P.dg;
    const int pix = a.pix0 + pg * 4 + lp;
    const bool pv = pix < pend;
    const int b = pv ? pix / HoWo : 0;
    const int p = pv ? pix - b * HoWo : 0;
    // sampling geometry (reference validity rule -1 < h < H, -1 < w < W)
    float lh = 0.f, lw = 0.f, m = 0.f;
    int gidx = 0;
    uint32_t cval = 0u;
    const int obase = ((b * P.dg + g) * 2 * P.K2 + 2 * t) * HoWo + p;
    const int mbase = ((b * P.dg + g) * P.K2 + t) * HoWo + p;
    if (pv) {
      const int i = t / P.kw, j = t - i * P.kw;
      const int ho = p / P.Wo, wo = p - ho * P.Wo;
      const float h = (float)(ho * P.sh - P.ph + i * P.dh) + ldf(off + obase);
      const float w = (float)(wo * P.sw - P.pw + j * P.dw) + ldf(off + obase + HoWo);
      m = ldf(msk + mbase);
      const float hf = floorf(h), wf = floorf(w);
      const int hl = (int)hf, wl = (int)wf;
      lh = h - hf;
      lw = w - wf;
      if ((h > -1.f) && (w > -1.f) && (h < (float)P.H) && (w < (float)P.W) && !(a.dbg & 1)) {
        const bool r0 = hl >= 0, r1 = hl + 1 <= P.H - 1, c0 = wl >= 0, c1 = wl + 1 <= P.W - 1;
        cval = (r0 && c0 ? 1u : 0u) | (r0 && c1 ? 2u : 0u) | (r1 && c0 ? 4u : 0u) |
               (r1 && c1 ? 8u : 0u);
        gidx = b * HW + hl * P.W + wl;
      }
    }
    const float hh = 1.f - lh, hw = 1.f - lw;
    const float bw[4] = {(cval & 1u) ? hh * hw : 0.f, (cval & 2u) ? hh * lw : 0.f,
                         (cval & 4u) ? lh * hw : 0.f, (cval & 8u) ? lh * lw : 0.f};
    const int d[4] = {0, 1, P.W, P.W + 1};
    float S[4] = {0.f, 0.f, 0.f, 0.f};
    if (cval != 0u) {
      const G* grow = gcol + (size_t)(unsigned)(pix - a.pix0) * rowlen + tg * P.Cgp + q * 8;
      for (int cb = 0; cb < P.nCB; ++cb) {
        const int cofs = g * P.Cgp + cb * kChunk;
        // gcol slice and the four corner slices, all loads issued first
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
#pragma unroll
          for (int e = 0; e < 8; ++e) S[c] = fmaf(gc[e], v[e], S[c]);
        }
        if (!(a.dbg & 2)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (cval & (1u << c)) {
              const float sk = bw[c] * m;
              float* dst = a.gx_nhwc + (size_t)(unsigned)((gidx + d[c]) * P.CS + cofs + 4 * q);
              red_add_v4(dst, gc[0] * sk, gc[1] * sk, gc[2] * sk, gc[3] * sk);
              red_add_v4(dst + 32, gc[4] * sk, gc[5] * sk, gc[6] * sk, gc[7] * sk);
            }
          }
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
    if (q == 0 && pv) {
      goff[obase] = Elem<T>::from_f(ah * m);
      goff[obase + HoWo] = Elem<T>::from_f(aw * m);
      gmsk[mbase] = Elem<T>::from_f(am);
    }
  }
}

}  // namespace

int launch_backward_scatter(const BwdDataArgs& a, cudaStream_t stream) {
  const Plan& P = a.plan;
  const long long nitems = (long long)(a.npix + 3) / 4 * (P.K2 * P.dg);
  long long blocks = (nitems + 7) / 8;
  const long long cap = (long long)a.num_sms * 16;
  if (blocks > cap) blocks = cap;
  if (blocks <= 0) return DCN_OK;
  switch (P.dtype) {
    case DCN_F32:
      dcn_bwd_scatter_kernel<float><<<(int)blocks, kThreads, 0, stream>>>(a);
      break;
    case DCN_F16:
      dcn_bwd_scatter_kernel<__half><<<(int)blocks, kThreads, 0, stream>>>(a);
      break;
    default:
      dcn_bwd_scatter_kernel<__nv_bfloat16><<<(int)blocks, kThreads, 0, stream>>>(a);
      break;
  }
  return cudaGetLastError() == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

}  // namespace dcn
