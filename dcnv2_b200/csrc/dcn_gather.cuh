// Bilinear gather of 32 channels and its store into a 128B-swizzled operand
// row, shared by the forward and the backward-weight kernels.
#pragma once
#include "dcn_common.cuh"

namespace dcn {

// Blends 32 channels at 4 corners: acc[c] = sum_i cw[i] * corner_i[c].
template <typename T>
__device__ __forceinline__ void gather32(const T* __restrict__ xb, const Sample& s, int cofs,
                                         int CS, float (&acc)[32]) {
#pragma unroll
  for (int c = 0; c < 32; ++c) acc[c] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (s.cw[i] != 0.f) {
      const T* src = xb + (size_t)s.cidx[i] * CS + cofs;
      if constexpr (std::is_same<T, float>::value) {
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = ldg_nc_v4(src + 4 * q);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          acc[4 * q + 0] = fmaf(s.cw[i], __uint_as_float(v[q].x), acc[4 * q + 0]);
          acc[4 * q + 1] = fmaf(s.cw[i], __uint_as_float(v[q].y), acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(s.cw[i], __uint_as_float(v[q].z), acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(s.cw[i], __uint_as_float(v[q].w), acc[4 * q + 3]);
        }
      } else {
        uint4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = ldg_nc_v4(src + 8 * q);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
          unpack8<T>(v[q], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[8 * q + e] = fmaf(s.cw[i], f[e], acc[8 * q + e]);
        }
      }
    }
  }
}

// Writes 32 blended channels as four 16-byte chunks (chunk0..chunk0+3) of row r
// of a SW128 K-major tile (and its lo twin at +lo_ofs for the f32 split).
template <typename T>
__device__ __forceinline__ void store_row32(uint32_t tile, uint32_t lo_ofs, int r, int chunk0,
                                            const float (&acc)[32]) {
  constexpr int kBF = OpOf<T>::kBF16;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t off = sw128_off(r, chunk0 + q);
    if constexpr (OpOf<T>::kSplit) {
      uint4 hi, lo;
      split2(acc[8 * q + 0], acc[8 * q + 1], hi.x, lo.x);
      split2(acc[8 * q + 2], acc[8 * q + 3], hi.y, lo.y);
      split2(acc[8 * q + 4], acc[8 * q + 5], hi.z, lo.z);
      split2(acc[8 * q + 6], acc[8 * q + 7], hi.w, lo.w);
      sts_v4(tile + off, hi);
      sts_v4(tile + lo_ofs + off, lo);
    } else {
      uint4 v;
      v.x = pack2<kBF>(acc[8 * q + 0], acc[8 * q + 1]);
      v.y = pack2<kBF>(acc[8 * q + 2], acc[8 * q + 3]);
      v.z = pack2<kBF>(acc[8 * q + 4], acc[8 * q + 5]);
      v.w = pack2<kBF>(acc[8 * q + 6], acc[8 * q + 7]);
      sts_v4(tile + off, v);
    }
  }
}

}  // namespace dcn
