// grad_output tile loads shared by the two backward kernels.
#pragma once
#include "dcn_common.cuh"
#include "dcn_plan.h"

namespace dcn {

// Loads grad_output[b, co, p] for the 8 consecutive flat pixels pix0..pix0+7
// (flat pixel = b*HoWo + p) as floats; zero outside the tensor.  `vec` allows one
// 16-byte load (two for f32): valid when HoWo % 8 == 0, pix0 % 8 == 0 and the
// tensor is 16-byte aligned, so the 8 pixels lie in one image and one line.
template <typename T>
__device__ __forceinline__ void load8_gout(const T* __restrict__ gout, const Plan& P,
                                           int pix0, int co, bool vec, float (&v)[8]) {
  if (co >= P.Co || pix0 >= P.totalP) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
    return;
  }
  if (vec) {
    const int b = fdiv(pix0, P.fd_howo);
    const int p = (int)(pix0 - b * P.HoWo);
    const T* src = gout + ((size_t)b * P.Co + co) * P.HoWo + p;
    if constexpr (std::is_same<T, float>::value) {
      const uint4 a = ldg_nc_v4(src), c = ldg_nc_v4(src + 4);
      v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
      v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
      v[4] = __uint_as_float(c.x); v[5] = __uint_as_float(c.y);
      v[6] = __uint_as_float(c.z); v[7] = __uint_as_float(c.w);
    } else {
      unpack8<T>(ldg_nc_v4(src), v);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int pix = pix0 + e;
      v[e] = 0.f;
      if (pix < P.totalP) {
        const int b = fdiv(pix, P.fd_howo);
        const int p = (int)(pix - b * P.HoWo);
        v[e] = ldf(gout + ((size_t)b * P.Co + co) * P.HoWo + p);
      }
    }
  }
}

// Raw 16-byte loads of 8 consecutive flat pixels of one grad_output row (the
// vector path of load8_gout), issued without consuming the result so several
// can be in flight; zero outside the tensor.
template <typename T>
struct GoutRaw {
  uint4 r[sizeof(T) / 2];
};

__device__ __forceinline__ uint4 ldg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T>
__device__ __forceinline__ void gout_raw_load(const T* __restrict__ gout, const Plan& P,
                                              int pix0, int co, GoutRaw<T>& g, bool plain = false) {
  if (co >= P.Co || pix0 >= P.totalP) {
#pragma unroll
    for (int k = 0; k < (int)(sizeof(T) / 2); ++k) g.r[k] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const int b = fdiv(pix0, P.fd_howo);
  const int p = (int)(pix0 - b * P.HoWo);
  const T* src = gout + ((size_t)b * P.Co + co) * P.HoWo + p;
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 2); ++k) g.r[k] = plain ? ldg_v4(src + k * 4) : ldg_nc_v4(src + k * 4);
}

template <typename T>
__device__ __forceinline__ void gout_raw_to_f(const GoutRaw<T>& g, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    v[0] = __uint_as_float(g.r[0].x); v[1] = __uint_as_float(g.r[0].y);
    v[2] = __uint_as_float(g.r[0].z); v[3] = __uint_as_float(g.r[0].w);
    v[4] = __uint_as_float(g.r[1].x); v[5] = __uint_as_float(g.r[1].y);
    v[6] = __uint_as_float(g.r[1].z); v[7] = __uint_as_float(g.r[1].w);
  } else {
    unpack8<T>(g.r[0], v);
  }
}

// Stores 8 floats as one 16-byte operand chunk at shared address `addr`
// (and the bf16 lo part at addr + lo_ofs for the f32 split).
template <typename T>
__device__ __forceinline__ void store8_op(uint32_t addr, uint32_t lo_ofs, const float (&v)[8]) {
  if constexpr (OpOf<T>::kSplit) {
    uint4 hi, lo;
    split2(v[0], v[1], hi.x, lo.x);
    split2(v[2], v[3], hi.y, lo.y);
    split2(v[4], v[5], hi.z, lo.z);
    split2(v[6], v[7], hi.w, lo.w);
    sts_v4(addr, hi);
    sts_v4(addr + lo_ofs, lo);
  } else {
    constexpr int kBF = OpOf<T>::kBF16;
    uint4 u;
    u.x = pack2<kBF>(v[0], v[1]);
    u.y = pack2<kBF>(v[2], v[3]);
    u.z = pack2<kBF>(v[4], v[5]);
    u.w = pack2<kBF>(v[6], v[7]);
    sts_v4(addr, u);
  }
}

}  // namespace dcn
