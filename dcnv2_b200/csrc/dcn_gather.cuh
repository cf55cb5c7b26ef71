// Coalesced bilinear gather shared by the forward and backward kernels.
//
// The packed input is channels-last, so one bilinear corner of a 64-channel
// block is one contiguous 128-byte line (bf16/f16) or 256 bytes (f32).  A warp
// processes 4 pixels at a time with 8 lanes per pixel: each lane owns 8
// channels (a 16-byte slice, 32 bytes for f32) of every corner line, so every
// warp-wide load touches only 4 lines (8 for f32) and the blended slice is
// exactly one 16-byte chunk of the pixel's swizzled operand row.
#pragma once
#include "dcn_common.cuh"

namespace dcn {

template <typename T>
struct GatherShape {
  static constexpr int kLPP = 8;                  // lanes per pixel
  static constexpr int kCPL = 8;                  // channels per lane
  static constexpr int kPPI = 4;                  // pixels per warp iteration
  static constexpr int kLD = (int)sizeof(T) / 2;  // 16-byte loads per corner slice
};

// Compact sampling geometry of one (pixel, tap, group): index of the top-left
// corner (hl*W + wl) and the four corner weights times the mask, zero for
// corners outside the image or when the sample itself is outside
// (-1 < h < H, -1 < w < W; reference com.cu:119-148, 187).
struct Geo {
  int base;
  float w[4];
};

__device__ __forceinline__ Geo make_geo(float h, float w, float m, int H, int W) {
  Geo g;
  const float hf = floorf(h), wf = floorf(w);
  const int hl = (int)hf, wl = (int)wf;
  const float lh = h - hf, lw = w - wf, hh = 1.f - lh, hw = 1.f - lw;
  const bool inside = (h > -1.f) && (w > -1.f) && (h < (float)H) && (w < (float)W);
  const bool r0 = inside && hl >= 0, r1 = inside && hl + 1 <= H - 1;
  const bool c0 = wl >= 0, c1 = wl + 1 <= W - 1;
  g.w[0] = (r0 && c0) ? hh * hw * m : 0.f;
  g.w[1] = (r0 && c1) ? hh * lw * m : 0.f;
  g.w[2] = (r1 && c0) ? lh * hw * m : 0.f;
  g.w[3] = (r1 && c1) ? lh * lw * m : 0.f;
  g.base = inside ? hl * W + wl : 0;
  return g;
}

__device__ __forceinline__ Geo zero_geo() {
  Geo g;
  g.base = 0;
  g.w[0] = g.w[1] = g.w[2] = g.w[3] = 0.f;
  return g;
}

// Raw corner slices of one lane (8 channels: one 16-byte load, two for f32):
// corner i at xrow + (base + d_i) * CS, d = {0, 1, W, W + 1}; slices of
// zero-weight corners are not loaded.
template <typename T>
__device__ __forceinline__ void load_corners(const T* __restrict__ xrow, const Geo& g, int W,
                                             int CS, uint4 (&v)[4][GatherShape<T>::kLD]) {
  constexpr int LD = GatherShape<T>::kLD;
  const int d[4] = {0, 1, W, W + 1};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int k = 0; k < LD; ++k) {
      v[i][k] = (g.w[i] != 0.f) ? ldg_nc_v4(xrow + (size_t)(g.base + d[i]) * CS + k * (8 / LD))
                                : make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Unpacks one lane's 8-channel corner slice to floats.
template <typename T>
__device__ __forceinline__ void unpack_slice(const uint4 (&v)[GatherShape<T>::kLD], float (&f)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    f[0] = __uint_as_float(v[0].x); f[1] = __uint_as_float(v[0].y);
    f[2] = __uint_as_float(v[0].z); f[3] = __uint_as_float(v[0].w);
    f[4] = __uint_as_float(v[1].x); f[5] = __uint_as_float(v[1].y);
    f[6] = __uint_as_float(v[1].z); f[7] = __uint_as_float(v[1].w);
  } else {
    unpack8<T>(v[0], f);
  }
}

// Blends the loaded corner slices: out[c] = sum_i w_i * corner_i[c].
template <typename T>
__device__ __forceinline__ void blend_corners(const uint4 (&v)[4][GatherShape<T>::kLD],
                                              const Geo& g, float (&out)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) out[c] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float f[8];
    unpack_slice<T>(v[i], f);
#pragma unroll
    for (int c = 0; c < 8; ++c) out[c] = fmaf(g.w[i], f[c], out[c]);
  }
}

// Stores a lane's 8 blended channels as 16-byte chunk q of row `row` of a SW128
// operand tile (128-byte rows of 64 16-bit elements); for f32 the bf16 hi part
// goes to the tile and the lo part to the twin tile at +lo_ofs.
template <typename T>
__device__ __forceinline__ void store_slice(uint32_t tile, uint32_t lo_ofs, int row, int q,
                                            const float (&s)[8]) {
  const uint32_t off = sw128_off(row, q);
  if constexpr (std::is_same<T, float>::value) {
    uint4 hi, lo;
    split2(s[0], s[1], hi.x, lo.x);
    split2(s[2], s[3], hi.y, lo.y);
    split2(s[4], s[5], hi.z, lo.z);
    split2(s[6], s[7], hi.w, lo.w);
    sts_v4(tile + off, hi);
    sts_v4(tile + lo_ofs + off, lo);
  } else {
    constexpr int kBF = OpOf<T>::kBF16;
    uint4 u;
    u.x = pack2<kBF>(s[0], s[1]);
    u.y = pack2<kBF>(s[2], s[3]);
    u.z = pack2<kBF>(s[4], s[5]);
    u.w = pack2<kBF>(s[6], s[7]);
    sts_v4(tile + off, u);
  }
}

// Geometry of one pixel row computed by a single lane and broadcast to the 8
// lanes that gather it: gidx = index of the top-left corner pixel in the packed
// input (b*H*W + hl*W + wl), w = corner weights times the mask (0 = skipped).
struct PixGeo {
  int gidx;
  float w[4];
};

__device__ __forceinline__ PixGeo make_pixgeo(int img_base, float h, float w, float m, int H, int W) {
  const Geo g = make_geo(h, w, m, H, W);
  PixGeo r;
  r.gidx = img_base + g.base;
  r.w[0] = g.w[0];
  r.w[1] = g.w[1];
  r.w[2] = g.w[2];
  r.w[3] = g.w[3];
  return r;
}

// As make_pixgeo, but with the 2 x 2 corner block moved inside the image: the
// block's top-left corner is clamped to row 0 .. max(H-2, 0) and column
// 0 .. max(W-2, 0) and the weights of the corners that lie inside the image are
// carried over to their place in the moved block (a corner outside the image
// has weight 0 already).  All four corner lines of the block are then inside the
// image (rows r and r + (H > 1), columns c and c + (W > 1)), so they can be
// loaded without a per-corner test; the blend is unchanged.
__device__ __forceinline__ PixGeo make_pixgeo_clamped(int img_base, float h, float w, float m, int H, int W) {
  const Geo g = make_geo(h, w, m, H, W);
  const float hf = floorf(h), wf = floorf(w);
  const int hl = (int)hf, wl = (int)wf;
  const int r = min(max(hl, 0), max(H - 2, 0));
  const int c = min(max(wl, 0), max(W - 2, 0));
  const int sy = hl - r, sx = wl - c;   // -1, 0 or 1 whenever a weight is non-zero
  // rows: (top, bottom) pairs of the original block -> moved block
  float t0 = g.w[0], t1 = g.w[1], b0 = g.w[2], b1 = g.w[3];
  if (sy < 0) { t0 = b0; t1 = b1; b0 = 0.f; b1 = 0.f; }
  else if (sy > 0) { b0 = t0; b1 = t1; t0 = 0.f; t1 = 0.f; }
  // columns: (left, right) of each row
  if (sx < 0) { t0 = t1; b0 = b1; t1 = 0.f; b1 = 0.f; }
  else if (sx > 0) { t1 = t0; b1 = b0; t0 = 0.f; b0 = 0.f; }
  PixGeo out;
  out.gidx = img_base + r * W + c;
  out.w[0] = t0;
  out.w[1] = t1;
  out.w[2] = b0;
  out.w[3] = b1;
  return out;
}

// Loads one lane's 8-channel slices of a clamped 2 x 2 block (no tests):
// corner i at p0 + {0, dx, dy, dy + dx} elements, p0 = the lane's top-left slice.
template <typename T>
__device__ __forceinline__ void load_block(const T* __restrict__ p0, size_t dx, size_t dy,
                                           uint4 (&v)[4][GatherShape<T>::kLD]) {
  constexpr int LD = GatherShape<T>::kLD;
  const T* p[4] = {p0, p0 + dx, p0 + dy, p0 + dy + dx};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < LD; ++k) v[i][k] = ldg_nc_v4(p[i] + k * (8 / LD));
}

__device__ __forceinline__ PixGeo zero_pixgeo() {
  PixGeo r;
  r.gidx = 0;
  r.w[0] = r.w[1] = r.w[2] = r.w[3] = 0.f;
  return r;
}

__device__ __forceinline__ PixGeo shfl_pixgeo(const PixGeo& g, int src) {
  PixGeo r;
  r.gidx = __shfl_sync(0xffffffffu, g.gidx, src);
#pragma unroll
  for (int i = 0; i < 4; ++i) r.w[i] = __shfl_sync(0xffffffffu, g.w[i], src);
  return r;
}

// Loads one lane's 8-channel slices of the 4 corners (pixel strides CS):
// corner i at xt + (gidx + d_i) * CS + cofs, d = {0, 1, W, W + 1}.
template <typename T>
__device__ __forceinline__ void load_corners_px(const T* __restrict__ xt, const PixGeo& g, int W,
                                                int CS, int cofs,
                                                uint4 (&v)[4][GatherShape<T>::kLD]) {
  constexpr int LD = GatherShape<T>::kLD;
  const int d[4] = {0, 1, W, W + 1};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T* p = xt + ((size_t)(unsigned)((g.gidx + d[i]) * CS + cofs));
#pragma unroll
    for (int k = 0; k < LD; ++k)
      v[i][k] = (g.w[i] != 0.f) ? ldg_nc_v4(p + k * (8 / LD)) : make_uint4(0u, 0u, 0u, 0u);
  }
}

// Blend for 16-bit inputs: 8 channels of the four corners, each sample formed
// in fp32 (two channels per packed f32x2 FMA, weights x mask in fp32) and
// rounded once to the operand format, as the reference forms the sample in
// float and rounds it once (com.cu:83-87, 119-148).
template <typename T>
__device__ __forceinline__ uint4 blend_packed(const uint4 (&v)[4][1], const float (&w)[4]) {
  float2 acc[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) acc[c] = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t in[4] = {v[i][0].x, v[i][0].y, v[i][0].z, v[i][0].w};
    const float2 wi = make_float2(w[i], w[i]);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float2 x;
      if constexpr (std::is_same<T, __half>::value) {
        x = __half22float2(*reinterpret_cast<const __half2*>(&in[c]));
      } else {
        x = make_float2(__uint_as_float(in[c] << 16), __uint_as_float(in[c] & 0xffff0000u));
      }
      acc[c] = __ffma2_rn(x, wi, acc[c]);
    }
  }
  constexpr int kBF = std::is_same<T, __half>::value ? 0 : 1;
  return make_uint4(pack2<kBF>(acc[0].x, acc[0].y), pack2<kBF>(acc[1].x, acc[1].y),
                    pack2<kBF>(acc[2].x, acc[2].y), pack2<kBF>(acc[3].x, acc[3].y));
}

// Blends and stores one lane's slice (packed math for 16-bit inputs, f32 math
// and a bf16 hi/lo split for f32 inputs).
template <typename T>
__device__ __forceinline__ void blend_store(const uint4 (&v)[4][GatherShape<T>::kLD], const PixGeo& g,
                                            uint32_t tile, uint32_t lo_ofs, int row, int q) {
  if constexpr (std::is_same<T, float>::value) {
    Geo gg;
    gg.base = 0;
    gg.w[0] = g.w[0]; gg.w[1] = g.w[1]; gg.w[2] = g.w[2]; gg.w[3] = g.w[3];
    float sl[8];
    blend_corners<T>(v, gg, sl);
    store_slice<T>(tile, lo_ofs, row, q, sl);
  } else {
    sts_v4(tile + sw128_off(row, q), blend_packed<T>(v, g.w));
  }
}

}  // namespace dcn
