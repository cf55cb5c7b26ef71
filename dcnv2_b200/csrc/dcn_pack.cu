// Layout kernels around the tensor-core kernels:
//  * input NCHW -> channels-last, group-padded [B][H][W][dg][Cgp] so one
//    bilinear corner of 64 channels is one 128-byte (bf16) line;
//  * weight -> pre-swizzled UMMA operand tiles, so one bulk copy per pipeline
//    stage lands a ready-to-use 128B-swizzled tile in shared memory;
//  * fp32 gradient accumulators -> the caller's layouts and element type.
#include "dcn_common.cuh"
#include "dcn_gout.cuh"
#include "dcn_kernels.h"

namespace dcn {

namespace {

// [B][C][H*W] -> [B][H*W][dg][Cgp] (channel order of perm_logical inside each
// 64-channel block); padded channels are written as zero.  A CTA moves 64-pixel
// x 64-channel blocks in a grid-stride loop: 16-byte loads along pixels (when
// `vec`: H*W % 8 == 0 and x 16-byte aligned), 16-byte stores along channels;
// the next block's loads are issued before the current block is stored.
template <typename T>
__global__ void __launch_bounds__(256) pack_input_kernel(const T* __restrict__ x,
                                                         T* __restrict__ xt, int C, int HW,
                                                         int Cg, int Cgp, int CS, int vec,
                                                         int npb, int ncb, int nblocks) {
  pdl_wait();
  constexpr int EPV = 16 / (int)sizeof(T);           // elements per 16-byte vector
  constexpr int kItems = 64 * (64 / EPV) / 256;       // 16-byte loads per thread and block
  __shared__ __align__(16) T tile[64][64 + EPV];      // [channel][pixel]
  const int tid = threadIdx.x;
  uint4 raw[kItems];
  auto issue = [&](int blk) {
    if (!vec || blk >= nblocks) return;
    const int pbk = blk % npb, rest = blk / npb;
    const int d0 = (rest % ncb) * 64, b = rest / ncb;
    const int g = d0 / Cgp, cb = d0 - g * Cgp;
    const T* xb = x + (size_t)b * C * HW;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int item = tid + 256 * k;
      const int c = item / (64 / EPV), pv = item - c * (64 / EPV);
      const int cc = cb + c, p = pbk * 64 + pv * EPV;
      raw[k] = (cc < Cg && p + EPV <= HW) ? ldg_nc_v4(xb + (size_t)(g * Cg + cc) * HW + p)
                                          : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  issue(blockIdx.x);
  for (int blk = blockIdx.x; blk < nblocks; blk += gridDim.x) {
    const int pbk = blk % npb, rest = blk / npb;
    const int d0 = (rest % ncb) * 64, b = rest / ncb;
    const int p0 = pbk * 64;
    const int g = d0 / Cgp, cb = d0 - g * Cgp;
    const T* xb = x + (size_t)b * C * HW;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int item = tid + 256 * k;
      const int c = item / (64 / EPV), pv = item - c * (64 / EPV);
      const int cc = cb + c, p = p0 + pv * EPV;
      T* dst = &tile[c][pv * EPV];
      if (vec && (cc >= Cg || p + EPV <= HW)) {
        *reinterpret_cast<uint4*>(dst) = raw[k];
      } else {
        for (int e = 0; e < EPV; ++e)
          dst[e] = (cc < Cg && p + e < HW) ? xb[(size_t)(g * Cg + cc) * HW + p + e] : Elem<T>::from_f(0.f);
      }
    }
    issue(blk + gridDim.x);
    __syncthreads();
    T* xo = xt + (size_t)b * HW * CS + d0;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
      const int item = tid + 256 * k;
      const int pl = item / (64 / EPV), cv = item - pl * (64 / EPV);
      const int p = p0 + pl;
      if (p >= HW) continue;
      alignas(16) T v[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) v[e] = tile[perm_logical(cv * EPV + e)][pl];
      *reinterpret_cast<uint4*>(xo + (size_t)p * CS + cv * EPV) = *reinterpret_cast<const uint4*>(v);
    }
  }
}

// Writes 8 consecutive K elements (one 16-byte chunk) of a UMMA operand row.
// hi/lo pair for the f32 split, else the 16-bit operand type.
template <typename T>
__device__ __forceinline__ void write_chunk(uint8_t* tile, size_t lo_ofs, int row, int chunk,
                                            const float (&v)[8]) {
  const uint32_t off = sw128_off(row, chunk);
  if constexpr (OpOf<T>::kSplit) {
    uint4 hi, lo;
    split2(v[0], v[1], hi.x, lo.x);
    split2(v[2], v[3], hi.y, lo.y);
    split2(v[4], v[5], hi.z, lo.z);
    split2(v[6], v[7], hi.w, lo.w);
    *reinterpret_cast<uint4*>(tile + off) = hi;
    *reinterpret_cast<uint4*>(tile + lo_ofs + off) = lo;
  } else {
    constexpr int kBF = OpOf<T>::kBF16;
    uint4 u;
    u.x = pack2<kBF>(v[0], v[1]);
    u.y = pack2<kBF>(v[2], v[3]);
    u.z = pack2<kBF>(v[4], v[5]);
    u.w = pack2<kBF>(v[6], v[7]);
    *reinterpret_cast<uint4*>(tile + off) = u;
  }
}

// Forward B operand: tile (ct, kc) holds rows co = ct*NT + r, K elements
// (t, g, cb*64 + e) of W[co][g*Cg + cb*64 + e][t].  One thread per 16-byte chunk.
template <typename T>
__device__ __forceinline__ void pack_weight_fwd_part(const T* __restrict__ w, uint8_t* __restrict__ wpk,
                                                     const Plan& P, int vb, int vg) {
  const long long nchunks = (long long)P.nCoT * P.nK * P.NT * 8;
  for (long long idx = vb * (long long)blockDim.x + threadIdx.x; idx < nchunks;
       idx += (long long)vg * blockDim.x) {
    const int chunk = (int)(idx & 7);
    const long long rt = idx >> 3;
    const int r = (int)(rt % P.NT);
    const long long tk = rt / P.NT;
    const int kc = (int)(tk % P.nK);
    const int ct = (int)(tk / P.nK);
    const int t = kc / (P.dg * P.nCB);
    const int rem = kc - t * (P.dg * P.nCB);
    const int g = rem / P.nCB, cb = rem - g * P.nCB;
    const int co = ct * P.NT + r;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int cc = cb * kChunk + perm_logical(chunk * 8 + e);
      v[e] = (co < P.Co && cc < P.Cg)
                 ? ldf(w + ((size_t)co * P.C + g * P.Cg + cc) * P.K2 + t)
                 : 0.f;
    }
    uint8_t* tile = wpk + (size_t)(ct * P.nK + kc) * P.wf_tile_bytes;
    write_chunk<T>(tile, (size_t)P.NT * 128, r, chunk, v);
  }
}

template <typename T>
__global__ void pack_weight_fwd_kernel(const T* __restrict__ w, uint8_t* __restrict__ wpk,
                                       const Plan P) {
  pdl_wait();
  pack_weight_fwd_part<T>(w, wpk, P, blockIdx.x, gridDim.x);
}

// Backward-data B operand (W transposed): tile (u, ko) of unit u = (set, cch)
// holds rows n = j*NC + nn for the gT (tap, group)s tg = set*gT + j of the set,
// channel cc = cch*NC + nn (packed order inside 64-channel blocks), and K
// elements co = ko*64 + e; rows of (tap, group)s past the end are zero.
// `zacc` (nz4 float4s, may be null) is zeroed on the side: the weight-gradient
// accumulators.
template <typename T>
__global__ void pack_weight_bwd_kernel(const T* __restrict__ w, uint8_t* __restrict__ wpk,
                                       const Plan P, float4* __restrict__ zacc, long long nz4,
                                       int* __restrict__ status) {
  pdl_wait();
  if (status != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *status = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nz4;
       i += (long long)gridDim.x * blockDim.x)
    zacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  const long long nchunks = (long long)P.gnU * P.nKo * P.gNC * 8;
  const int nTG = P.K2 * P.dg;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < nchunks;
       idx += (long long)gridDim.x * blockDim.x) {
    const int chunk = (int)(idx & 7);
    const long long rt = idx >> 3;
    const int n = (int)(rt % P.gNC);
    const long long uk = rt / P.gNC;
    const int ko = (int)(uk % P.nKo);
    const int u = (int)(uk / P.nKo);
    const int set = u / P.nCC, cch = u - set * P.nCC;
    const int j = n / P.NC, nn = n - j * P.NC;
    const int tg = set * P.gT + j;
    const int t = tg / P.dg, g = tg - t * P.dg;
    const int cc = cch * P.NC + (nn & ~63) + perm_logical(nn & 63);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int co = ko * kChunk + chunk * 8 + e;
      v[e] = (tg < nTG && co < P.Co && cc < P.Cg)
                 ? ldf(w + ((size_t)co * P.C + g * P.Cg + cc) * P.K2 + t)
                 : 0.f;
    }
    uint8_t* tile = wpk + (size_t)(u * P.nKo + ko) * P.wd_tile_bytes;
    write_chunk<T>(tile, (size_t)P.gNC * 128, n, chunk, v);
  }
}

// grad_output NCHW -> operand blocks: block (pixel block pb of 64 flat pixels,
// Co chunk ko of 64) is 64 rows (pixels) x 64 Co in the operand type, rows of
// 128 bytes with the 128-byte swizzle (f32: bf16 hi block then lo block).  The
// same bytes serve as the K-major A operand of the backward-data GEMM (M =
// pixels, K = Co) and the MN-major A operand of the backward-weight GEMM (M = Co,
// K = pixels).  grad_bias partial sums (over the pixels this CTA visits) are
// added to the fp32 accumulator `gb` when it is not null.
template <typename T>
__global__ void __launch_bounds__(256) pack_gout_kernel(const T* __restrict__ gout,
                                                        uint8_t* __restrict__ gpk,
                                                        float* __restrict__ gb, const Plan P,
                                                        int vec) {
  pdl_wait();
  __shared__ float tile[64][65];
  const int ko = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int nPB = (int)((P.totalP + 63) / 64);
  const size_t blk_bytes = (size_t)P.nsplit * 8192;
  float bsum[2] = {0.f, 0.f};
  // the next block's grad_output rows are loaded while this block is stored
  GoutRaw<T> raw[2];
  auto issue = [&](int pb) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = tid + 256 * k;
      if (vec && pb < nPB) gout_raw_load<T>(gout, P, pb * 64 + (item & 7) * 8, ko * kChunk + (item >> 3), raw[k]);
    }
  };
  issue(blockIdx.x);
  for (int pb = blockIdx.x; pb < nPB; pb += gridDim.x) {
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = tid + 256 * k;
      const int col = item >> 3, ch = item & 7;   // Co row within the chunk, 8-pixel group
      float v[8];
      const int co = ko * kChunk + col;
      if (vec) {
        gout_raw_to_f<T>(raw[k], v);
      } else {
        load8_gout<T>(gout, P, pb * 64 + ch * 8, co, false, v);
      }
      bsum[k] += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
#pragma unroll
      for (int e = 0; e < 8; ++e) tile[col][ch * 8 + e] = v[e];
    }
    issue(pb + gridDim.x);
    __syncthreads();
    uint8_t* blk = gpk + ((size_t)pb * P.nKo + ko) * blk_bytes;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = tid + 256 * k;
      const int row = item >> 3, c = item & 7;    // pixel row, 16-byte chunk (8 Co)
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = tile[c * 8 + e][row];
      const uint32_t off = sw128_off(row, c);
      if constexpr (OpOf<T>::kSplit) {
        uint4 hi, lo;
        split2(v[0], v[1], hi.x, lo.x);
        split2(v[2], v[3], hi.y, lo.y);
        split2(v[4], v[5], hi.z, lo.z);
        split2(v[6], v[7], hi.w, lo.w);
        *reinterpret_cast<uint4*>(blk + off) = hi;
        *reinterpret_cast<uint4*>(blk + 8192 + off) = lo;
      } else {
        constexpr int kBF = OpOf<T>::kBF16;
        uint4 u;
        u.x = pack2<kBF>(v[0], v[1]);
        u.y = pack2<kBF>(v[2], v[3]);
        u.z = pack2<kBF>(v[4], v[5]);
        u.w = pack2<kBF>(v[6], v[7]);
        *reinterpret_cast<uint4*>(blk + off) = u;
      }
    }
  }
  if (gb != nullptr) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float s = bsum[k];
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      s += __shfl_xor_sync(0xffffffffu, s, 4);
      const int co = ko * kChunk + ((tid + 256 * k) >> 3);
      if ((lane & 7) == 0 && co < P.Co) atomicAdd(gb + co, s);
    }
  }
}

// fp32 [B][H*W][dg][Cgp] -> T [B][C][H*W].  One CTA of 256 threads moves 64
// pixels x 64 channels of one group block: 16-byte loads along channels, 16-byte stores
// along pixels (when `vec`: H*W % 8 == 0 and gx 16-byte aligned).
template <typename T>
__device__ __forceinline__ void finish_grad_input_block(const float* __restrict__ gxn, T* __restrict__ gx, int C,
                                                        int HW, int Cg, int Cgp, int CS, int vec, int bx, int by,
                                                        int bz, float (&tile)[64][65]) {
  constexpr int EPV = 16 / (int)sizeof(T);
  const int b = bz;
  const int d0 = by * 64;
  const int p0 = bx * 64;
  const int g = d0 / Cgp, cb = d0 - g * Cgp;
  const float* src = gxn + (size_t)b * HW * CS + d0;
  const int tid = threadIdx.x;
  // 256 threads: each loads its four 16-byte pieces before storing any, so the
  // four loads are in flight together
  float4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int item = tid + 256 * k;
    const int p = p0 + (item >> 4);
    v[k] = p < HW ? *reinterpret_cast<const float4*>(src + (size_t)p * CS + (item & 15) * 4)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int item = tid + 256 * k;
    const int pl = item >> 4, cv = item & 15;
    tile[pl][cv * 4 + 0] = v[k].x;
    tile[pl][cv * 4 + 1] = v[k].y;
    tile[pl][cv * 4 + 2] = v[k].z;
    tile[pl][cv * 4 + 3] = v[k].w;
  }
  __syncthreads();
  T* dst = gx + (size_t)b * C * HW;
  for (int item = tid; item < 64 * (64 / EPV); item += 256) {
    const int c = item / (64 / EPV), pv = item - c * (64 / EPV);
    const int cc = cb + c;
    if (cc >= Cg) continue;
    const int p = p0 + pv * EPV;
    T* o = dst + (size_t)(g * Cg + cc) * HW + p;
    if (vec && p + EPV <= HW) {
      alignas(16) T v[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) v[e] = Elem<T>::from_f(tile[pv * EPV + e][c]);
      *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(v);
    } else {
      for (int e = 0; e < EPV && p + e < HW; ++e) o[e] = Elem<T>::from_f(tile[pv * EPV + e][c]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) finish_grad_input_kernel(const float* __restrict__ gxn,
                                                                T* __restrict__ gx, int C, int HW,
                                                                int Cg, int Cgp, int CS, int vec) {
  pdl_wait();
  __shared__ float tile[64][65];                      // [pixel][channel]
  finish_grad_input_block<T>(gxn, gx, C, HW, Cg, Cgp, CS, vec, blockIdx.x, blockIdx.y, blockIdx.z, tile);
}

// fp32 [Co][K2][dg][Cgp] -> T [Co][C][K2]; fp32 [Co] -> T [Co]; block vb of vg
template <typename T>
__device__ __forceinline__ void finish_grad_weight_part(const float* __restrict__ gw, const float* __restrict__ gb,
                                                        T* __restrict__ gwo, T* __restrict__ gbo, const Plan& P,
                                                        int vb, int vg) {
  const long long n = (long long)P.Co * P.C * P.K2;
  for (long long idx = vb * (long long)blockDim.x + threadIdx.x; idx < n; idx += (long long)vg * blockDim.x) {
    const int t = (int)(idx % P.K2);
    const long long r = idx / P.K2;
    const int c = (int)(r % P.C);
    const int co = (int)(r / P.C);
    const int g = c / P.Cg, cc = c - g * P.Cg;
    gwo[idx] = Elem<T>::from_f(gw[((size_t)co * P.K2 + t) * P.CS + g * P.Cgp + cc]);
    if (gbo != nullptr && idx < P.Co) gbo[idx] = Elem<T>::from_f(gb[idx]);
  }
}

template <typename T>
__global__ void finish_grad_weight_kernel(const float* __restrict__ gw, const float* __restrict__ gb,
                                          T* __restrict__ gwo, T* __restrict__ gbo, const Plan P) {
  pdl_wait();
  finish_grad_weight_part<T>(gw, gb, gwo, gbo, P, blockIdx.x, gridDim.x);
}

// Both finishing passes in one launch (NCHW): blocks 0 .. nA-1 transpose
// grad_input tiles (block b = (x, y, z) of the separate kernel's grid
// (nx, ny, B), x fastest), the rest convert grad_weight / grad_bias.
template <typename T>
__global__ void __launch_bounds__(256) finish_grads_kernel(const float* __restrict__ gxn, T* __restrict__ gx,
                                                           int vec, int nx, int ny, int nA,
                                                           const float* __restrict__ gw,
                                                           const float* __restrict__ gb, T* __restrict__ gwo,
                                                           T* __restrict__ gbo, const Plan P) {
  pdl_wait();
  __shared__ float tile[64][65];
  const int bid = blockIdx.x;
  if (bid < nA) {
    const int bx = bid % nx, r = bid / nx;
    finish_grad_input_block<T>(gxn, gx, P.C, P.H * P.W, P.Cg, P.Cgp, P.CS, vec, bx, r % ny, r / ny, tile);
  } else {
    finish_grad_weight_part<T>(gw, gb, gwo, gbo, P, bid - nA, (int)gridDim.x - nA);
  }
}

// ---------------------------------------------------------------------------
// Register-transpose input pack for 16-bit tensors (H*W % 8 == 0, 16-byte
// aligned): a thread moves an 8 x 8 block (eight 16-byte loads, 32 byte
// permutes, eight 16-byte stores) without shared memory.

// word k of pixel e of an 8 x 8 16-bit block whose rows 2k, 2k+1 are ra, rb
__device__ __forceinline__ uint32_t tr_word(const uint4& ra, const uint4& rb, int e) {
  const uint32_t wa = e < 2 ? ra.x : e < 4 ? ra.y : e < 6 ? ra.z : ra.w;
  const uint32_t wb = e < 2 ? rb.x : e < 4 ? rb.y : e < 6 ? rb.z : rb.w;
  return __byte_perm(wa, wb, (e & 1) ? 0x7632 : 0x5410);
}

__device__ __forceinline__ void transpose8x8_b16(const uint4 (&row)[8], uint4 (&col)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e)
    col[e] = make_uint4(tr_word(row[0], row[1], e), tr_word(row[2], row[3], e), tr_word(row[4], row[5], e),
                        tr_word(row[6], row[7], e));
}

// x [B][C][HW] -> xt [B][HW][dg][Cgp] (perm_logical order).  Thread: 16-byte
// chunk q of a 64-channel block and 8 pixels; q varies fastest so that the
// eight chunks of a pixel's 128-byte line are stored by one warp instruction.
// When `acc` is not null the fp32 accumulator of the same layout (the backward's
// grad_input sums) is zeroed alongside, and `status` (if not null) is cleared.
template <typename T>
__device__ __forceinline__ void pack_input_rt_part(const T* __restrict__ x, T* __restrict__ xt, int C, int HW,
                                                   int Cg, int Cgp, int CS, long long nthr,
                                                   float* __restrict__ acc, int* __restrict__ status, int vb,
                                                   int vg) {
  const int np8 = HW >> 3, nblk = CS >> 6;
  if (status != nullptr && vb == 0 && threadIdx.x == 0) *status = 0;
  for (long long idx = vb * (long long)blockDim.x + threadIdx.x; idx < nthr; idx += (long long)vg * blockDim.x) {
    const int q = (int)(idx & 7);
    const long long r1 = idx >> 3;
    const int p8 = (int)(r1 % np8);
    const long long r2 = r1 / np8;
    const int blk = (int)(r2 % nblk), b = (int)(r2 / nblk);
    const int d0 = blk * 64, g = d0 / Cgp, cb = d0 - g * Cgp;
    uint4 row[8], col[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int cc = cb + perm_logical(8 * q + r);   // logical channel of position 8q + r
      row[r] = cc < Cg ? ldg_nc_v4(x + ((size_t)b * C + g * Cg + cc) * HW + p8 * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    transpose8x8_b16(row, col);
    const size_t eo = ((size_t)b * HW + p8 * 8) * CS + d0 + q * 8;
    T* o = xt + eo;
#pragma unroll
    for (int e = 0; e < 8; ++e) *reinterpret_cast<uint4*>(o + (size_t)e * CS) = col[e];
    if (acc != nullptr) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float4* a4 = reinterpret_cast<float4*>(acc + eo + (size_t)e * CS);
        a4[0] = z;
        a4[1] = z;
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) pack_input_rt_kernel(const T* __restrict__ x, T* __restrict__ xt,
                                                            int C, int HW, int Cg, int Cgp, int CS,
                                                            long long nthr, float* __restrict__ acc,
                                                            int* __restrict__ status) {
  pdl_wait();
  pack_input_rt_part<T>(x, xt, C, HW, Cg, Cgp, CS, nthr, acc, status, blockIdx.x, gridDim.x);
}

// The forward's input pack (register transpose) and weight pack in one launch:
// blocks 0 .. nA-1 pack the input, the rest the weight tiles.
template <typename T>
__global__ void __launch_bounds__(256) pack_forward_kernel(const T* __restrict__ x, T* __restrict__ xt, int HW,
                                                           long long nthr, int* __restrict__ status, int nA,
                                                           const T* __restrict__ w, uint8_t* __restrict__ wpk,
                                                           const Plan P) {
  pdl_wait();
  if ((int)blockIdx.x < nA)
    pack_input_rt_part<T>(x, xt, P.C, HW, P.Cg, P.Cgp, P.CS, nthr, nullptr, status, blockIdx.x, nA);
  else
    pack_weight_fwd_part<T>(w, wpk, P, blockIdx.x - nA, (int)gridDim.x - nA);
}

// ---------------------------------------------------------------------------
// Channels-last (DCN_NHWC) activations.

// Loads 4 consecutive logical channels [lc0, lc0+4) of one pixel row `src`
// (channels of one group, Cg of them) as floats; zero past Cg.  `vec`: one 8- or
// 16-byte load (the run lies inside the group and is 4-element aligned).
template <typename T>
__device__ __forceinline__ void load4_row(const T* __restrict__ src, int lc0, int Cg, bool vec, float (&v)[4]) {
  if (vec && lc0 + 4 <= Cg) {
    if constexpr (sizeof(T) == 4) {
      const uint4 u = ldg_nc_v4(src + lc0);
      v[0] = __uint_as_float(u.x); v[1] = __uint_as_float(u.y);
      v[2] = __uint_as_float(u.z); v[3] = __uint_as_float(u.w);
    } else {
      const uint2 u = ldg_nc_v2(src + lc0);
      v[0] = raw_to_f<T>(u.x & 0xffffu); v[1] = raw_to_f<T>(u.x >> 16);
      v[2] = raw_to_f<T>(u.y & 0xffffu); v[3] = raw_to_f<T>(u.y >> 16);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = lc0 + e < Cg ? ldf(src + lc0 + e) : 0.f;
  }
}

// x [B][HW][C] -> xt [B][HW][dg][Cgp] (perm_logical order inside each 64-channel
// block, padded channels zero).  One thread per 8-element physical slice q of a
// block: its two runs of 4 logical channels (slice_lo / slice_hi) are read with
// vector loads and stored as one slice; `acc` (the backward's fp32 grad_input
// accumulator of the same layout) is zeroed alongside and `status` cleared.
template <typename T>
__global__ void __launch_bounds__(256) pack_input_nhwc_kernel(const T* __restrict__ x, T* __restrict__ xt,
                                                              int C, int Cg, int Cgp, int CS, long long nslices,
                                                              int vec, float* __restrict__ acc,
                                                              int* __restrict__ status) {
  pdl_wait();
  if (status != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *status = 0;
  const int spp = CS >> 3;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < nslices;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long pix = idx / spp;
    const int sl = (int)(idx - pix * spp);
    const int d0 = (sl >> 3) << 6, q = sl & 7;
    const int g = d0 / Cgp, cb = d0 - g * Cgp;
    const T* src = x + (size_t)pix * C + (size_t)g * Cg;
    float lo[4], hi[4];
    load4_row<T>(src, cb + slice_lo(q), Cg, vec, lo);
    load4_row<T>(src, cb + slice_hi(q), Cg, vec, hi);
    const size_t eo = (size_t)pix * CS + d0 + 8 * q;
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<float4*>(xt + eo) = make_float4(lo[0], lo[1], lo[2], lo[3]);
      *reinterpret_cast<float4*>(xt + eo + 4) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    } else {
      constexpr int kBF = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
      *reinterpret_cast<uint4*>(xt + eo) =
          make_uint4(pack2<kBF>(lo[0], lo[1]), pack2<kBF>(lo[2], lo[3]), pack2<kBF>(hi[0], hi[1]),
                     pack2<kBF>(hi[2], hi[3]));
    }
    if (acc != nullptr) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(acc + eo) = z;
      *reinterpret_cast<float4*>(acc + eo + 4) = z;
    }
  }
}

// fp32 [B][HW][dg][Cgp] (logical channel order) -> T [B][HW][C].  One thread per
// run of 4 channels of a group (vector load and store when Cg % 4 == 0 and gx is
// 16-byte aligned), else per element.
template <typename T>
__global__ void __launch_bounds__(256) finish_grad_input_nhwc_kernel(const float* __restrict__ gxn,
                                                                     T* __restrict__ gx, int C, int Cg, int Cgp,
                                                                     int CS, long long nruns, int vec) {
  pdl_wait();
  const int rpp = C >> 2;   // runs per pixel when vec (C % 4 == 0)
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < nruns;
       idx += (long long)gridDim.x * blockDim.x) {
    if (vec) {
      const long long pix = idx / rpp;
      const int c = (int)(idx - pix * rpp) * 4;
      const int g = c / Cg, cc = c - g * Cg;
      const float4 v = *reinterpret_cast<const float4*>(gxn + (size_t)pix * CS + g * Cgp + cc);
      T* o = gx + (size_t)pix * C + c;
      if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(o) = v;
      } else {
        constexpr int kBF = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
        *reinterpret_cast<uint2*>(o) = make_uint2(pack2<kBF>(v.x, v.y), pack2<kBF>(v.z, v.w));
      }
    } else {
      const long long pix = idx / C;
      const int c = (int)(idx - pix * C);
      const int g = c / Cg, cc = c - g * Cg;
      gx[idx] = Elem<T>::from_f(gxn[(size_t)pix * CS + g * Cgp + cc]);
    }
  }
}

// grad_output [totalP][Co] (channels-last) -> the operand blocks of
// pack_gout_kernel (64 pixels x 64 Co, 128-byte rows with the 128-byte swizzle;
// f32 as bf16 hi then lo).  Thread: pixel row `row` and 8-Co chunk c of a block,
// one 16-byte load (two for f32) when Co % 8 == 0 and grad_output is aligned.
// grad_bias partial sums go to `gb` when it is not null.
template <typename T>
__global__ void __launch_bounds__(256) pack_gout_nhwc_kernel(const T* __restrict__ gout,
                                                             uint8_t* __restrict__ gpk,
                                                             float* __restrict__ gb, const Plan P, int vec) {
  pdl_wait();
  const int ko = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31;
  const int nPB = (int)((P.totalP + 63) / 64);
  const size_t blk_bytes = (size_t)P.nsplit * 8192;
  const int c = tid & 7;                 // the thread's 8-Co chunk (fixed)
  const int co0 = ko * kChunk + c * 8;
  float bsum[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) bsum[e] = 0.f;
  for (int pb = blockIdx.x; pb < nPB; pb += gridDim.x) {
    uint8_t* blk = gpk + ((size_t)pb * P.nKo + ko) * blk_bytes;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int row = (tid >> 3) + 32 * k;
      const long long pix = (long long)pb * 64 + row;
      float v[8];
      if (pix < P.totalP && vec && co0 + 8 <= P.Co) {
        const T* src = gout + (size_t)pix * P.Co + co0;
        if constexpr (sizeof(T) == 4) {
          const uint4 a = ldg_nc_v4(src), b = ldg_nc_v4(src + 4);
          v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
          v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
          v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y);
          v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
        } else {
          unpack8<T>(ldg_nc_v4(src), v);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          v[e] = (pix < P.totalP && co0 + e < P.Co) ? ldf(gout + (size_t)pix * P.Co + co0 + e) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) bsum[e] += v[e];
      const uint32_t off = sw128_off(row, c);
      if constexpr (OpOf<T>::kSplit) {
        uint4 hi, lo;
        split2(v[0], v[1], hi.x, lo.x);
        split2(v[2], v[3], hi.y, lo.y);
        split2(v[4], v[5], hi.z, lo.z);
        split2(v[6], v[7], hi.w, lo.w);
        *reinterpret_cast<uint4*>(blk + off) = hi;
        *reinterpret_cast<uint4*>(blk + 8192 + off) = lo;
      } else {
        constexpr int kBF = OpOf<T>::kBF16;
        *reinterpret_cast<uint4*>(blk + off) =
            make_uint4(pack2<kBF>(v[0], v[1]), pack2<kBF>(v[2], v[3]), pack2<kBF>(v[4], v[5]),
                       pack2<kBF>(v[6], v[7]));
      }
    }
  }
  if (gb != nullptr) {
    // lanes l, l + 8, l + 16, l + 24 hold the same chunk; the warps' sums meet
    // in shared memory and the CTA adds each Co once to the accumulator (one
    // global atomic per Co and CTA: same-address atomics from every warp took
    // hundreds of microseconds)
    __shared__ float sb[64];
    if (tid < 64) sb[tid] = 0.f;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float sum = bsum[e];
      sum += __shfl_xor_sync(0xffffffffu, sum, 8);
      sum += __shfl_xor_sync(0xffffffffu, sum, 16);
      if (lane < 8) atomicAdd(&sb[c * 8 + e], sum);
    }
    __syncthreads();
    if (tid < 64 && ko * kChunk + tid < P.Co) atomicAdd(gb + ko * kChunk + tid, sb[tid]);
  }
}

template <typename F>
int dispatch(int dtype, F&& f) {
  cudaError_t e;
  switch (dtype) {
    case DCN_F32: e = f(float{}); break;
    case DCN_F16: e = f(__half{}); break;
    default: e = f(__nv_bfloat16{}); break;
  }
  return e == cudaSuccess ? DCN_OK : DCN_E_CUDA;
}

int grid_for(long long n, int threads) {
  long long g = (n + threads - 1) / threads;
  if (g > 148LL * 16) g = 148LL * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

int launch_pack_input(const Plan& P, const void* x, void* xt, float* zero_acc, int* status,
                      cudaStream_t s) {
  const int HW = P.H * P.W;
  if (P.nhwc) {
    const long long nslices = (long long)P.B * HW * (P.CS / 8);
    const int vec = (P.C % 4 == 0) && (P.Cg % 4 == 0) && (((uintptr_t)x & 15u) == 0);
    return dispatch(P.dtype, [&](auto tag) {
      using T = decltype(tag);
      return launch_k(pack_input_nhwc_kernel<T>, dim3(grid_for(nslices, 256)), dim3(256), 0, s,
                      static_cast<const T*>(x), static_cast<T*>(xt), P.C, P.Cg, P.Cgp, P.CS, nslices, vec,
                      zero_acc, status);
    });
  }
  const int vec = (HW % 8 == 0) && (((uintptr_t)x & 15u) == 0);
  const int npb = ceil_div(HW, 64), ncb = P.CS / 64;
  const long long nblocks = (long long)npb * ncb * P.B;
  if (nblocks >= (1LL << 31)) return DCN_E_UNSUPPORTED;
  const int grid = (int)(nblocks < 148LL * 8 ? nblocks : 148LL * 8);
  if (vec && P.esz == 2) {
    const long long nthr = (long long)P.B * (HW / 8) * (P.CS / 64) * 8;
    return dispatch(P.dtype, [&](auto tag) {
      using T = decltype(tag);
      if constexpr (sizeof(T) != 2) return cudaErrorInvalidValue;
      else return launch_k(pack_input_rt_kernel<T>, dim3(grid_for(nthr, 256)), dim3(256), 0, s, static_cast<const T*>(x), static_cast<T*>(xt),
                                                                     P.C, HW, P.Cg, P.Cgp, P.CS, nthr,
                                                                     zero_acc, status);
    });
  }
  if (status != nullptr && cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return DCN_E_CUDA;
  if (zero_acc != nullptr &&
      cudaMemsetAsync(zero_acc, 0, (size_t)P.B * HW * P.CS * sizeof(float), s) != cudaSuccess)
    return DCN_E_CUDA;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(pack_input_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(x), static_cast<T*>(xt), P.C,
                                              HW, P.Cg, P.Cgp, P.CS, vec, npb, ncb, (int)nblocks);
  });
}

int launch_pack_forward(const Plan& P, const void* x, void* xt, int* status, const void* w, uint8_t* wpk,
                        cudaStream_t s) {
  const int HW = P.H * P.W;
  const bool rt = !P.nhwc && P.esz == 2 && (HW % 8 == 0) && (((uintptr_t)x & 15u) == 0);
  if (!rt) return DCN_E_UNSUPPORTED;
  const long long nthr = (long long)P.B * (HW / 8) * (P.CS / 64) * 8;
  const long long nA = grid_for(nthr, 256);
  const long long nw = (long long)P.nCoT * P.nK * P.NT * 8;
  long long nW = (nw + 255) / 256;
  if (nW > 148) nW = 148;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) != 2) return cudaErrorInvalidValue;
    else
      return launch_k(pack_forward_kernel<T>, dim3((unsigned)(nA + nW)), dim3(256), 0, s, static_cast<const T*>(x),
                      static_cast<T*>(xt), HW, nthr, status, (int)nA, static_cast<const T*>(w), wpk, P);
  });
}

int launch_pack_weight_fwd(const Plan& P, const void* w, uint8_t* wpk, cudaStream_t s) {
  const long long n = (long long)P.nCoT * P.nK * P.NT * 8;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(pack_weight_fwd_kernel<T>, dim3(grid_for(n, 256)), dim3(256), 0, s, static_cast<const T*>(w), wpk, P);
  });
}

int launch_pack_weight_bwd(const Plan& P, const void* w, uint8_t* wpk, float* zero_acc, size_t zero_bytes,
                           int* status, cudaStream_t s) {
  const long long n = (long long)P.gnU * P.nKo * P.gNC * 8;
  if (zero_bytes % 16 != 0 || ((uintptr_t)zero_acc & 15u) != 0) return DCN_E_UNSUPPORTED;
  const long long nz4 = zero_acc ? (long long)(zero_bytes / 16) : 0;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(pack_weight_bwd_kernel<T>, dim3(grid_for(n > nz4 ? n : nz4, 256)), dim3(256), 0, s, static_cast<const T*>(w), wpk, P, reinterpret_cast<float4*>(zero_acc), nz4, status);
  });
}

int launch_pack_gout(const Plan& P, const void* gout, uint8_t* gpk, float* gb, int vec,
                     cudaStream_t s) {
  const int nPB = (int)((P.totalP + 63) / 64);
  int gx = 2048 / P.nKo;  // about 14 CTAs per SM in total, pixel blocks strided
  if (gx < 1) gx = 1;
  if (gx > nPB) gx = nPB;
  dim3 grid(gx, P.nKo);
  if (P.nhwc) {
    const int v = (P.Co % 8 == 0) && (((uintptr_t)gout & 15u) == 0);
    return dispatch(P.dtype, [&](auto tag) {
      using T = decltype(tag);
      return launch_k(pack_gout_nhwc_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(gout), gpk, gb,
                      P, v);
    });
  }
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(pack_gout_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(gout), gpk, gb, P, vec);
  });
}

int launch_finish_grad_input(const Plan& P, const float* gxn, void* gx, cudaStream_t s) {
  const int HW = P.H * P.W;
  if (P.nhwc) {
    const int vec = (P.Cg % 4 == 0) && (((uintptr_t)gx & 15u) == 0);
    const long long n = (long long)P.B * HW * P.C / (vec ? 4 : 1);
    return dispatch(P.dtype, [&](auto tag) {
      using T = decltype(tag);
      return launch_k(finish_grad_input_nhwc_kernel<T>, dim3(grid_for(n, 256)), dim3(256), 0, s, gxn,
                      static_cast<T*>(gx), P.C, P.Cg, P.Cgp, P.CS, n, vec);
    });
  }
  const int vec = (HW % 8 == 0) && (((uintptr_t)gx & 15u) == 0);
  dim3 grid(ceil_div(HW, 64), P.CS / 64, P.B);
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(finish_grad_input_kernel<T>, dim3(grid), dim3(256), 0, s, gxn, static_cast<T*>(gx), P.C, HW, P.Cg,
                                                     P.Cgp, P.CS, vec);
  });
}

int launch_finish_grads(const Plan& P, const float* gxn, void* gx, const float* gw, const float* gb, void* gwo,
                        void* gbo, cudaStream_t s) {
  const int HW = P.H * P.W;
  if (P.nhwc) return DCN_E_UNSUPPORTED;
  const int vec = (HW % 8 == 0) && (((uintptr_t)gx & 15u) == 0);
  const long long nx = ceil_div(HW, 64), ny = P.CS / 64;
  const long long nA = nx * ny * P.B;
  const long long n = (long long)P.Co * P.C * P.K2;
  long long nW = (n + 255) / 256;
  if (nW > 148) nW = 148;
  if (nA + nW >= (1LL << 31)) return DCN_E_UNSUPPORTED;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(finish_grads_kernel<T>, dim3((unsigned)(nA + nW)), dim3(256), 0, s, gxn, static_cast<T*>(gx),
                    vec, (int)nx, (int)ny, (int)nA, gw, gb, static_cast<T*>(gwo), static_cast<T*>(gbo), P);
  });
}

int launch_finish_grad_weight(const Plan& P, const float* gw, const float* gb, void* gwo,
                              void* gbo, cudaStream_t s) {
  const long long n = (long long)P.Co * P.C * P.K2;
  return dispatch(P.dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_k(finish_grad_weight_kernel<T>, dim3(grid_for(n, 256)), dim3(256), 0, s, gw, gb, static_cast<T*>(gwo), static_cast<T*>(gbo), P);
  });
}

}  // namespace dcn
