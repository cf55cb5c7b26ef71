// Shared device helpers for the sm_100a DCNv2 kernels: mbarriers with bounded
// waits, bulk (TMA) copies, tcgen05 (UMMA) descriptors / MMA / TMEM access, and
// element conversions.  Every wait on an mbarrier gives up after
// DCN_WAIT_TIMEOUT_NS, records DCN_DEVERR_TIMEOUT in the caller's error word and
// raises a CTA-wide abort flag, so a broken pipeline ends the kernel instead of
// hanging the GPU.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "dcn_b200.h"
#include "dcn_plan.h"

#ifndef DCN_WAIT_TIMEOUT_NS
#define DCN_WAIT_TIMEOUT_NS 4000000000ull  // 4 s: far above any legitimate wait
#endif

namespace dcn {

// n / f.d for 0 <= n < 2^31 (see FastDiv)
__device__ __forceinline__ int fdiv(int n, const FastDiv& f) {
  return f.d == 1 ? n : (int)(__umulhi((uint32_t)n, f.m) >> f.sh);
}

// ---------------------------------------------------------------- basics
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread is suspended (issuing nothing)
// until the phase completes or about `ns` nanoseconds have passed.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Suspend-time hint of the bounded waits below (ns); 0 selects polling with a
// growing __nanosleep between polls instead.  Measured on the README layer:
// the same instruction count either way (waiting warps issue little), the tile
// scatter 183.3 -> 181.5 us with a 20 us hint (the warp resumes as soon as the
// phase completes instead of at the end of its sleep); the clock and the abort
// flag are checked after every suspended poll.
#ifndef DCN_MBAR_SUSPEND_NS
#define DCN_MBAR_SUSPEND_NS 20000
#endif
constexpr uint32_t kMbarSuspendNs = DCN_MBAR_SUSPEND_NS;

// Longest sleep between two failed polls of an mbarrier (ns).  Waiting warps
// that spin without sleeping took most of the issue slots of the tile scatter
// (ncu: 142 warp instructions per sample, issue 66% active).
#ifndef DCN_MBAR_MAX_SLEEP_NS
#define DCN_MBAR_MAX_SLEEP_NS 256
#endif
constexpr uint32_t kMbarMaxSleepNs = DCN_MBAR_MAX_SLEEP_NS;

// Waits for the phase of parity `parity` to complete.  Returns false (and
// records a timeout) when the wait exceeds DCN_WAIT_TIMEOUT_NS or when another
// warp of the CTA has already aborted.  Single-thread form: for code run by one
// elected lane (bulk-copy and MMA issuers); whole warps use mbar_wait_warp.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  // the clock and the abort flag are consulted only every 256 polls, and a
  // failed poll backs off with a growing sleep (32 ns doubling up to
  // kMbarMaxSleepNs), so that waiting warps cost the working warps as few
  // issue slots as possible
  uint64_t t0 = 0;
  uint32_t ns = 32;
  for (uint32_t i = 1;; ++i) {
    if (kMbarSuspendNs) {
      if (mbar_try_wait_suspend(bar, parity, kMbarSuspendNs)) return true;
    } else {
      if (mbar_try_wait(bar, parity)) return true;
      __nanosleep(ns);
      if (ns < kMbarMaxSleepNs) ns <<= 1;
    }
    if (kMbarSuspendNs || (i & 255u) == 0u) {
      if (*abort_flag) return false;
      const uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > DCN_WAIT_TIMEOUT_NS) {
        raise_error(err, DCN_DEVERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Warp-collective form of mbar_wait: all 32 lanes of the warp call it and all
// get the same answer.  Every lane polls the barrier, the loop ends only when
// every lane has seen the phase complete (__all_sync), and the decision to give
// up (abort flag or timeout) is taken by lane 0 and broadcast, so no lane leaves
// early and the warp reaches the next __syncwarp or .sync.aligned instruction
// converged, whether the wait succeeded or not.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int* err,
                                               volatile int* abort_flag) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  uint32_t ns = 32;
  for (uint32_t i = 1;; ++i) {
    if (kMbarSuspendNs) {
      if (__all_sync(0xffffffffu, mbar_try_wait_suspend(bar, parity, kMbarSuspendNs))) return true;
    } else {
      if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
      __nanosleep(ns);
      if (ns < kMbarMaxSleepNs) ns <<= 1;
    }
    if (kMbarSuspendNs || (i & 255u) == 0u) {
      int give_up = 0;
      if (lane == 0) {
        if (*abort_flag) {
          give_up = 1;
        } else {
          const uint64_t now = globaltimer();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > DCN_WAIT_TIMEOUT_NS) {
            raise_error(err, DCN_DEVERR_TIMEOUT);
            *abort_flag = 1;
            give_up = 1;
          }
        }
      }
      if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
    }
  }
}

// Bounded wait used during teardown: ignores the abort flag (the barrier is
// still expected to complete) but never spins longer than the timeout.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > DCN_WAIT_TIMEOUT_NS) {
      raise_error(err, DCN_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (tensor core / TMA) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- bulk copy (TMA engine)
// Untiled bulk copy global -> shared; completion is signalled as tx bytes on `bar`.
// Source and destination 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 3-D tiled TMA load of a box (no multicast) into this CTA's shared memory,
// completion as tx bytes on an mbarrier.  Coordinates are element indices,
// innermost first; the innermost one times the element size must be a multiple
// of 16 bytes.  Out-of-range elements of the box are filled with zeros.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// Programmatic dependent launch.  Every kernel of this library is launched with
// the previous kernel of its stream allowed to be still running; it calls
// pdl_wait() before its first global-memory access (the wait returns once the
// previous grid has completed and its writes are visible), so only its launch
// and set-up (barrier init, TMEM allocation) overlap the previous kernel's end.
// No kernel triggers its dependents early (griddepcontrol.launch_dependents):
// measured on the README layer, an early trigger made the step slower
// (537 vs 504 us).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Warpgroup register re-allocation: every warp of a warpgroup executes the same
// call; the block's register file (launch registers x threads) is redistributed.
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one CTA, kind::f16 (f16 or bf16 operands, f32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (two x16 loads, one wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr + 16u));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128-byte swizzle (Swizzle<3,4,3>), sm_100 format:
// start address [0,14), leading byte offset [16,30), stride byte offset [32,46),
// version 1 at [46,48), layout type 2 (SWIZZLE_128B) at [61,64).  All >> 4.
//   K-major : rows of 128 B (64 16-bit elements of K); SBO = 1024 B between
//             8-row groups; LBO unused.
//   MN-major: rows of 128 B (64 16-bit elements of M or N) per K index;
//             SBO = byte stride between groups of 8 K rows, LBO = byte stride
//             between 64-element M/N atoms.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Shared-memory matrix descriptor, no swizzle (K-major: 8-row x 16-byte core
// matrices; lbo = byte distance of the core matrices adjacent in K, sbo = of the
// 8-row groups).
__device__ __forceinline__ uint64_t nosw_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor for kind::f16: f32 accumulator, A/B format (0 f16, 1 bf16),
// major-ness of A and B (0 K-major, 1 MN-major), M and N.
__host__ __device__ constexpr uint32_t make_idesc(int bf16, int a_mn, int b_mn, int M, int N) {
  return (1u << 4) | ((uint32_t)bf16 << 7) | ((uint32_t)bf16 << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 1024-byte aligned
// SW128 tile whose rows are 128 B apart.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// ---------------------------------------------------------------- element types
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  return Elem<T>::to_f(*p);
}

// Operand type fed to the tensor core for an input type: f16 stays f16; bf16 and
// f32 (as a bf16 hi/lo pair) run on bf16.
template <typename T>
struct OpOf {
  static constexpr int kBF16 = 1;
  static constexpr bool kSplit = false;
};
template <>
struct OpOf<float> {
  static constexpr int kBF16 = 1;
  static constexpr bool kSplit = true;
};
template <>
struct OpOf<__half> {
  static constexpr int kBF16 = 0;
  static constexpr bool kSplit = false;
};

// Packs two floats into the 16-bit operand type (bf16 when kBF16, else f16).
template <int kBF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (kBF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// bf16 hi/lo split of two floats: a ~= hi + lo with |a - hi - lo| <= 2^-17 |a|.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  float2 hf = __bfloat1622float2(h);
  __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<uint32_t*>(&h);
  lo = *reinterpret_cast<uint32_t*>(&l);
}

// Unpacks 8 packed 16-bit values (one uint4) into floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __half>::value) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 x = __half22float2(h);
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    } else {
      // bf16 is the top half of an f32: two bit operations, no conversion
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Raw element load issued where it is written (volatile asm is not moved to the
// first use), for prefetching: 16-bit types as their bit pattern, f32 as bits.
template <typename T>
__device__ __forceinline__ uint32_t ldg_raw(const T* p) {
  uint32_t r;
  if constexpr (sizeof(T) == 2) {
    unsigned short h;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(h) : "l"(p));
    r = h;
  } else {
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  }
  return r;
}

// Converts a raw element (see ldg_raw) to float.
template <typename T>
__device__ __forceinline__ float raw_to_f(uint32_t r) {
  if constexpr (std::is_same<T, float>::value) {
    return __uint_as_float(r);
  } else if constexpr (std::is_same<T, __half>::value) {
    return __half2float(__ushort_as_half((unsigned short)r));
  } else {
    return __uint_as_float(r << 16);
  }
}

__device__ __forceinline__ uint2 ldg_nc_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Sum of the elements held in 16 bytes (eight 16-bit values, or four f32), in fp32.
template <typename T>
__device__ __forceinline__ float sum8(const uint4& w) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, float>::value) {
      s += __uint_as_float(u[i]);
    } else {
      s += raw_to_f<T>(u[i] & 0xffffu) + raw_to_f<T>(u[i] >> 16);
    }
  }
  return s;
}

// Vector fp32 reduction into global memory (sm_90+).
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// ---------------------------------------------------------------- channel order
// Inside every 64-channel block the packed input (and every operand derived
// from it) stores channels in the order that makes the 8 channels a lane owns
// contiguous: physical position 8q + r holds logical channel 4q + r (r < 4) or
// 32 + 4q + (r - 4) (r >= 4).  A lane's 16-byte slice q is then logical channels
// [4q, 4q+4) and [32+4q, 32+4q+4), so the grad_input scatter (in logical order)
// fills whole 32-byte sectors with two lanes per red.add instruction.
// DCN_PERM=0 (study builds) keeps the logical order instead: lane q then owns
// logical channels [8q, 8q+8), one 32-byte sector of fp32 per lane.
#ifndef DCN_PERM
#define DCN_PERM 1
#endif
__host__ __device__ __forceinline__ int perm_logical(int pp) {
#if DCN_PERM
  const int q = pp >> 3, r = pp & 7;
  return r < 4 ? 4 * q + r : 32 + 4 * q + (r - 4);
#else
  return pp;
#endif
}
// Logical channel (inside the 64-channel block) of the first and of the fifth
// element of physical 16-byte slice q: where a lane's two fp32 quadruples go.
__host__ __device__ __forceinline__ int slice_lo(int q) { return DCN_PERM ? 4 * q : 8 * q; }
__host__ __device__ __forceinline__ int slice_hi(int q) { return DCN_PERM ? 32 + 4 * q : 8 * q + 4; }

// ---------------------------------------------------------------- sampling geometry
// Bilinear sampling geometry of one (pixel, tap, group): the four corner
// weights (already multiplied by the modulation mask; zero for corners outside
// the image) and the corner pixel indices.  Follows the reference's validity
// rule -1 < h < H, -1 < w < W and per-corner zero padding (com.cu:119-148, 187).
struct Sample {
  float h, w;        // sample position
  float lh, lw;      // fractional parts
  float m;           // modulation mask
  float cw[4];       // corner weights * mask (0 for corners outside the image)
  int cidx[4];       // corner pixel index h*W + w (valid only when cw != 0 or flag set)
  uint32_t cvalid;   // bit i: corner i inside the image
  bool inside;       // -1 < h < H and -1 < w < W
};

__device__ __forceinline__ Sample make_sample(float h, float w, float m, int H, int W) {
  Sample s;
  s.h = h;
  s.w = w;
  s.m = m;
  s.inside = (h > -1.f) && (w > -1.f) && (h < (float)H) && (w < (float)W);
  const float hf = floorf(h), wf = floorf(w);
  const int hl = (int)hf, wl = (int)wf;
  s.lh = h - hf;
  s.lw = w - wf;
  const float hh = 1.f - s.lh, hw = 1.f - s.lw;
  const bool r0 = hl >= 0, r1 = hl + 1 <= H - 1, c0 = wl >= 0, c1 = wl + 1 <= W - 1;
  s.cvalid = 0;
  if (s.inside) {
    s.cvalid = (r0 && c0 ? 1u : 0u) | (r0 && c1 ? 2u : 0u) | (r1 && c0 ? 4u : 0u) |
               (r1 && c1 ? 8u : 0u);
  }
  s.cw[0] = (s.cvalid & 1u) ? hh * hw * m : 0.f;
  s.cw[1] = (s.cvalid & 2u) ? hh * s.lw * m : 0.f;
  s.cw[2] = (s.cvalid & 4u) ? s.lh * hw * m : 0.f;
  s.cw[3] = (s.cvalid & 8u) ? s.lh * s.lw * m : 0.f;
  s.cidx[0] = hl * W + wl;
  s.cidx[1] = hl * W + wl + 1;
  s.cidx[2] = (hl + 1) * W + wl;
  s.cidx[3] = (hl + 1) * W + wl + 1;
  return s;
}

}  // namespace dcn
