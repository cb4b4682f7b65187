// qe_fused_util.cuh — building blocks of the fused cluster sampler:
// TMA bulk loads with mbarrier completion, 8-element smem loads, warp
// reductions and small sorts.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qe_common.cuh"

namespace qe {
namespace fz {

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Bounded wait on an mbarrier phase.  Returns false if the phase did not
// complete within `limit` polls (the caller records an error; it never hangs).
// Each poll may suspend the thread for up to kTryWaitHintNs (it resumes as
// soon as the phase completes) and sleeps 128 ns after a miss, so the bound
// is about limit * (kTryWaitHintNs + 128 ns).
constexpr uint32_t kTryWaitHintNs = 1000;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
  uint32_t done = 0;
  for (uint32_t i = 0; i < limit; ++i) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitHintNs)
        : "memory");
    if (done) return true;
    __nanosleep(128);   // fewer polls while the copy is in flight
  }
  return false;
}
// Order this thread's earlier generic-proxy smem accesses before later
// async-proxy (bulk copy) writes.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 1-D bulk copy global -> shared, completion counted on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- element loads
// Load 8 consecutive elements starting at smem element offset `off` (a
// multiple of 8) as fp32; elements at or beyond `nvalid` read as -inf.
template <typename T> struct Load8;
template <> struct Load8<__nv_bfloat16> {
  static __device__ __forceinline__ void run(const void* buf, int off, int nvalid, float x[8]) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(buf) + off);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(ws[i] << 16);
      x[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
    }
    if (nvalid < 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) if (i >= nvalid) x[i] = -INFINITY;
    }
  }
};
template <> struct Load8<__half> {
  static __device__ __forceinline__ void run(const void* buf, int off, int nvalid, float x[8]) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(buf) + off);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&ws[i]);
      float2 f = __half22float2(h);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
    if (nvalid < 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) if (i >= nvalid) x[i] = -INFINITY;
    }
  }
};
template <> struct Load8<float> {
  static __device__ __forceinline__ void run(const void* buf, int off, int nvalid, float x[8]) {
    const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(buf) + off);
    const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(buf) + off + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    if (nvalid < 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) if (i >= nvalid) x[i] = -INFINITY;
    }
  }
};

// Max of 8 consecutive elements starting at smem element offset `off`
// (NaN-propagating); elements at or beyond `nvalid` are ignored.  16-bit
// types use packed max on the raw words, without unpacking.
template <typename T> struct Max8;
template <> struct Max8<__nv_bfloat16> {
  static __device__ __forceinline__ float run(const void* buf, int off, int nvalid) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(buf) + off);
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    if (nvalid < 8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (2 * i >= nvalid) ws[i] = 0xFF80FF80u;                 // -inf, -inf
        else if (2 * i + 1 >= nvalid) ws[i] = (ws[i] & 0xFFFFu) | 0xFF800000u;
      }
    }
    __nv_bfloat162 a = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&ws[0]), *reinterpret_cast<__nv_bfloat162*>(&ws[1]));
    __nv_bfloat162 b = __hmax2_nan(*reinterpret_cast<__nv_bfloat162*>(&ws[2]), *reinterpret_cast<__nv_bfloat162*>(&ws[3]));
    a = __hmax2_nan(a, b);
    const float lo = __bfloat162float(__low2bfloat16(a)), hi = __bfloat162float(__high2bfloat16(a));
    return (lo != lo || hi != hi) ? NAN : fmaxf(lo, hi);
  }
};
template <> struct Max8<__half> {
  static __device__ __forceinline__ float run(const void* buf, int off, int nvalid) {
    const uint4 w = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(buf) + off);
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    if (nvalid < 8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (2 * i >= nvalid) ws[i] = 0xFC00FC00u;
        else if (2 * i + 1 >= nvalid) ws[i] = (ws[i] & 0xFFFFu) | 0xFC000000u;
      }
    }
    __half2 a = __hmax2_nan(*reinterpret_cast<__half2*>(&ws[0]), *reinterpret_cast<__half2*>(&ws[1]));
    __half2 b = __hmax2_nan(*reinterpret_cast<__half2*>(&ws[2]), *reinterpret_cast<__half2*>(&ws[3]));
    a = __hmax2_nan(a, b);
    const float lo = __low2float(a), hi = __high2float(a);
    return (lo != lo || hi != hi) ? NAN : fmaxf(lo, hi);
  }
};
template <> struct Max8<float> {
  static __device__ __forceinline__ float run(const void* buf, int off, int nvalid) {
    float x[8];
    Load8<float>::run(buf, off, nvalid, x);
    float m = x[0];
    bool nan = x[0] != x[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) { m = fmaxf(m, x[i]); nan |= x[i] != x[i]; }
    return nan ? NAN : m;
  }
};

// Apply the repetition penalty to the elements whose bit is set in `bits8`.
__device__ __forceinline__ void apply_penalty8(uint32_t bits8, float rp, float x[8]) {
  if (bits8) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((bits8 >> i) & 1u) x[i] = penalise(x[i], rp);
  }
}

// ---------------------------------------------------------------- ordering
// Monotone map of a float to uint32 (NaN above +inf).
__device__ __forceinline__ uint32_t ordered_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0xFFFFFFFFu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Race order on (r desc, id asc); NaN r never wins.
__device__ __forceinline__ bool rbetter(float r, int id, float rb, int ib) {
  if (r != r) return false;
  return r > rb || (r == rb && id < ib);
}

}  // namespace fz
}  // namespace qe
