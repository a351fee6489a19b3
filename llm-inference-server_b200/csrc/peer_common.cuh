// Device helpers shared by the peer-memory collectives (peer_allreduce.cu,
// oproj_allreduce.cu): system-scope release / acquire flags, bounded flag waits, L1-bypassing
// 16-byte loads, and 16-byte vectors of 16- or 32-bit elements summed in float32.
#pragma once

#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 16-byte load that bypasses L1 (peer data changes between calls).
__device__ __forceinline__ uint4 ld_cg(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Wait until flags[0..world) >= epoch (thread t < world watches flag t).  Returns false
// on the deadline.
static __device__ bool wait_flags(const uint32_t* flags, int world, uint32_t epoch, uint64_t deadline) {
  bool ok = true;
  if (threadIdx.x < world) {
    while (int32_t(ld_acquire_sys(flags + threadIdx.x) - epoch) < 0) {
      if (global_ns() > deadline) {
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

template <typename T>
struct Pack8;  // eight 16-bit or four 32-bit elements in 16 bytes
template <>
struct Pack8<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void add(float (&a)[8], uint4 v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      a[2 * i] += f.x;
      a[2 * i + 1] += f.y;
    }
  }
  __device__ static uint4 pack(const float (&a)[8]) {
    uint4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    return v;
  }
};
template <>
struct Pack8<__half> {
  static constexpr int N = 8;
  __device__ static void add(float (&a)[8], uint4 v) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      a[2 * i] += f.x;
      a[2 * i + 1] += f.y;
    }
  }
  __device__ static uint4 pack(const float (&a)[8]) {
    uint4 v;
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(a[2 * i], a[2 * i + 1]);
    return v;
  }
};
template <>
struct Pack8<float> {
  static constexpr int N = 4;
  __device__ static void add(float (&a)[8], uint4 v) {
    a[0] += __uint_as_float(v.x);
    a[1] += __uint_as_float(v.y);
    a[2] += __uint_as_float(v.z);
    a[3] += __uint_as_float(v.w);
  }
  __device__ static uint4 pack(const float (&a)[8]) {
    return make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
  }
};

}  // namespace pa
