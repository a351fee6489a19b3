// Shared device helpers for the sm_100a paged-attention kernels: storage dtypes,
// vector loads with float conversion, mbarrier and TMA (cp.async.bulk.tensor) PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "paged_attention_b200.h"

namespace pa {

// Device error word bits (workspace word 0).
constexpr int kErrBlockId = 1;       // block id outside [0, pool_num_blocks)
constexpr int kErrSlot = 2;          // slot outside the pool
constexpr int kErrWaitTimeout = 4;   // an mbarrier wait ran out of its iteration limit

// An mbarrier wait gives up after this many polls (each try_wait suspends for a
// hardware-chosen interval, so this is far beyond any real TMA latency) and the
// kernel records kErrWaitTimeout instead of spinning forever.
constexpr uint32_t kWaitLimit = 1u << 24;

constexpr float kLog2e = 1.4426950408889634f;

template <typename T> struct DType;
template <> struct DType<float> { static constexpr int code = PA_DTYPE_F32; };
template <> struct DType<__half> { static constexpr int code = PA_DTYPE_F16; };
template <> struct DType<__nv_bfloat16> { static constexpr int code = PA_DTYPE_BF16; };

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_float(float x);
template <> __device__ __forceinline__ float from_float<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Two packed 16-bit values -> two floats (exact widening).
__device__ __forceinline__ float2 unpack2(uint32_t w, __nv_bfloat16*) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2(uint32_t w, __half*) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// Load N consecutive elements of T at p (aligned to N*sizeof(T)) as floats.
template <typename T, int N> struct VecLoad;
template <> struct VecLoad<float, 2> {
  __device__ __forceinline__ static void run(const float* p, float* o) {
    float2 v = *reinterpret_cast<const float2*>(p); o[0] = v.x; o[1] = v.y;
  }
};
template <> struct VecLoad<float, 4> {
  __device__ __forceinline__ static void run(const float* p, float* o) {
    float4 v = *reinterpret_cast<const float4*>(p); o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <typename T> struct VecLoad16x2 {
  __device__ __forceinline__ static void run(const T* p, float* o) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    float2 a = unpack2(w, (T*)nullptr); o[0] = a.x; o[1] = a.y;
  }
};
template <typename T> struct VecLoad16x4 {
  __device__ __forceinline__ static void run(const T* p, float* o) {
    uint2 w = *reinterpret_cast<const uint2*>(p);
    float2 a = unpack2(w.x, (T*)nullptr), b = unpack2(w.y, (T*)nullptr);
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
};
template <> struct VecLoad<__nv_bfloat16, 2> : VecLoad16x2<__nv_bfloat16> {};
template <> struct VecLoad<__nv_bfloat16, 4> : VecLoad16x4<__nv_bfloat16> {};
template <> struct VecLoad<__half, 2> : VecLoad16x2<__half> {};
template <> struct VecLoad<__half, 4> : VecLoad16x4<__half> {};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false if the barrier did not complete within kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ---------------------------------------------------------------- TMA
// 3-D tiled bulk tensor load global -> shared, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}
// 2-D form: c0 is the innermost coordinate (its byte offset must be a multiple of 16).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

__device__ __forceinline__ void set_error(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

}  // namespace pa
