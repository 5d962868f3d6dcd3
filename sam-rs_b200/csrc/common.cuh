// common.cuh - dtype helpers and the device status word shared by every kernel of the library.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace samrs {

// Device status word (one per device, in the library's static device memory). Kernels never trap:
// a bounded wait that runs out or a failed geometry check stores a nonzero code and the kernel
// returns early; the host reads it with samrs_device_status().
enum StatusCode : unsigned int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,  // mbarrier / TMA wait exceeded its iteration bound
  kStatusMmaTimeout = 2,   // wait on a tcgen05 commit exceeded its bound
  kStatusBadGeometry = 3,  // launch geometry does not match the kernel's assumptions
};

// The library is a single translation unit (samrs_abi.cu includes every kernel header), so the
// word is defined here.
__device__ unsigned int g_status = 0;

__device__ __forceinline__ void report(unsigned int code) { atomicCAS(&g_status, 0u, code); }

// Test hooks (samrs_test_hooks): a shorter bound for every wait (cycles; 0 = the built-in ~1 s), and a key
// tile whose K load CTA 0 of the global kernel never issues (-1 = none), so that a test can watch a bounded
// wait run out, the kernel return with the status word set, and the library recover. Nothing else reads them.
__device__ long long g_wait_limit = 0;
__device__ int g_withhold_key_tile = -1;

// Number of bf16 global-layer CTAs (one head x 256 query rows) that the exact fixup launch recomputed,
// read and cleared by samrs_recompute_count(). A statistic for the caller, not read by any kernel.
__device__ unsigned long long g_recomputed = 0;

// Per-layer recompute counters of the host's speculative-pass policy (global_policy.h): a measuring call
// zeroes its layer's slot on its stream and points the fixup launch at it. No kernel reads them.
constexpr int kPolicySlots = 64;
__device__ unsigned long long g_policy_counts[kPolicySlots];

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

}  // namespace samrs
