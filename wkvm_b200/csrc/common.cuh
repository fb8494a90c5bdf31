// Shared device helpers for the wkvm_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/wkvm_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wkvm_b200 kernels are written for sm_100a (B200) only"
#endif

namespace wkvm {

// Element loads/stores for the three activation dtypes the ops accept.
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// A per-token gate (g or beta) of the gated delta rule: fp32 when the caller
// passed WKVM_GATES_F32, else the activation dtype.
template <typename Tin>
__device__ __forceinline__ float load_gate(const void* p, int64_t i, bool f32) {
  return f32 ? static_cast<const float*>(p)[i] : to_f32(static_cast<const Tin*>(p)[i]);
}

// Streaming 128-bit state access. The recurrent state of one (slot, head) is
// touched exactly once per kernel launch, so loads bypass L1 allocation and
// stores skip L1 too: nothing in the launch re-reads them. The state is
// updated in place, so the read-only (.nc) path is not used.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.L1::no_allocate.v4.f32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Records the first error a kernel meets into the caller's optional status
// word (device memory, 0 == ok). Kernels skip the offending work instead of
// trapping, so the context stays usable.
__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Process-wide opt-in (wkvm_set_decode_overlap) for programmatic dependent
// launch of the single-token decode kernels.
bool decode_overlap();

}  // namespace wkvm

#define WKVM_CUDA_TRY(expr)                         \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return WKVM_ERR_CUDA;    \
  } while (0)
