// Shared host/device helpers for the B200 attention library: error state, launch accounting,
// bf16 conversion, and small numeric helpers used by the CUDA-core kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include <utility>

#include "../../include/attn_b200.h"

namespace attn {

// ---- host-side error state (per calling thread) -------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();
void count_launch(int n = 1);

// Check the launch that just happened; returns ATTN_OK or ATTN_ERR_CUDA with the message set.
int check_launch(const char* what);
// The same for a launch whose error the launch call returned (cudaLaunchKernelEx).
int check_launch(const char* what, cudaError_t launched);

#define ATTN_REQUIRE(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      ::attn::set_error(__VA_ARGS__);           \
      return ATTN_ERR_ARG;                      \
    }                                           \
  } while (0)

#define ATTN_CUDA_TRY(call)                                                        \
  do {                                                                             \
    cudaError_t e_ = (call);                                                       \
    if (e_ != cudaSuccess) {                                                       \
      ::attn::set_error("%s failed: %s", #call, cudaGetErrorString(e_));           \
      return ATTN_ERR_CUDA;                                                        \
    }                                                                              \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- programmatic dependent launch ------------------------------------------------------------
// The kernels of a training step launch with programmatic stream serialization: a kernel's CTAs may
// be placed on the SMs as soon as every CTA of its predecessor on the stream has started (or
// signalled grid_dependents_launch), so their set-up (barrier initialisation, TMEM allocation,
// descriptor prefetch) overlaps the predecessor's last wave.  Every thread of such a kernel calls
// grid_dependency_wait() before its first global-memory access: it returns once the predecessor
// grid has completed and its writes are visible (at once when the kernel was launched without the
// attribute or its predecessor is not a kernel).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launch_pdl sets the attribute: yes unless the environment variable ATTN_NO_PDL is set to
// a non-empty value other than "0" when the library first launches (every kernel then waits for its
// predecessor to complete, as with a plain launch).
bool pdl_enabled();

// Launch `kernel` on `s` with programmatic stream serialization allowed.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same for a kernel of CTA pairs: clusters of two consecutive CTAs along x (grid.x even).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_pairs(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                    Args&&... args) {
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- device-side element helpers ----------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

// Load 4 consecutive elements (16 B for float, 8 B for bf16) as floats; p must be aligned.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// ---- GELU of the feed-forward block ---------------------------------------------------------
// The tanh form of activation_kernel (core/kernels.py:243-248), gelu(x) = 0.5 x (1 + tanh(u)) with
// u = K0 (x + K1 x^3), and its derivative as gelu_backward_kernel writes it (core/kernels.py:432-440).
// FAST selects the tanh.approx.f32 instruction (the bf16 tensor-core path, whose outputs are rounded
// to bf16 anyway); otherwise tanhf (the float32 path, 1e-5 parity).
constexpr float GELU_K0 = 0.7978845608f, GELU_K1 = 0.044715f, GELU_K1x3 = 0.134145f;
enum { ACT_NONE = ATTN_ACT_NONE, ACT_GELU = ATTN_ACT_GELU, ACT_GELU_BWD = ATTN_ACT_GELU_BWD };

template <bool FAST>
__device__ __forceinline__ float gelu_tanh_of(float x) {
  const float u = GELU_K0 * (x + GELU_K1 * x * x * x);
  if constexpr (FAST) {
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return t;
  } else {
    return tanhf(u);
  }
}

template <bool FAST>
__device__ __forceinline__ float gelu_fwd(float x) {
  return 0.5f * x * (1.f + gelu_tanh_of<FAST>(x));
}

template <bool FAST>
__device__ __forceinline__ float gelu_grad(float x) {
  const float t = gelu_tanh_of<FAST>(x);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * (GELU_K0 * (1.f + GELU_K1x3 * x * x));
}

}  // namespace attn
