// Shared helpers for the kvengine_b200 sm_100a kernels: status codes, dtype
// conversions with the reference's rounding points, warp reductions, and a
// bounded wait used by every spin loop in this library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "../../include/kvengine_b200.h"

namespace kve {

// Sets the thread-local message returned by kve_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
void count_launch();

// Called right after every kernel launch of this library.
inline int check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(KVE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return KVE_OK;
}

// Device-side error recording: first error wins. `status` may be null.
__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  // Round a float to this storage type and back (identity for fp32).
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};

// Rotate-half RoPE of one pair (x1 = element d, x2 = element d + hd/2), as
// kvengine/forward.py:49-69 computes it in the model dtype: cos/sin rounded to
// the dtype first, every product and the sum rounded like elementwise torch ops.
template <typename T>
__device__ __forceinline__ float rope_first(float x1, float x2, float c, float s) {
  const float cb = Elem<T>::round(c), sb = Elem<T>::round(s);
  return __fadd_rn(Elem<T>::round(__fmul_rn(x1, cb)), Elem<T>::round(__fmul_rn(-x2, sb)));
}
template <typename T>
__device__ __forceinline__ float rope_second(float x1, float x2, float c, float s) {
  const float cb = Elem<T>::round(c), sb = Elem<T>::round(s);
  return __fadd_rn(Elem<T>::round(__fmul_rn(x2, cb)), Elem<T>::round(__fmul_rn(x1, sb)));
}
template <typename T>
__device__ __forceinline__ void rope_pair(float x1, float x2, float c, float s, T* o1, T* o2) {
  *o1 = Elem<T>::from_f(rope_first<T>(x1, x2, c, s));
  *o2 = Elem<T>::from_f(rope_second<T>(x1, x2, c, s));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every spin-wait in this library gives up after this long and reports
// KVE_ERR_TIMEOUT instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Programmatic dependent launch. Kernels of this library are launched so that
// the next kernel in the stream may be scheduled, and run its prologue, while
// this one drains. The contract every kernel keeps: grid_dep_wait() comes before
// its first access, read or write, to global memory that an earlier kernel may
// write (it returns once the kernels before it in the stream have completed and
// their writes are visible); only inputs declared constant, such as model
// weights in kve_forward, are read before it. grid_dep_launch() follows it.
// Both are no-ops for a plain launch.
// The wait is an inline-asm memory barrier, which the compiler honours only for
// memory it cannot prove private: a load through a `const T* __restrict__` kernel
// parameter may be scheduled above it. Inputs that an earlier kernel writes are
// therefore never declared __restrict__ (constant weights may be).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Dependent launches are on unless KVE_PDL=0 is set in the environment.
bool pdl_enabled();

// Launch with the programmatic-stream-serialization attribute (plus any extra
// attributes, e.g. a cluster shape).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             const cudaLaunchAttribute* extra, int n_extra, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[4];
  int n = 0;
  for (int i = 0; i < n_extra && n < 3; ++i) attrs[n++] = extra[i];
  if (pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  return launch_kernel_ex(kernel, grid, block, smem, stream, nullptr, 0, std::forward<Args>(args)...);
}

}  // namespace kve
