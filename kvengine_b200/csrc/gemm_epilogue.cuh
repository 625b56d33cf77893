// GEMM epilogues shared by the CUDA-core and tcgen05 kernels. Rounding points
// follow the reference's module-by-module torch ops in the model dtype:
// nn.Linear output rounded once (bias added before that rounding), the
// residual add rounded again, SwiGLU as round(round(silu(round(g))) * round(u)).
#pragma once

#include <math.h>

#include "kve_common.cuh"

namespace kve {

struct EpiArgs {
  int mode;           // KVE_EPI_*
  int out_dtype;      // KVE_F32 / KVE_BF16 (the dtype rounding happens in)
  int ld_out;         // leading dimension of out (n, or n/2 for SILU_MUL)
  const float* bias;  // [n] (BIAS)
  const void* residual;  // [m, n] in out_dtype (RESIDUAL); may alias out
  void* out;
  int w_static;       // w is written by no kernel that may still run: its loads may start early
  // kEpiQkvRope only: the qkv projection's output goes straight to its consumers.
  int nq, nkv, hd;
  const int32_t* positions;  // [m]
  const int32_t* slots;      // [m] pool slot of each token's K/V
  const float* rope_cos;     // [rope_len, hd / 2]
  const float* rope_sin;
  int rope_len;
  void* q_out;               // [m, nq * hd]
  void* pool_k;              // [num_slots, nkv * hd]
  void* pool_v;
  int64_t num_slots;
  int* status;
};

// Internal epilogue of the tcgen05 GEMM (not in the C ABI): bias, bf16 rounding,
// RoPE of the q and k heads, q to q_out, k and v to their pool slots - the
// qkv projection and kve_qkv_rope_append in one pass.
constexpr int kEpiQkvRope = KVE_EPI_SILU_MUL + 1;

__device__ __forceinline__ float round_to(int dtype, float v) {
  return dtype == KVE_BF16 ? Elem<__nv_bfloat16>::round(v) : v;
}

__device__ __forceinline__ void write_out(const EpiArgs& e, int row, int col, float v) {
  size_t idx = (size_t)row * e.ld_out + col;
  if (e.out_dtype == KVE_BF16) static_cast<__nv_bfloat16*>(e.out)[idx] = __float2bfloat16_rn(v);
  else static_cast<float*>(e.out)[idx] = v;
}

__device__ __forceinline__ float read_res(const EpiArgs& e, int row, int col) {
  size_t idx = (size_t)row * e.ld_out + col;
  if (e.out_dtype == KVE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(e.residual)[idx]);
  return static_cast<const float*>(e.residual)[idx];
}

// STORE / BIAS / RESIDUAL for one element.
__device__ __forceinline__ void epi_store(const EpiArgs& e, int row, int col, float acc) {
  float v = acc;
  if (e.mode == KVE_EPI_BIAS) {
    v = __fadd_rn(acc, e.bias[col]);
  } else if (e.mode == KVE_EPI_RESIDUAL) {
    v = __fadd_rn(read_res(e, row, col), round_to(e.out_dtype, acc));
  }
  write_out(e, row, col, v);
}

__device__ __forceinline__ float silu_ref(float g) { return g / (1.0f + expf(-g)); }

// SiLU with the fast exponential and division intrinsics: a few fp32 ulp, and
// branch-free, so the SwiGLU pairs of one thread overlap instead of running one
// division slow-path check after another. The exponent is capped at 80 so the
// denominator stays below 2^126, the range __fdividef is exact to 2 ulp in; for
// g < -80 the true result (|g| e^g < 1e-33) and this one are both 0 to within
// bf16 rounding of any sum they enter. The result is rounded to the model dtype
// right after, where the difference from g / (1 + expf(-g)) is far below one
// bf16 ulp except next to a rounding boundary.
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(fminf(-g, 80.0f))); }

// SwiGLU pair: gate and up accumulators of output column j.
__device__ __forceinline__ void epi_silu_mul(const EpiArgs& e, int row, int j, float gate, float up) {
  float g = round_to(e.out_dtype, gate);
  float u = round_to(e.out_dtype, up);
  float s = round_to(e.out_dtype, silu_ref(g));
  write_out(e, row, j, __fmul_rn(s, u));
}

int gemm_simt(const void* x, const void* w, int dtype, int m, int n, int k, const EpiArgs& e,
              cudaStream_t stream);
int gemm_tc(const void* x, const void* w, int m, int n, int k, const EpiArgs& e, void* workspace,
            size_t workspace_bytes, int* status, cudaStream_t stream);
size_t gemm_tc_workspace_bytes(int m, int n, int k);

// kve_gemm_ex with the weight-is-constant hint (model weights in kve_forward).
int gemm_run(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue, const float* bias,
             const void* residual, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
             int* dev_status, int algo, bool w_static, cudaStream_t stream);

// The fused qkv projection of one layer (bf16): x [m, k] times w_qkv [n, k]^T
// plus bias, then the work of kve_qkv_rope_append. `e` carries the rope fields.
int gemm_qkv_rope(const void* x, const void* w, int m, int n, int k, const EpiArgs& e, cudaStream_t stream);

}  // namespace kve
