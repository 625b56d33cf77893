// kve_gemm: argument checks and the choice between the two GEMM kernels
// (tcgen05 for bf16, CUDA-core for fp32; kve_gemm_ex can force either).
#include "gemm_epilogue.cuh"

using namespace kve;

extern "C" size_t kve_gemm_workspace_bytes(int m, int n, int k, int dtype) {
  if (m <= 0 || n <= 0 || k <= 0 || dtype != KVE_BF16) return 0;
  return gemm_tc_workspace_bytes(m, n, k);
}

namespace kve {

int gemm_run(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue, const float* bias,
             const void* residual, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
             int* dev_status, int algo, bool w_static, cudaStream_t stream) {
  if (m < 0 || n < 1 || k < 1) return set_error(KVE_ERR_ARG, "kve_gemm: bad sizes m=%d n=%d k=%d", m, n, k);
  if (m == 0) return KVE_OK;
  if (!x || !w || !out) return set_error(KVE_ERR_ARG, "kve_gemm: null pointer");
  if (dtype != KVE_F32 && dtype != KVE_BF16) return set_error(KVE_ERR_DTYPE, "kve_gemm: dtype %d", dtype);
  if (out_dtype != KVE_F32 && out_dtype != KVE_BF16)
    return set_error(KVE_ERR_DTYPE, "kve_gemm: out_dtype %d", out_dtype);
  if (epilogue < KVE_EPI_STORE || epilogue > KVE_EPI_SILU_MUL)
    return set_error(KVE_ERR_ARG, "kve_gemm: epilogue %d", epilogue);
  if (epilogue == KVE_EPI_BIAS && !bias) return set_error(KVE_ERR_ARG, "kve_gemm: BIAS needs bias");
  if (epilogue == KVE_EPI_RESIDUAL && !residual) return set_error(KVE_ERR_ARG, "kve_gemm: RESIDUAL needs residual");
  if (epilogue == KVE_EPI_SILU_MUL && (n % 2)) return set_error(KVE_ERR_SHAPE, "kve_gemm: SILU_MUL needs even n");
  EpiArgs e{};
  e.mode = epilogue;
  e.out_dtype = out_dtype;
  e.ld_out = epilogue == KVE_EPI_SILU_MUL ? n / 2 : n;
  e.bias = bias;
  e.residual = residual;
  e.out = out;
  e.w_static = w_static ? 1 : 0;
  if (algo == KVE_GEMM_AUTO) algo = dtype == KVE_BF16 ? KVE_GEMM_TCGEN05 : KVE_GEMM_SIMT;
  if (algo == KVE_GEMM_TCGEN05) {
    if (dtype != KVE_BF16) return set_error(KVE_ERR_DTYPE, "kve_gemm: tcgen05 path takes bf16 inputs");
    return gemm_tc(x, w, m, n, k, e, workspace, workspace_bytes, dev_status, stream);
  }
  if (algo == KVE_GEMM_SIMT) return gemm_simt(x, w, dtype, m, n, k, e, stream);
  return set_error(KVE_ERR_ARG, "kve_gemm: algo %d", algo);
}

}  // namespace kve

extern "C" int kve_gemm_ex(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue,
                           const float* bias, const void* residual, void* out, int out_dtype,
                           void* workspace, size_t workspace_bytes, int* dev_status, int algo,
                           cudaStream_t stream) {
  return gemm_run(x, w, dtype, m, n, k, epilogue, bias, residual, out, out_dtype, workspace, workspace_bytes,
                  dev_status, algo, false, stream);
}

extern "C" int kve_gemm(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue,
                        const float* bias, const void* residual, void* out, int out_dtype, void* workspace,
                        size_t workspace_bytes, int* dev_status, cudaStream_t stream) {
  return kve_gemm_ex(x, w, dtype, m, n, k, epilogue, bias, residual, out, out_dtype, workspace,
                     workspace_bytes, dev_status, KVE_GEMM_AUTO, stream);
}
