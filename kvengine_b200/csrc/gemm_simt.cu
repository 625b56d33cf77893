// CUDA-core GEMM y = x w^T (fp32 or bf16 inputs, fp32 accumulation) with the
// library's fused epilogues.
//
// Every output element is one sequential FMA chain over k = 0 .. K-1 in a
// single thread, so its value does not depend on m, on the element's position
// in the tile, or on the grid: a 1-row draft pass and a k+1-row verify pass of
// the same model produce bit-identical rows. This is the fp32 path
// (correctness configuration); bf16 uses the tcgen05 kernel in gemm_tc.cu.
#include <math.h>

#include "gemm_epilogue.cuh"

namespace kve {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;
constexpr int kThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads)
gemm_simt_kernel(const T* x, const T* __restrict__ w, int m, int n, int k, EpiArgs e) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < k; k0 += BK) {
    // 64x16 tiles: thread loads 4 elements of each (rows r, k column c).
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      int idx = threadIdx.x + u * kThreads;
      int r = idx / BK, c = idx % BK;
      int gm = m0 + r, gn = n0 + r, gk = k0 + c;
      xs[c][r] = (gm < m && gk < k) ? Elem<T>::to_f(x[(size_t)gm * k + gk]) : 0.f;
      ws[c][r] = (gn < n && gk < k) ? Elem<T>::to_f(w[(size_t)gn * k + gk]) : 0.f;
    }
    __syncthreads();
    const int kmax = min(BK, k - k0);
    for (int kk = 0; kk < kmax; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      int gn = n0 + tx * 4 + j;
      if (e.mode == KVE_EPI_SILU_MUL) {
        if (gn + 1 < n) epi_silu_mul(e, gm, gn / 2, acc[i][j], acc[i][j + 1]);
      } else {
        if (gn < n) epi_store(e, gm, gn, acc[i][j]);
        if (gn + 1 < n) epi_store(e, gm, gn + 1, acc[i][j + 1]);
      }
    }
  }
}

}  // namespace

int gemm_simt(const void* x, const void* w, int dtype, int m, int n, int k, const EpiArgs& e,
              cudaStream_t stream) {
  dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM);
  if (dtype == KVE_F32) {
    launch_kernel(gemm_simt_kernel<float>, dim3(grid), dim3(kThreads), 0, stream, static_cast<const float*>(x),
                                                           static_cast<const float*>(w), m, n, k, e);
  } else if (dtype == KVE_BF16) {
    launch_kernel(gemm_simt_kernel<__nv_bfloat16>, dim3(grid), dim3(kThreads), 0, stream,
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), m, n, k, e);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_gemm: dtype %d", dtype);
  }
  return check_launch("kve_gemm(simt)");
}

}  // namespace kve
