// Fused greedy acceptance (argmax over the vocab for every verify row, prefix
// match against the drafts, emitted tokens) and a plain row-argmax kernel.
//
// One CTA scans one 151,936-wide logits row with 16-byte loads (HBM-bound:
// the row is read exactly once). The last CTA to finish a sequence's k+1 rows
// (per-sequence arrival counter in the workspace) runs the acceptance with a
// warp ballot and resets the counter to zero, so the workspace stays clean.
#include <math.h>

#include <mutex>

#include "kve_common.cuh"

namespace kve {
namespace {

constexpr int kArgmaxThreads = 512;

// (v1, i1) beats (v2, i2): NaN is the maximum (torch.argmax semantics), larger
// values win, equal values resolve to the lower index.
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  bool n1 = isnan(v1), n2 = isnan(v2);
  if (n1 || n2) return (n1 && n2) ? (i1 < i2) : n1;
  if (v1 != v2) return v1 > v2;
  return i1 < i2;
}

template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float* p, float (&o)[4]) {
    float4 v = __ldcs(reinterpret_cast<const float4*>(p));
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[8]) {
    uint4 v = __ldcs(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      o[2 * j] = f.x; o[2 * j + 1] = f.y;
    }
  }
};

// Argmax of x[lo, hi) of one row (x is the row's start, indices are absolute;
// with vec_ok, lo is a multiple of the vector width). The result, valid in
// thread 0, goes to best_v / best_i.
template <typename T>
__device__ __forceinline__ void range_argmax(const T* x, int lo, int hi, bool vec_ok, float& best_v, int& best_i) {
  best_v = -INFINITY;
  best_i = 0x7fffffff;
  constexpr int N = Vec<T>::N;
  const int v0 = vec_ok ? lo / N : 0;
  const int nvec = vec_ok ? hi / N : 0;  // vectors [v0, nvec), then elements [max(lo, nvec * N), hi)
  constexpr int U = 4;
  int v = v0 + threadIdx.x;
  for (; v + (U - 1) * kArgmaxThreads < nvec; v += U * kArgmaxThreads) {
    float buf[U][N];
#pragma unroll
    for (int u = 0; u < U; ++u) Vec<T>::load(x + (size_t)(v + u * kArgmaxThreads) * N, buf[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      int base = (v + u * kArgmaxThreads) * N;
#pragma unroll
      for (int j = 0; j < N; ++j)
        if (better(buf[u][j], base + j, best_v, best_i)) { best_v = buf[u][j]; best_i = base + j; }
    }
  }
  for (; v < nvec; v += kArgmaxThreads) {
    float buf[N];
    Vec<T>::load(x + (size_t)v * N, buf);
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (better(buf[j], v * N + j, best_v, best_i)) { best_v = buf[j]; best_i = v * N + j; }
  }
  for (int i = max(lo, nvec * N) + threadIdx.x; i < hi; i += kArgmaxThreads) {
    float f = Elem<T>::to_f(x[i]);
    if (better(f, i, best_v, best_i)) { best_v = f; best_i = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
  }
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best_v; si[warp] = best_i; }
  __syncthreads();
  if (warp == 0) {
    best_v = lane < kArgmaxThreads / 32 ? sv[lane] : -INFINITY;
    best_i = lane < kArgmaxThreads / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
    }
  }
}

template <typename T>
__device__ __forceinline__ int row_argmax(const T* x, int cols, bool vec_ok) {
  float v;
  int i;
  range_argmax(x, 0, cols, vec_ok, v, i);
  return i;  // valid in thread 0
}

// Three CTAs per SM (at most 40 registers a thread): a verify batch's rows
// (64 x 5 = 320) then run in one wave on 148 SMs instead of 296 + 24.
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads, 3)
accept_kernel(const T* logits, int64_t row_stride, const int32_t* drafts,
              int64_t dsb, int64_t dsj, int k, int vocab, bool vec_ok, int32_t* __restrict__ preds, int32_t* __restrict__ n_acc,
              int32_t* __restrict__ emitted, int32_t* __restrict__ counters) {
  grid_dep_wait();
  grid_dep_launch();
  const int row = blockIdx.x;
  const int b = row / (k + 1);
  int best = row_argmax(logits + (size_t)row * row_stride, vocab, vec_ok);
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    preds[row] = best;
    __threadfence();
    int prev = atomicAdd(&counters[b], 1);
    is_last = (prev == k);
    if (is_last) counters[b] = 0;  // every row of b has arrived: leave the workspace zeroed
  }
  __syncthreads();
  if (!is_last || threadIdx.x >= 32) return;
  __threadfence();
  const int lane = threadIdx.x;
  int p = lane <= k ? __ldcg(preds + (size_t)b * (k + 1) + lane) : -1;
  int d = lane < k ? drafts[b * dsb + lane * dsj] : -1;
  unsigned mism = __ballot_sync(0xffffffffu, lane < k && p != d);
  int n = mism ? (__ffs(mism) - 1) : k;
  int pn = __shfl_sync(0xffffffffu, p, n);
  if (lane <= k) {
    int e = lane < n ? d : (lane == n ? pn : -1);
    emitted[(size_t)b * (k + 1) + lane] = e;
  }
  if (lane == 0) n_acc[b] = n;
}

// Row argmax; with `scatter_out`, row i's result is also written to
// scatter_out[scatter_idx[i]] (the draft loop places each draft token straight
// into its slot of the verify pass's token ids).
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads)
argmax_kernel(const T* x, int64_t row_stride, int cols, bool vec_ok, int32_t* __restrict__ out,
              const int32_t* scatter_idx, int32_t* __restrict__ scatter_out, int64_t scatter_len,
              int* __restrict__ status) {
  grid_dep_wait();
  grid_dep_launch();
  int best = row_argmax(x + (size_t)blockIdx.x * row_stride, cols, vec_ok);
  if (threadIdx.x == 0) {
    out[blockIdx.x] = best;
    if (scatter_out) {
      const int j = scatter_idx[blockIdx.x];
      if (j >= 0 && j < scatter_len) scatter_out[j] = best;
      else report(status, KVE_ERR_BOUNDS);
    }
  }
}

// Row argmax split over a cluster of `parts` CTAs (consecutive CTAs form one
// row's cluster): CTA p scans columns [p * chunk, (p + 1) * chunk) and rank 0
// combines the parts' (value, index) pairs through distributed shared memory.
// `better` is a total order, so the result is the one argmax_kernel gives; with
// few rows (the draft's 64) a single CTA per row leaves most SMs idle and each
// scans 300 KB at one SM's load rate.
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads)
argmax_split_kernel(const T* x, int64_t row_stride, int cols, bool vec_ok, int parts, int chunk,
                    int32_t* __restrict__ out, const int32_t* scatter_idx, int32_t* __restrict__ scatter_out,
                    int64_t scatter_len, int* __restrict__ status) {
  grid_dep_wait();
  grid_dep_launch();
  const int row = blockIdx.x / parts, part = blockIdx.x % parts;
  const int lo = min(part * chunk, cols), hi = min(lo + chunk, cols);
  float v;
  int i;
  range_argmax(x + (size_t)row * row_stride, lo, hi, vec_ok, v, i);
  __shared__ float s_v;
  __shared__ int s_i;
  if (threadIdx.x == 0) {
    s_v = v;
    s_i = i;
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (part == 0 && threadIdx.x == 0) {
    const uint32_t av = static_cast<uint32_t>(__cvta_generic_to_shared(&s_v));
    const uint32_t ai = static_cast<uint32_t>(__cvta_generic_to_shared(&s_i));
    for (int p = 1; p < parts; ++p) {
      uint32_t rv, ri;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rv) : "r"(av), "r"(p));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ri) : "r"(ai), "r"(p));
      float pv;
      int pi;
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(rv) : "memory");
      asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(pi) : "r"(ri) : "memory");
      if (better(pv, pi, v, i)) { v = pv; i = pi; }
    }
    out[row] = i;
    if (scatter_out) {
      const int j = scatter_idx[row];
      if (j >= 0 && j < scatter_len) scatter_out[j] = i;
      else report(status, KVE_ERR_BOUNDS);
    }
  }
  // The parts stay resident until rank 0 has read them.
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

bool vec_aligned(const void* p, int64_t row_stride, int elem) {
  return ((uintptr_t)p % 16 == 0) && ((row_stride * elem) % 16 == 0);
}

}  // namespace
}  // namespace kve

using namespace kve;

extern "C" size_t kve_greedy_accept_workspace_bytes(int batch) {
  size_t b = (size_t)(batch > 0 ? batch : 0) * sizeof(int32_t);
  return (b + 255) / 256 * 256;
}

extern "C" int kve_greedy_accept(const void* logits, int dtype, int64_t row_stride,
                                 const int32_t* drafts, int64_t draft_stride_b, int64_t draft_stride_j, int batch, int k, int vocab,
                                 int32_t* out_preds, int32_t* out_n_accepted, int32_t* out_emitted,
                                 void* workspace, size_t workspace_bytes, int* dev_status,
                                 cudaStream_t stream) {
  (void)dev_status;
  if (batch < 0 || k < 1 || k > 31 || vocab < 1 || row_stride < vocab)
    return set_error(KVE_ERR_ARG, "kve_greedy_accept: bad sizes batch=%d k=%d vocab=%d stride=%lld",
                     batch, k, vocab, (long long)row_stride);
  if (batch == 0) return KVE_OK;
  if (!logits || !drafts || !out_preds || !out_n_accepted || !out_emitted)
    return set_error(KVE_ERR_ARG, "kve_greedy_accept: null pointer");
  if (!workspace || workspace_bytes < kve_greedy_accept_workspace_bytes(batch))
    return set_error(KVE_ERR_WORKSPACE, "kve_greedy_accept: workspace needs %zu bytes",
                     kve_greedy_accept_workspace_bytes(batch));
  dim3 grid(batch * (k + 1));
  int32_t* counters = static_cast<int32_t*>(workspace);
  if (dtype == KVE_F32) {
    launch_kernel(accept_kernel<float>, dim3(grid), dim3(kArgmaxThreads), 0, stream,
        static_cast<const float*>(logits), row_stride, drafts, draft_stride_b, draft_stride_j, k, vocab,
        vec_aligned(logits, row_stride, 4), out_preds, out_n_accepted, out_emitted, counters);
  } else if (dtype == KVE_BF16) {
    launch_kernel(accept_kernel<__nv_bfloat16>, dim3(grid), dim3(kArgmaxThreads), 0, stream,
        static_cast<const __nv_bfloat16*>(logits), row_stride, drafts, draft_stride_b, draft_stride_j, k, vocab,
        vec_aligned(logits, row_stride, 2), out_preds, out_n_accepted, out_emitted, counters);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_greedy_accept: dtype %d", dtype);
  }
  return check_launch("kve_greedy_accept");
}

namespace {
// Parts per row for argmax_split_kernel (cluster size, at most the portable 8):
// as many CTAs as fit the SMs in one wave, none for wide batches or short rows.
int argmax_parts(int rows, int cols) {
  if (cols < 8 * 4096) return 1;
  const int want = 2 * 148 / rows;  // one wave at two 512-thread CTAs per SM
  return want >= 8 ? 8 : want >= 4 ? 4 : want >= 2 ? 2 : 1;
}

template <typename T>
int argmax_split_launch(const T* x, int rows, int cols, int64_t row_stride, bool vec_ok, int parts, int32_t* out,
                        const int32_t* scatter_idx, int32_t* scatter_out, int64_t scatter_len, int* status,
                        cudaStream_t stream) {
  constexpr int N = Vec<T>::N;
  const int chunk = ((cols + parts - 1) / parts + N - 1) / N * N;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = parts;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaError_t err = launch_kernel_ex(argmax_split_kernel<T>, dim3(rows * parts), dim3(kArgmaxThreads), 0, stream,
                                     &attr, 1, x, row_stride, cols, vec_ok, parts, chunk, out, scatter_idx,
                                     scatter_out, scatter_len, status);
  if (err != cudaSuccess) {
    cudaGetLastError();
    count_launch();
    return set_error(KVE_ERR_CUDA, "kve_argmax_rows(split): launch failed: %s", cudaGetErrorString(err));
  }
  return check_launch("kve_argmax_rows");
}

int argmax_launch(const void* x, int dtype, int rows, int cols, int64_t row_stride, int32_t* out,
                  const int32_t* scatter_idx, int32_t* scatter_out, int64_t scatter_len, int* status,
                  cudaStream_t stream) {
  const int parts = argmax_parts(rows, cols);
  if (parts > 1 && dtype == KVE_F32)
    return argmax_split_launch(static_cast<const float*>(x), rows, cols, row_stride, vec_aligned(x, row_stride, 4),
                               parts, out, scatter_idx, scatter_out, scatter_len, status, stream);
  if (parts > 1 && dtype == KVE_BF16)
    return argmax_split_launch(static_cast<const __nv_bfloat16*>(x), rows, cols, row_stride,
                               vec_aligned(x, row_stride, 2), parts, out, scatter_idx, scatter_out, scatter_len,
                               status, stream);
  if (dtype == KVE_F32) {
    launch_kernel(argmax_kernel<float>, dim3(rows), dim3(kArgmaxThreads), 0, stream,
        static_cast<const float*>(x), row_stride, cols, vec_aligned(x, row_stride, 4), out, scatter_idx, scatter_out,
        scatter_len, status);
  } else if (dtype == KVE_BF16) {
    launch_kernel(argmax_kernel<__nv_bfloat16>, dim3(rows), dim3(kArgmaxThreads), 0, stream,
        static_cast<const __nv_bfloat16*>(x), row_stride, cols, vec_aligned(x, row_stride, 2), out, scatter_idx,
        scatter_out, scatter_len, status);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_argmax_rows: dtype %d", dtype);
  }
  return check_launch("kve_argmax_rows");
}
}  // namespace

extern "C" int kve_argmax_rows(const void* x, int dtype, int rows, int cols, int64_t row_stride,
                               int32_t* out, cudaStream_t stream) {
  if (rows < 0 || cols < 1 || row_stride < cols)
    return set_error(KVE_ERR_ARG, "kve_argmax_rows: bad sizes");
  if (rows == 0) return KVE_OK;
  if (!x || !out) return set_error(KVE_ERR_ARG, "kve_argmax_rows: null pointer");
  return argmax_launch(x, dtype, rows, cols, row_stride, out, nullptr, nullptr, 0, nullptr, stream);
}

extern "C" int kve_argmax_rows_scatter(const void* x, int dtype, int rows, int cols, int64_t row_stride,
                                       int32_t* out, const int32_t* scatter_idx, int32_t* scatter_out,
                                       int64_t scatter_len, int* dev_status, cudaStream_t stream) {
  if (rows < 0 || cols < 1 || row_stride < cols || scatter_len < 0)
    return set_error(KVE_ERR_ARG, "kve_argmax_rows_scatter: bad sizes");
  if (rows == 0) return KVE_OK;
  if (!x || !out || !scatter_idx || !scatter_out)
    return set_error(KVE_ERR_ARG, "kve_argmax_rows_scatter: null pointer");
  return argmax_launch(x, dtype, rows, cols, row_stride, out, scatter_idx, scatter_out, scatter_len, dev_status,
                       stream);
}

// ---------------------------------------------------------------------------
// Allocation-free greedy acceptance.
//
// kve_greedy_accept asks the caller for a small device workspace (one int32
// arrival counter per sequence). Some callers cannot provide one on demand: a
// host with no device allocator of its own (a plain C or FFI caller holding only
// the logits and output pointers), or code running where an allocation is not
// allowed (inside a CUDA-graph capture, or a serving loop with a fixed memory
// budget). This entry point takes the counters from a file-scope device array
// instead, so it allocates nothing.
//
// * The array holds kNoAllocMaxBatch counters (16 KiB); larger batches are
//   rejected with KVE_ERR_ARG before anything is launched.
// * The counters must be zero when a call starts. The array is zero when the
//   module loads and every completed call leaves it zero again (the last CTA of
//   each sequence resets that sequence's counter).
// * Calls on one device share the array: two calls that overlap in time (on
//   different streams without ordering between them) race on it. Order them on
//   one stream, or use kve_greedy_accept with a workspace per stream.
// * The device address of the array is looked up once per device, with that
//   device current, on its first call. That lookup is not a stream operation,
//   but it may load the module; make the first call on each device outside any
//   stream capture.
namespace kve {
namespace {

constexpr int kNoAllocMaxBatch = 4096;
static __device__ __align__(256) int32_t g_accept_counters[kNoAllocMaxBatch];

constexpr int kMaxDevices = 64;
std::mutex g_counter_mu;
int32_t* g_counter_ptr[kMaxDevices] = {};

// Device address of g_accept_counters on the current device, or null with the
// error message set.
int32_t* accept_counters_for_current_device() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error(KVE_ERR_CUDA, "kve_greedy_accept_noalloc: no current device (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> g(g_counter_mu);
  if (!g_counter_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_accept_counters);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      set_error(KVE_ERR_CUDA, "kve_greedy_accept_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return nullptr;
    }
    g_counter_ptr[dev] = static_cast<int32_t*>(p);
  }
  return g_counter_ptr[dev];
}

}  // namespace
}  // namespace kve

extern "C" int kve_greedy_accept_noalloc_max_batch(void) { return kve::kNoAllocMaxBatch; }

extern "C" int kve_greedy_accept_noalloc(const void* logits, int dtype, int64_t row_stride, const int32_t* drafts,
                                         int64_t draft_stride_b, int64_t draft_stride_j, int batch, int k,
                                         int vocab, int32_t* out_preds, int32_t* out_n_accepted,
                                         int32_t* out_emitted, cudaStream_t stream) {
  if (batch < 0 || k < 1 || k > 31 || vocab < 1 || row_stride < vocab)
    return set_error(KVE_ERR_ARG, "kve_greedy_accept_noalloc: bad sizes batch=%d k=%d vocab=%d stride=%lld",
                     batch, k, vocab, (long long)row_stride);
  if (batch > kNoAllocMaxBatch)
    return set_error(KVE_ERR_ARG,
                     "kve_greedy_accept_noalloc: batch %d exceeds the built-in maximum of %d sequences "
                     "(use kve_greedy_accept with a workspace)",
                     batch, kNoAllocMaxBatch);
  if (batch == 0) return KVE_OK;
  if (!logits || !drafts || !out_preds || !out_n_accepted || !out_emitted)
    return set_error(KVE_ERR_ARG, "kve_greedy_accept_noalloc: null pointer");
  if (dtype != KVE_F32 && dtype != KVE_BF16) return set_error(KVE_ERR_DTYPE, "kve_greedy_accept_noalloc: dtype %d", dtype);
  int32_t* counters = accept_counters_for_current_device();
  if (!counters) return KVE_ERR_CUDA;
  dim3 grid(batch * (k + 1));
  if (dtype == KVE_F32) {
    launch_kernel(accept_kernel<float>, grid, dim3(kArgmaxThreads), 0, stream, static_cast<const float*>(logits),
                  row_stride, drafts, draft_stride_b, draft_stride_j, k, vocab, vec_aligned(logits, row_stride, 4),
                  out_preds, out_n_accepted, out_emitted, counters);
  } else {
    launch_kernel(accept_kernel<__nv_bfloat16>, grid, dim3(kArgmaxThreads), 0, stream,
                  static_cast<const __nv_bfloat16*>(logits), row_stride, drafts, draft_stride_b, draft_stride_j, k,
                  vocab, vec_aligned(logits, row_stride, 2), out_preds, out_n_accepted, out_emitted, counters);
  }
  return check_launch("kve_greedy_accept_noalloc");
}
