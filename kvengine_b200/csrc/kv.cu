// Paged-cache writes and the small per-token kernels of the forward pass:
// KV append (plain and fused with rotary embedding), history gather, token
// embedding and RMSNorm. All are HBM/latency-bound copies or row reductions.
#include <math.h>

#include "kve_common.cuh"
#include "passes.cuh"

namespace kve {
namespace {

// ---------------------------------------------------------------- append
// One 16-byte chunk per thread; chunks [0, n*cpr) are K rows, [n*cpr, 2*n*cpr) V rows.
__global__ void kv_append_kernel(const uint4* k_new, const uint4* v_new, const int64_t* slots, int n_tokens,
                                 int chunks_per_row,
                                 uint4* __restrict__ pool_k, uint4* __restrict__ pool_v,
                                 int64_t num_slots, int* status) {
  grid_dep_wait();
  grid_dep_launch();
  int64_t total = (int64_t)n_tokens * chunks_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < 2 * total;
       i += (int64_t)gridDim.x * blockDim.x) {
    bool is_v = i >= total;
    int64_t j = is_v ? i - total : i;
    int64_t t = j / chunks_per_row, c = j % chunks_per_row;
    int64_t slot = slots[t];
    if (slot < 0 || slot >= num_slots) { report(status, KVE_ERR_BOUNDS); continue; }
    const uint4* src = is_v ? v_new : k_new;
    uint4* dst = is_v ? pool_v : pool_k;
    dst[slot * chunks_per_row + c] = src[t * chunks_per_row + c];
  }
}

// ------------------------------------------------------- rope + append
// CTA per token. Rotate-half pairing (d, d + hd/2) exactly as
// kvengine/forward.py:49-69; cos/sin are rounded to the model dtype first and
// every product/sum is rounded like the reference's elementwise torch ops.
// rope_pair (kve_common.cuh) is the rotation itself, shared with the fused
// qkv GEMM epilogue.

template <typename T>
__global__ void qkv_rope_append_kernel(const T* qkv, int nq, int nkv, int hd, const int32_t* positions,
                                       const int32_t* slots,
                                       const float* __restrict__ rope_cos,
                                       const float* __restrict__ rope_sin, int rope_len,
                                       T* __restrict__ q_out, T* __restrict__ pool_k,
                                       T* __restrict__ pool_v, int64_t num_slots, int* status) {
  grid_dep_wait();
  grid_dep_launch();
  const int t = blockIdx.x;
  const int half = hd / 2;
  const int width = (nq + 2 * nkv) * hd;
  const T* row = qkv + (size_t)t * width;
  int pos = positions[t];
  int64_t slot = slots[t];
  bool pos_ok = pos >= 0 && pos < rope_len;
  bool slot_ok = slot >= 0 && slot < num_slots;
  if (threadIdx.x == 0) {
    if (!pos_ok || !slot_ok) report(status, KVE_ERR_BOUNDS);
  }
  if (!pos_ok) pos = 0;
  const float* cr = rope_cos + (size_t)pos * half;
  const float* sr = rope_sin + (size_t)pos * half;
  // q and k heads: one thread per rotation pair.
  const int pairs = (nq + nkv) * half;
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    int head = p / half, d = p % half;
    const T* src = row + head * hd;
    float x1 = Elem<T>::to_f(src[d]), x2 = Elem<T>::to_f(src[d + half]);
    float c = cr[d], s = sr[d];
    T *o1, *o2;
    if (head < nq) {
      T* dst = q_out + ((size_t)t * nq + head) * hd;
      o1 = dst + d; o2 = dst + d + half;
    } else {
      if (!slot_ok) continue;
      T* dst = pool_k + ((size_t)slot * nkv + (head - nq)) * hd;
      o1 = dst + d; o2 = dst + d + half;
    }
    rope_pair<T>(x1, x2, c, s, o1, o2);
  }
  if (!slot_ok) return;
  const T* vsrc = row + (nq + nkv) * hd;
  T* vdst = pool_v + (size_t)slot * nkv * hd;
  for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) vdst[i] = vsrc[i];
}

// ------------------------------------------------------------- gather
template <typename T>
__global__ void gather_kv_kernel(const T* pool, const int32_t* table, int length,
                                 int nkv, int hd, int bs, int64_t num_blocks, T* __restrict__ out,
                                 int* status) {
  grid_dep_wait();
  grid_dep_launch();
  int64_t total = (int64_t)nkv * length * hd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int d = i % hd;
    int64_t r = i / hd;
    int t = r % length;
    int h = r / length;
    int64_t blk = table[t / bs];
    if (blk < 0 || blk >= num_blocks) { report(status, KVE_ERR_BOUNDS); out[i] = T(); continue; }
    out[i] = pool[(((blk * bs) + t % bs) * nkv + h) * hd + d];
  }
}

// -------------------------------------------------------------- embed
template <typename T>
__global__ void embed_kernel(const int32_t* ids, const T* __restrict__ table, int hidden, int vocab,
                             T* __restrict__ out, int* status) {
  grid_dep_wait();
  grid_dep_launch();
  int t = blockIdx.x;
  int id = ids[t];
  bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) report(status, KVE_ERR_BOUNDS);
  const T* src = table + (size_t)(ok ? id : 0) * hidden;
  T* dst = out + (size_t)t * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = ok ? src[i] : T();
}

// ------------------------------------------------------------ rmsnorm
// Qwen2RMSNorm: w * round_T(x * (1 / sqrt(mean(x^2) + eps))). The reduction
// order is fixed by (hidden, blockDim), so a row's result never depends on
// which other rows are in the batch.
constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads)
rmsnorm_kernel(const T* x, const float* __restrict__ w, int hidden, float eps, const int32_t* row_index,
               T* __restrict__ out, int w_static) {
  // x and row_index are written by earlier kernels: no __restrict__ on them, so no
  // load through them can be scheduled above the dependency wait.
  // Thread t owns elements t, t + 256, ...: the first kNormRegs of them stay in
  // registers between the sum of squares and the scaling (one read of x), and the
  // weights for them are read before the dependency wait when they are constant.
  constexpr int kNormRegs = 8;  // hidden <= 2048 fully in registers
  float wv[kNormRegs];
  if (w_static) {
#pragma unroll
    for (int j = 0; j < kNormRegs; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      wv[j] = i < hidden ? w[i] : 0.f;
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  if (!w_static) {
#pragma unroll
    for (int j = 0; j < kNormRegs; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      wv[j] = i < hidden ? w[i] : 0.f;
    }
  }
  int r = blockIdx.x;
  int src_row = row_index ? row_index[r] : r;
  const T* xr = x + (size_t)src_row * hidden;
  float xv[kNormRegs];
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    xv[j] = i < hidden ? Elem<T>::to_f(xr[i]) : 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j)
    if (threadIdx.x + j * kNormThreads < hidden) ss = fmaf(xv[j], xv[j], ss);
  for (int i = threadIdx.x + kNormRegs * kNormThreads; i < hidden; i += kNormThreads) {
    float v = Elem<T>::to_f(xr[i]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  __shared__ float red[kNormThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float inv = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  T* orow = out + (size_t)r * hidden;
#pragma unroll
  for (int j = 0; j < kNormRegs; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < hidden) orow[i] = Elem<T>::from_f(__fmul_rn(wv[j], Elem<T>::round(__fmul_rn(xv[j], inv))));
  }
  for (int i = threadIdx.x + kNormRegs * kNormThreads; i < hidden; i += kNormThreads) {
    float v = Elem<T>::round(__fmul_rn(Elem<T>::to_f(xr[i]), inv));
    orow[i] = Elem<T>::from_f(__fmul_rn(w[i], v));
  }
}

inline int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > 148 * 32) g = 148 * 32;
  return (int)g;
}

inline int elem_size(int dtype) { return dtype == KVE_F32 ? 4 : dtype == KVE_BF16 ? 2 : 0; }

}  // namespace
}  // namespace kve

using namespace kve;

extern "C" int kve_kv_append(const void* k_new, const void* v_new, int dtype, const int64_t* slot_ids,
                             int n_tokens, int num_kv_heads, int head_dim, void* pool_k, void* pool_v,
                             int64_t num_slots, int* dev_status, cudaStream_t stream) {
  int es = elem_size(dtype);
  if (!es) return set_error(KVE_ERR_DTYPE, "kve_kv_append: dtype %d", dtype);
  if (n_tokens < 0 || num_kv_heads < 1 || head_dim < 1 || num_slots < 0)
    return set_error(KVE_ERR_ARG, "kve_kv_append: bad sizes");
  if (n_tokens == 0) return KVE_OK;
  int64_t row_bytes = (int64_t)num_kv_heads * head_dim * es;
  if (row_bytes % 16) return set_error(KVE_ERR_SHAPE, "kve_kv_append: row bytes %lld not a multiple of 16",
                                       (long long)row_bytes);
  if (!k_new || !v_new || !slot_ids || !pool_k || !pool_v)
    return set_error(KVE_ERR_ARG, "kve_kv_append: null pointer");
  for (const void* p : {k_new, v_new, (const void*)pool_k, (const void*)pool_v})
    if ((uintptr_t)p % 16) return set_error(KVE_ERR_ARG, "kve_kv_append: pointers must be 16-byte aligned");
  int cpr = (int)(row_bytes / 16);
  int threads = 256;
  launch_kernel(kv_append_kernel, dim3(grid_for(2LL * n_tokens * cpr, threads)), dim3(threads), 0, stream,
      static_cast<const uint4*>(k_new), static_cast<const uint4*>(v_new), slot_ids, n_tokens, cpr,
      static_cast<uint4*>(pool_k), static_cast<uint4*>(pool_v), num_slots, dev_status);
  return check_launch("kve_kv_append");
}

extern "C" int kve_qkv_rope_append(const void* qkv, int dtype, int n_tokens, int num_heads,
                                   int num_kv_heads, int head_dim, const int32_t* positions,
                                   const int32_t* slots, const float* rope_cos, const float* rope_sin,
                                   int rope_len, void* q_out, void* pool_k, void* pool_v,
                                   int64_t num_slots, int* dev_status, cudaStream_t stream) {
  if (n_tokens < 0 || num_heads < 1 || num_kv_heads < 1 || head_dim < 2 || head_dim % 2 ||
      num_heads % num_kv_heads)
    return set_error(KVE_ERR_ARG, "kve_qkv_rope_append: bad sizes");
  if (n_tokens == 0) return KVE_OK;
  if (!qkv || !positions || !slots || !rope_cos || !rope_sin || !q_out || !pool_k || !pool_v)
    return set_error(KVE_ERR_ARG, "kve_qkv_rope_append: null pointer");
  int threads = 128;
  if (dtype == KVE_F32) {
    launch_kernel(qkv_rope_append_kernel<float>, dim3(n_tokens), dim3(threads), 0, stream,
        static_cast<const float*>(qkv), num_heads, num_kv_heads, head_dim, positions, slots, rope_cos,
        rope_sin, rope_len, static_cast<float*>(q_out), static_cast<float*>(pool_k),
        static_cast<float*>(pool_v), num_slots, dev_status);
  } else if (dtype == KVE_BF16) {
    launch_kernel(qkv_rope_append_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(threads), 0, stream,
        static_cast<const __nv_bfloat16*>(qkv), num_heads, num_kv_heads, head_dim, positions, slots,
        rope_cos, rope_sin, rope_len, static_cast<__nv_bfloat16*>(q_out),
        static_cast<__nv_bfloat16*>(pool_k), static_cast<__nv_bfloat16*>(pool_v), num_slots, dev_status);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_qkv_rope_append: dtype %d", dtype);
  }
  return check_launch("kve_qkv_rope_append");
}

extern "C" int kve_gather_kv(const void* pool, int dtype, const int32_t* block_table, int length,
                             int num_kv_heads, int head_dim, int block_size, int64_t num_blocks, void* out,
                             int* dev_status, cudaStream_t stream) {
  if (length < 0 || num_kv_heads < 1 || head_dim < 1 || block_size < 1)
    return set_error(KVE_ERR_ARG, "kve_gather_kv: bad sizes");
  if (length == 0) return KVE_OK;
  if (!pool || !block_table || !out) return set_error(KVE_ERR_ARG, "kve_gather_kv: null pointer");
  int64_t work = (int64_t)num_kv_heads * length * head_dim;
  if (dtype == KVE_F32) {
    launch_kernel(gather_kv_kernel<float>, dim3(grid_for(work, 256)), dim3(256), 0, stream,
        static_cast<const float*>(pool), block_table, length, num_kv_heads, head_dim, block_size,
        num_blocks, static_cast<float*>(out), dev_status);
  } else if (dtype == KVE_BF16) {
    launch_kernel(gather_kv_kernel<__nv_bfloat16>, dim3(grid_for(work, 256)), dim3(256), 0, stream,
        static_cast<const __nv_bfloat16*>(pool), block_table, length, num_kv_heads, head_dim,
        block_size, num_blocks, static_cast<__nv_bfloat16*>(out), dev_status);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_gather_kv: dtype %d", dtype);
  }
  return check_launch("kve_gather_kv");
}

extern "C" int kve_embed(const int32_t* ids, int n_tokens, const void* table, int dtype, int hidden,
                         int vocab, void* out, int* dev_status, cudaStream_t stream) {
  if (n_tokens < 0 || hidden < 1 || vocab < 1) return set_error(KVE_ERR_ARG, "kve_embed: bad sizes");
  if (n_tokens == 0) return KVE_OK;
  if (!ids || !table || !out) return set_error(KVE_ERR_ARG, "kve_embed: null pointer");
  if (dtype == KVE_F32) {
    launch_kernel(embed_kernel<float>, dim3(n_tokens), dim3(256), 0, stream, ids, static_cast<const float*>(table), hidden,
                                                      vocab, static_cast<float*>(out), dev_status);
  } else if (dtype == KVE_BF16) {
    launch_kernel(embed_kernel<__nv_bfloat16>, dim3(n_tokens), dim3(256), 0, stream,
        ids, static_cast<const __nv_bfloat16*>(table), hidden, vocab, static_cast<__nv_bfloat16*>(out),
        dev_status);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_embed: dtype %d", dtype);
  }
  return check_launch("kve_embed");
}

int kve::rmsnorm_run(const void* x, int dtype, const float* weight, int rows, int hidden, float eps,
                     const int32_t* row_index, void* out, bool w_static, cudaStream_t stream) {
  if (rows < 0 || hidden < 1) return set_error(KVE_ERR_ARG, "kve_rmsnorm: bad sizes");
  if (rows == 0) return KVE_OK;
  if (!x || !weight || !out) return set_error(KVE_ERR_ARG, "kve_rmsnorm: null pointer");
  if (dtype == KVE_F32) {
    launch_kernel(rmsnorm_kernel<float>, dim3(rows), dim3(kNormThreads), 0, stream,
        static_cast<const float*>(x), weight, hidden, eps, row_index, static_cast<float*>(out), w_static ? 1 : 0);
  } else if (dtype == KVE_BF16) {
    launch_kernel(rmsnorm_kernel<__nv_bfloat16>, dim3(rows), dim3(kNormThreads), 0, stream,
        static_cast<const __nv_bfloat16*>(x), weight, hidden, eps, row_index,
        static_cast<__nv_bfloat16*>(out), w_static ? 1 : 0);
  } else {
    return set_error(KVE_ERR_DTYPE, "kve_rmsnorm: dtype %d", dtype);
  }
  return check_launch("kve_rmsnorm");
}

extern "C" int kve_rmsnorm(const void* x, int dtype, const float* weight, int rows, int hidden, float eps,
                           const int32_t* row_index, void* out, cudaStream_t stream) {
  return rmsnorm_run(x, dtype, weight, rows, hidden, eps, row_index, out, false, stream);
}
