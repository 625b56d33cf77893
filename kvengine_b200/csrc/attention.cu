// Paged multi-query GQA verify attention.
//
// CTA = (context chunk, sequence x kv-head, query tile). All query rows of one
// kv-head group (q tokens x group heads, <= 64 rows) share every K/V tile the
// CTA stages through shared memory, so each K/V byte is read from HBM once per
// query tile. Keys are visited in absolute 32-key tiles; chunks of 512 keys
// run in parallel and are merged in a fixed order by a second kernel. A
// query's result therefore depends only on its own position and keys: the
// draft's 1-row pass and the target's k+1-row pass agree bit for bit.
//
// Softmax is online in fp32 (scores, running max and sum, and the P.V
// accumulator all fp32), masked keys contribute exact zeros.
#include <math.h>

#include "kve_common.cuh"

namespace kve {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kWarps = kAttnThreads / 32;
constexpr int kKeyTile = 32;
constexpr int kChunk = 512;
constexpr int kMaxRows = 64;
constexpr int kRowsPerWarp = kMaxRows / kWarps;

struct AttnParams {
  const void* q;
  const void* pool_k;
  const void* pool_v;
  const int32_t* tables;
  int table_stride;
  const int32_t* ctx_lens;
  const int32_t* q_lens;
  const int32_t* q_offsets;
  int nq, nkv, group, qt;  // qt = query tokens per tile
  int bs;
  int64_t num_blocks;
  float scale;
  void* out;
  float* ws;  // split mode partials, null otherwise
  int n_chunks, n_qtiles;
  int* status;
};

__host__ __device__ inline size_t partial_floats(int hd) { return (size_t)kMaxRows * (hd + 2); }

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnThreads)
paged_attn_kernel(AttnParams p) {
  constexpr int DPL = HD / 32;  // output dims per lane
  constexpr int VEC = 16 / sizeof(T);
  constexpr int VPR = HD / VEC;  // 16-byte vectors per key row
  extern __shared__ float smem[];
  float* qs = smem;                          // [kMaxRows][HD]
  float* ks = qs + kMaxRows * HD;            // [kKeyTile][HD + 1]
  float* vs = ks + kKeyTile * (HD + 1);      // [kKeyTile][HD]

  const int c = blockIdx.x, bh = blockIdx.y, qtile = blockIdx.z;
  const int b = bh / p.nkv, h = bh % p.nkv;
  const int ctx = p.ctx_lens[b], ql = p.q_lens[b], qoff = p.q_offsets[b];
  if (ql < 0 || ctx < ql || ctx > p.table_stride * p.bs) {
    if (threadIdx.x == 0 && c == 0 && qtile == 0) report(p.status, KVE_ERR_BOUNDS);
    return;
  }
  const int t0 = qtile * p.qt;
  if (t0 >= ql) return;
  const int nt = min(p.qt, ql - t0);
  const int rows = nt * p.group;
  const int first_pos = ctx - ql + t0;
  const int last_pos = first_pos + nt - 1;
  const int key_lo = c * kChunk;
  if (key_lo > last_pos) return;  // no row of this tile reads this chunk
  const int key_hi = min(min(ctx, key_lo + kChunk), last_pos + 1);

  const T* q = static_cast<const T*>(p.q);
  const T* pk = static_cast<const T*>(p.pool_k);
  const T* pv = static_cast<const T*>(p.pool_v);
  for (int i = threadIdx.x; i < rows * HD; i += kAttnThreads) {
    int r = i / HD, d = i % HD;
    int t = r / p.group, g = r % p.group;
    qs[i] = Elem<T>::to_f(q[((size_t)(qoff + t0 + t) * p.nq + h * p.group + g) * HD + d]);
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float m[kRowsPerWarp], l[kRowsPerWarp], acc[kRowsPerWarp][DPL];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i) {
    m[i] = -INFINITY; l[i] = 0.f;
#pragma unroll
    for (int dd = 0; dd < DPL; ++dd) acc[i][dd] = 0.f;
  }
  const int32_t* table = p.tables + (size_t)b * p.table_stride;

  for (int kt = key_lo; kt < key_hi; kt += kKeyTile) {
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * kKeyTile * VPR; i += kAttnThreads) {
      bool is_v = i >= kKeyTile * VPR;
      int j = is_v ? i - kKeyTile * VPR : i;
      int kk = j / VPR, vec = j % VPR;
      int key = kt + kk;
      float vals[VEC];
      bool ok = key < key_hi;
      int64_t blk = ok ? table[key / p.bs] : 0;
      if (ok && (blk < 0 || blk >= p.num_blocks)) { report(p.status, KVE_ERR_BOUNDS); ok = false; }
      if (ok) {
        size_t base = (((size_t)blk * p.bs + key % p.bs) * p.nkv + h) * HD + vec * VEC;
        uint4 raw = *reinterpret_cast<const uint4*>((is_v ? pv : pk) + base);
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int u = 0; u < VEC; ++u) vals[u] = Elem<T>::to_f(e[u]);
      } else {
#pragma unroll
        for (int u = 0; u < VEC; ++u) vals[u] = 0.f;
      }
      float* dst = is_v ? vs + kk * HD + vec * VEC : ks + kk * (HD + 1) + vec * VEC;
#pragma unroll
      for (int u = 0; u < VEC; ++u) dst[u] = vals[u];
    }
    __syncthreads();
    const int key = kt + lane;
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * kWarps;
      if (r >= rows) break;
      const int pos = first_pos + r / p.group;
      float s = -INFINITY;
      if (key < key_hi && key <= pos) {
        const float* qr = qs + r * HD;
        const float* kr = ks + lane * (HD + 1);
        float dot = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; ++d) dot = fmaf(qr[d], kr[d], dot);
        s = dot * p.scale;
      }
      float tmax = warp_max(s);
      if (tmax == -INFINITY) continue;  // whole tile masked for this row
      float m_new = fmaxf(m[i], tmax);
      float corr = expf(m[i] - m_new);
      float pr = (s == -INFINITY) ? 0.f : expf(s - m_new);
      l[i] = l[i] * corr + warp_sum(pr);
#pragma unroll
      for (int dd = 0; dd < DPL; ++dd) acc[i][dd] *= corr;
#pragma unroll 8
      for (int j = 0; j < kKeyTile; ++j) {
        float pj = __shfl_sync(0xffffffffu, pr, j);
        const float* vr = vs + j * HD + lane;
#pragma unroll
        for (int dd = 0; dd < DPL; ++dd) acc[i][dd] = fmaf(pj, vr[dd * 32], acc[i][dd]);
      }
      m[i] = m_new;
    }
  }

  if (p.ws == nullptr) {
    T* out = static_cast<T*>(p.out);
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * kWarps;
      if (r >= rows) break;
      int t = r / p.group, g = r % p.group;
      T* o = out + ((size_t)(qoff + t0 + t) * p.nq + h * p.group + g) * HD;
#pragma unroll
      for (int dd = 0; dd < DPL; ++dd) o[lane + dd * 32] = Elem<T>::from_f(acc[i][dd] / l[i]);
    }
  } else {
    float* part = p.ws + ((((size_t)bh * p.n_qtiles + qtile) * p.n_chunks) + c) * partial_floats(HD);
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
      const int r = warp + i * kWarps;
      if (r >= rows) break;
      float* pr = part + (size_t)r * (HD + 2);
#pragma unroll
      for (int dd = 0; dd < DPL; ++dd) pr[lane + dd * 32] = acc[i][dd];
      if (lane == 0) { pr[HD] = m[i]; pr[HD + 1] = l[i]; }
    }
  }
}

// Merge chunk partials in chunk order. A row at position pos reads chunks
// 0 .. pos / kChunk; with a single chunk this reproduces acc / l exactly.
template <typename T, int HD>
__global__ void __launch_bounds__(kAttnThreads)
attn_combine_kernel(AttnParams p) {
  constexpr int DPL = HD / 32;
  const int bh = blockIdx.x, qtile = blockIdx.y;
  const int b = bh / p.nkv, h = bh % p.nkv;
  const int ctx = p.ctx_lens[b], ql = p.q_lens[b], qoff = p.q_offsets[b];
  if (ql < 0 || ctx < ql || ctx > p.table_stride * p.bs) return;
  const int t0 = qtile * p.qt;
  if (t0 >= ql) return;
  const int nt = min(p.qt, ql - t0);
  const int rows = nt * p.group;
  const int first_pos = ctx - ql + t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = p.ws + (((size_t)bh * p.n_qtiles + qtile) * p.n_chunks) * partial_floats(HD);
  T* out = static_cast<T*>(p.out);
  for (int r = warp; r < rows; r += kWarps) {
    const int pos = first_pos + r / p.group;
    const int live = pos / kChunk + 1;
    float mx = -INFINITY;
    for (int c = 0; c < live; ++c) mx = fmaxf(mx, base[c * partial_floats(HD) + (size_t)r * (HD + 2) + HD]);
    float lsum = 0.f, acc[DPL];
#pragma unroll
    for (int dd = 0; dd < DPL; ++dd) acc[dd] = 0.f;
    for (int c = 0; c < live; ++c) {
      const float* pr = base + c * partial_floats(HD) + (size_t)r * (HD + 2);
      float w = expf(pr[HD] - mx);
      lsum += pr[HD + 1] * w;
#pragma unroll
      for (int dd = 0; dd < DPL; ++dd) acc[dd] += pr[lane + dd * 32] * w;
    }
    int t = r / p.group, g = r % p.group;
    T* o = out + ((size_t)(qoff + t0 + t) * p.nq + h * p.group + g) * HD;
#pragma unroll
    for (int dd = 0; dd < DPL; ++dd) o[lane + dd * 32] = Elem<T>::from_f(acc[dd] / lsum);
  }
}

template <typename T, int HD>
int launch(AttnParams& p, int batch, cudaStream_t stream) {
  size_t smem = sizeof(float) * ((size_t)kMaxRows * HD + kKeyTile * (HD + 1) + kKeyTile * HD);
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(paged_attn_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured = true;
  }
  dim3 grid(p.n_chunks, batch * p.nkv, p.n_qtiles);
  paged_attn_kernel<T, HD><<<grid, kAttnThreads, smem, stream>>>(p);
  int rc = check_launch("kve_paged_verify_attn");
  if (rc || !p.ws) return rc;
  attn_combine_kernel<T, HD><<<dim3(batch * p.nkv, p.n_qtiles), kAttnThreads, 0, stream>>>(p);
  return check_launch("kve_paged_verify_attn(combine)");
}

int qtile_tokens(int group) { return group >= kMaxRows ? 1 : kMaxRows / group; }

}  // namespace
}  // namespace kve

using namespace kve;

extern "C" size_t kve_paged_attn_workspace_bytes(int batch, int max_q_len, int max_ctx, int num_heads,
                                                 int num_kv_heads, int head_dim) {
  if (batch <= 0 || num_kv_heads <= 0 || max_ctx <= kChunk || head_dim <= 0) return 0;
  int group = num_heads / num_kv_heads;
  int qt = qtile_tokens(group);
  size_t n_qtiles = (max_q_len + qt - 1) / qt;
  size_t n_chunks = (max_ctx + kChunk - 1) / kChunk;
  return (size_t)batch * num_kv_heads * n_qtiles * n_chunks * partial_floats(head_dim) * sizeof(float);
}

extern "C" int kve_paged_verify_attn(const void* q, int dtype, const void* pool_k, const void* pool_v,
                                     const int32_t* block_tables, int table_stride, const int32_t* ctx_lens,
                                     const int32_t* q_lens, const int32_t* q_offsets, int batch,
                                     int max_q_len, int max_ctx, int num_heads, int num_kv_heads,
                                     int head_dim, int block_size, int64_t num_blocks, float scale,
                                     void* out, void* workspace, size_t workspace_bytes, int* dev_status,
                                     cudaStream_t stream) {
  if (batch < 0 || max_q_len < 0 || max_ctx < 0 || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads || block_size < 1 || table_stride < 1 || num_blocks < 1)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: bad sizes");
  if (batch == 0 || max_q_len == 0) return KVE_OK;
  if (head_dim != 64 && head_dim != 128)
    return set_error(KVE_ERR_SHAPE, "kve_paged_verify_attn: head_dim %d (supported: 64, 128)", head_dim);
  int group = num_heads / num_kv_heads;
  if (group > kMaxRows) return set_error(KVE_ERR_SHAPE, "kve_paged_verify_attn: group %d > %d", group, kMaxRows);
  if (!q || !pool_k || !pool_v || !block_tables || !ctx_lens || !q_lens || !q_offsets || !out)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: null pointer");
  if ((uintptr_t)pool_k % 16 || (uintptr_t)pool_v % 16)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: pool pointers must be 16-byte aligned");
  AttnParams p{};
  p.q = q; p.pool_k = pool_k; p.pool_v = pool_v; p.tables = block_tables; p.table_stride = table_stride;
  p.ctx_lens = ctx_lens; p.q_lens = q_lens; p.q_offsets = q_offsets;
  p.nq = num_heads; p.nkv = num_kv_heads; p.group = group; p.qt = qtile_tokens(group);
  p.bs = block_size; p.num_blocks = num_blocks; p.scale = scale; p.out = out; p.status = dev_status;
  p.n_qtiles = (max_q_len + p.qt - 1) / p.qt;
  p.n_chunks = (max_ctx + kChunk - 1) / kChunk;
  if (p.n_chunks < 1) p.n_chunks = 1;
  p.ws = nullptr;
  if (p.n_chunks > 1) {
    size_t need = kve_paged_attn_workspace_bytes(batch, max_q_len, max_ctx, num_heads, num_kv_heads, head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(KVE_ERR_WORKSPACE, "kve_paged_verify_attn: workspace needs %zu bytes", need);
    p.ws = static_cast<float*>(workspace);
  }
  if (dtype == KVE_F32) {
    return head_dim == 64 ? launch<float, 64>(p, batch, stream) : launch<float, 128>(p, batch, stream);
  } else if (dtype == KVE_BF16) {
    return head_dim == 64 ? launch<__nv_bfloat16, 64>(p, batch, stream)
                          : launch<__nv_bfloat16, 128>(p, batch, stream);
  }
  return set_error(KVE_ERR_DTYPE, "kve_paged_verify_attn: dtype %d", dtype);
}
