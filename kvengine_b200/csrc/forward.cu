// kve_forward: the launch sequence of one model pass over a ragged batch.
// Host code only; every kernel it launches is one of the library's entry points (the GEMMs
// through gemm_run, which may request the constant weights before the previous kernel ends).
#include "gemm_epilogue.cuh"
#include "passes.cuh"

#include <cstring>
#include <vector>

namespace {

inline size_t max3(size_t a, size_t b, size_t c) { return a > b ? (a > c ? a : c) : (b > c ? b : c); }

#define KVE_TRY(expr)          \
  do {                         \
    int _rc = (expr);          \
    if (_rc != KVE_OK) return _rc; \
  } while (0)

}  // namespace

using namespace kve;

extern "C" size_t kve_forward_gemm_ws_bytes(const kve_model_t* m, int n_tokens, int n_out) {
  if (!m || n_tokens <= 0) return 0;
  int qkv = (m->num_heads + 2 * m->num_kv_heads) * m->head_dim;
  int q = m->num_heads * m->head_dim;
  size_t a = kve_gemm_workspace_bytes(n_tokens, qkv, m->hidden, m->dtype);
  size_t b = kve_gemm_workspace_bytes(n_tokens, m->hidden, q, m->dtype);
  size_t c = kve_gemm_workspace_bytes(n_tokens, 2 * m->intermediate, m->hidden, m->dtype);
  size_t d = kve_gemm_workspace_bytes(n_tokens, m->hidden, m->intermediate, m->dtype);
  size_t e = n_out > 0 ? kve_gemm_workspace_bytes(n_out, m->vocab, m->hidden, m->dtype) : 0;
  size_t r = max3(a, b, c);
  return max3(r, d, e);
}

extern "C" size_t kve_forward_attn_ws_bytes(const kve_model_t* m, int n_seqs, int max_q_len, int max_ctx) {
  if (!m) return 0;
  return kve_paged_attn_workspace_bytes(n_seqs, max_q_len, max_ctx, m->num_heads, m->num_kv_heads, m->head_dim);
}

// Layers [l0, l1) of a pass: the embedding when l0 == 0, the final norm and the
// vocabulary projection when l1 == num_layers (kve_forward is the whole range).
extern "C" int kve_forward_layers(const kve_model_t* m, const kve_batch_t* b, const kve_scratch_t* s, int l0,
                                  int l1, cudaStream_t stream) {
  if (!m || !b || !s || !m->layers) return set_error(KVE_ERR_ARG, "kve_forward: null argument");
  if (l0 < 0 || l1 > m->num_layers || l0 > l1)
    return set_error(KVE_ERR_ARG, "kve_forward_layers: bad layer range [%d, %d)", l0, l1);
  if (b->n_tokens < 0 || b->n_seqs < 0 || b->n_out < 0)
    return set_error(KVE_ERR_ARG, "kve_forward: bad batch sizes");
  if (b->n_tokens == 0) return KVE_OK;
  const int dt = m->dtype;
  const int H = m->hidden, M = b->n_tokens;
  const int qsz = m->num_heads * m->head_dim;
  const int qkv = qsz + 2 * m->num_kv_heads * m->head_dim;
  const int64_t num_slots = m->num_blocks * m->block_size;
  const float scale = 1.0f / sqrtf((float)m->head_dim);

  // The fused qkv epilogue needs bf16, 16-byte aligned outputs and heads that
  // tile 128-feature blocks; otherwise the projection and the RoPE append run apart.
  const int hd = m->head_dim;
  const bool fused_qkv = dt == KVE_BF16 && hd % 8 == 0 && 128 % hd == 0 && m->rope_len > 0 &&
                         (uintptr_t)s->q % 16 == 0 && (uintptr_t)m->rope_cos % 16 == 0 &&
                         (uintptr_t)m->rope_sin % 16 == 0;

  if (l0 == 0) KVE_TRY(kve_embed(b->ids, M, m->embed, dt, H, m->vocab, s->hidden, s->dev_status, stream));
  for (int l = l0; l < l1; ++l) {
    const kve_layer_t& L = m->layers[l];
    KVE_TRY(rmsnorm_run(s->hidden, dt, L.ln1, M, H, m->rms_eps, nullptr, s->normed, true, stream));
    if (fused_qkv) {
      // bf16: projection, bias, RoPE and the K/V append in one kernel.
      EpiArgs e{};
      e.bias = L.b_qkv;
      e.w_static = 1;
      e.nq = m->num_heads; e.nkv = m->num_kv_heads; e.hd = m->head_dim;
      e.positions = b->positions; e.slots = b->slots;
      e.rope_cos = m->rope_cos; e.rope_sin = m->rope_sin; e.rope_len = m->rope_len;
      e.q_out = s->q; e.pool_k = L.pool_k; e.pool_v = L.pool_v; e.num_slots = num_slots;
      e.status = s->dev_status;
      KVE_TRY(gemm_qkv_rope(s->normed, L.w_qkv, M, qkv, H, e, stream));
    } else {
      KVE_TRY(gemm_run(s->normed, L.w_qkv, dt, M, qkv, H, KVE_EPI_BIAS, L.b_qkv, nullptr, s->qkv, dt,
                       s->gemm_ws, s->gemm_ws_bytes, s->dev_status, KVE_GEMM_AUTO, true, stream));
      KVE_TRY(kve_qkv_rope_append(s->qkv, dt, M, m->num_heads, m->num_kv_heads, m->head_dim, b->positions,
                                  b->slots, m->rope_cos, m->rope_sin, m->rope_len, s->q, L.pool_k, L.pool_v,
                                  num_slots, s->dev_status, stream));
    }
    KVE_TRY(paged_attn_run(s->q, dt, L.pool_k, L.pool_v, b->block_tables, b->table_stride, b->ctx_lens,
                                  b->q_lens, b->q_offsets, b->n_seqs, b->max_q_len, b->max_ctx, m->num_heads,
                                  m->num_kv_heads, m->head_dim, m->block_size, m->num_blocks, scale, s->attn,
                                  s->attn_ws, s->attn_ws_bytes, s->dev_status, true, stream));
    KVE_TRY(gemm_run(s->attn, L.w_o, dt, M, H, qsz, KVE_EPI_RESIDUAL, nullptr, s->hidden, s->hidden, dt,
                     s->gemm_ws, s->gemm_ws_bytes, s->dev_status, KVE_GEMM_AUTO, true, stream));
    KVE_TRY(rmsnorm_run(s->hidden, dt, L.ln2, M, H, m->rms_eps, nullptr, s->normed, true, stream));
    KVE_TRY(gemm_run(s->normed, L.w_gu, dt, M, 2 * m->intermediate, H, KVE_EPI_SILU_MUL, nullptr, nullptr,
                     s->act, dt, s->gemm_ws, s->gemm_ws_bytes, s->dev_status, KVE_GEMM_AUTO, true, stream));
    KVE_TRY(gemm_run(s->act, L.w_down, dt, M, H, m->intermediate, KVE_EPI_RESIDUAL, nullptr, s->hidden,
                     s->hidden, dt, s->gemm_ws, s->gemm_ws_bytes, s->dev_status, KVE_GEMM_AUTO, true, stream));
  }
  if (b->n_out == 0 || l1 < m->num_layers) return KVE_OK;
  KVE_TRY(rmsnorm_run(s->hidden, dt, m->final_norm, b->n_out, H, m->rms_eps, b->out_rows, s->out_normed, true, stream));
  KVE_TRY(gemm_run(s->out_normed, m->lm_head, dt, b->n_out, m->vocab, H, KVE_EPI_STORE, nullptr, nullptr,
                   b->logits, b->logits_dtype, s->gemm_ws, s->gemm_ws_bytes, s->dev_status, KVE_GEMM_AUTO, true, stream));
  return KVE_OK;
}

extern "C" int kve_forward(const kve_model_t* m, const kve_batch_t* b, const kve_scratch_t* s,
                           cudaStream_t stream) {
  if (!m) return set_error(KVE_ERR_ARG, "kve_forward: null argument");
  return kve_forward_layers(m, b, s, 0, m->num_layers, stream);
}

// kve_forward recorded into a CUDA graph and launched as one: the pass's ~170 kernel
// launches (programmatic dependent launches become programmatic graph edges) reach
// the GPU without the per-launch work of a stream launch.
//
// The caller's slot holds a GraphSlot: the executable graph plus the signature of
// the capture it was made from - per node its type and, for kernel nodes, the
// function, block shape, dynamic shared memory and cluster shape. A later capture
// with the same signature (same kernels, new pointers, sizes and grids) updates the
// executable graph in place; any other capture re-instantiates it. Updating in place
// across a change of kernel function, block shape or cluster shape (the attention
// kernel's row blocks and the GEMMs' launch shapes depend on the batch) was measured
// to leave some launches stale on this driver: a pass recorded for a prompt-sized
// batch and then for a decode-sized one gave wrong results after the update.
namespace {

struct GraphSlot {
  cudaGraphExec_t exec = nullptr;
  std::vector<uint64_t> sig;
};

// False if some node could not be queried (the caller then re-instantiates).
bool graph_signature(cudaGraph_t g, std::vector<uint64_t>& sig) {
  sig.clear();
  size_t n = 0;
  if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess) return false;
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return false;
  size_t edges = 0;
  if (cudaGraphGetEdges(g, nullptr, nullptr, &edges) != cudaSuccess) return false;
  sig.reserve(n * 5 + 2);
  sig.push_back(n);
  sig.push_back(edges);
  for (cudaGraphNode_t node : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(node, &t) != cudaSuccess) return false;
    sig.push_back((uint64_t)t);
    if (t != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams kp;
    if (cudaGraphKernelNodeGetParams(node, &kp) != cudaSuccess) return false;
    sig.push_back((uint64_t)(uintptr_t)kp.func);
    sig.push_back((uint64_t)kp.blockDim.x | (uint64_t)kp.blockDim.y << 21 | (uint64_t)kp.blockDim.z << 42);
    sig.push_back((uint64_t)kp.sharedMemBytes);
    cudaKernelNodeAttrValue v;
    memset(&v, 0, sizeof(v));
    if (cudaGraphKernelNodeGetAttribute(node, cudaKernelNodeAttributeClusterDimension, &v) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    sig.push_back((uint64_t)v.clusterDim.x | (uint64_t)v.clusterDim.y << 21 | (uint64_t)v.clusterDim.z << 42);
  }
  return true;
}

}  // namespace

extern "C" int kve_forward_layers_graphed(const kve_model_t* m, const kve_batch_t* b, const kve_scratch_t* s,
                                          int l0, int l1, void** graph_slot, cudaStream_t stream) {
  if (!graph_slot) return set_error(KVE_ERR_ARG, "kve_forward_graphed: null graph slot");
  if (!m || !b || !s) return set_error(KVE_ERR_ARG, "kve_forward_graphed: null argument");
  if (l0 < 0 || l1 > m->num_layers || l0 > l1)
    return set_error(KVE_ERR_ARG, "kve_forward_layers_graphed: bad layer range [%d, %d)", l0, l1);
  if (b->n_tokens == 0) return KVE_OK;
  cudaError_t e = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(KVE_ERR_CUDA, "kve_forward_graphed: stream capture: %s", cudaGetErrorString(e));
  }
  const int rc = kve_forward_layers(m, b, s, l0, l1, stream);
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(stream, &graph);
  if (rc != KVE_OK || e != cudaSuccess || !graph) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc != KVE_OK ? rc : set_error(KVE_ERR_CUDA, "kve_forward_graphed: end capture: %s", cudaGetErrorString(e));
  }
  GraphSlot* slot = static_cast<GraphSlot*>(*graph_slot);
  if (!slot) {
    slot = new GraphSlot();
    *graph_slot = slot;
  }
  std::vector<uint64_t> sig;
  const bool sig_ok = graph_signature(graph, sig);
  bool updated = false;
  if (slot->exec && sig_ok && sig == slot->sig) {
    cudaGraphExecUpdateResultInfo info;
    updated = cudaGraphExecUpdate(slot->exec, graph, &info) == cudaSuccess;
    if (!updated) cudaGetLastError();
  }
  if (!updated) {
    if (slot->exec) cudaGraphExecDestroy(slot->exec);
    slot->exec = nullptr;
    slot->sig.clear();
    e = cudaGraphInstantiate(&slot->exec, graph, 0);
    if (e != cudaSuccess) {
      slot->exec = nullptr;
      cudaGraphDestroy(graph);
      cudaGetLastError();
      return set_error(KVE_ERR_CUDA, "kve_forward_graphed: instantiate: %s", cudaGetErrorString(e));
    }
    if (sig_ok) slot->sig.swap(sig);
  }
  cudaGraphDestroy(graph);
  e = cudaGraphLaunch(slot->exec, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(KVE_ERR_CUDA, "kve_forward_graphed: launch: %s", cudaGetErrorString(e));
  }
  return KVE_OK;
}

extern "C" int kve_forward_graphed(const kve_model_t* m, const kve_batch_t* b, const kve_scratch_t* s,
                                   void** graph_slot, cudaStream_t stream) {
  if (!m) return set_error(KVE_ERR_ARG, "kve_forward_graphed: null argument");
  return kve_forward_layers_graphed(m, b, s, 0, m->num_layers, graph_slot, stream);
}

extern "C" int kve_forward_graph_free(void* graph_slot) {
  GraphSlot* slot = static_cast<GraphSlot*>(graph_slot);
  if (!slot) return KVE_OK;
  if (slot->exec) cudaGraphExecDestroy(slot->exec);
  delete slot;
  return KVE_OK;
}
