/*
 * kvengine_b200 — C ABI of the B200 (sm_100a) speculative-decoding verify path.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t,
 * launches asynchronously on that stream and returns an int status
 * (KVE_OK == 0, negative on error; kve_last_error() has the message).
 * Nothing here allocates device memory or throws: buffers and workspaces are
 * owned by the caller. A workspace must be zero-filled once before its first
 * use; the kernels leave it zeroed again when they finish.
 *
 * Device-side checks (an out-of-range slot or block id, a wait that ran out)
 * never trap: the kernel skips the access and writes the first error code into
 * `dev_status` (an int in device memory, may be NULL), which the caller reads.
 *
 * Each entry point names the reference code (kvengine, file:line) it replaces.
 */
#ifndef KVENGINE_B200_H
#define KVENGINE_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  KVE_OK = 0,
  KVE_ERR_ARG = -1,        /* bad pointer, size or enum */
  KVE_ERR_SHAPE = -2,      /* unsupported shape (e.g. head_dim not 64/128) */
  KVE_ERR_DTYPE = -3,      /* unsupported dtype */
  KVE_ERR_CUDA = -4,       /* a CUDA runtime/driver call failed */
  KVE_ERR_TIMEOUT = -5,    /* a bounded device-side wait gave up */
  KVE_ERR_WORKSPACE = -6,  /* workspace missing or too small */
  KVE_ERR_BOUNDS = -7      /* device side: slot / block / token id out of range */
};

enum { KVE_F32 = 0, KVE_BF16 = 1 };

/* GEMM epilogues: out[m, :] from acc[m, :] = sum_k x[m,k] * w[n,k].
 *   STORE     out = round(acc)
 *   BIAS      out = round(acc + bias[n])                (q/k/v projections)
 *   RESIDUAL  out = round(residual + round(acc))        (o_proj, down_proj + residual add;
 *                                                        out may alias residual)
 *   SILU_MUL  w rows interleaved (2j = gate_j, 2j+1 = up_j); out has n/2 columns,
 *             out[m, j] = round(round(silu(round(gate))) * round(up))   (Qwen2MLP) */
enum { KVE_EPI_STORE = 0, KVE_EPI_BIAS = 1, KVE_EPI_RESIDUAL = 2, KVE_EPI_SILU_MUL = 3 };

/* GEMM kernel selection for kve_gemm_ex: AUTO = tcgen05 for bf16, SIMT for fp32. */
enum { KVE_GEMM_AUTO = 0, KVE_GEMM_SIMT = 1, KVE_GEMM_TCGEN05 = 2 };

int kve_version(void);
const char* kve_last_error(void);
/* Number of kernels this library has launched in this process (for launch accounting). */
unsigned long long kve_launch_count(void);

/* Fused greedy acceptance.
 * Replaces kvengine/speculative.py:167-182: `target_preds = argmax(t_logits[u-1:])`
 * over the k+1 verify rows, the longest prefix with preds[j] == drafts[j], and the
 * emitted tokens drafts[:n] + [preds[n]] (preds[k] is the bonus when n == k).
 * logits: [batch, k+1, vocab] rows `row_stride` elements apart (fp32 or bf16).
 * drafts: int32, draft j of sequence b at drafts[b * draft_stride_b + j * draft_stride_j]
 * ([batch, k] row-major is stride_b = k, stride_j = 1).
 * Outputs (int32): preds [batch, k+1], n_accepted [batch], emitted [batch, k+1]
 * (entries past n are -1). argmax ties resolve to the lowest index and NaN counts
 * as the maximum, as torch.argmax does. 1 <= k <= 31. */
size_t kve_greedy_accept_workspace_bytes(int batch);
int kve_greedy_accept(const void* logits, int dtype, int64_t row_stride, const int32_t* drafts,
                      int64_t draft_stride_b, int64_t draft_stride_j, int batch, int k, int vocab,
                      int32_t* out_preds, int32_t* out_n_accepted, int32_t* out_emitted,
                      void* workspace, size_t workspace_bytes, int* dev_status, cudaStream_t stream);

/* Allocation-free variant of kve_greedy_accept: same arguments and results,
 * minus the workspace. It has no counterpart in kvengine; it exists for callers
 * that cannot allocate device memory at the call site (plain C/FFI hosts without
 * a device allocator, code inside a CUDA-graph capture, fixed-budget serving
 * loops). Its per-sequence counters live in a static device array of
 * kve_greedy_accept_noalloc_max_batch() entries (4096); a larger batch returns
 * KVE_ERR_ARG without launching. The array starts at zero and every completed
 * call leaves it at zero. All calls on one device share it, so calls must not
 * overlap in time (keep them on one stream). The array's device address is
 * looked up on the first call on each device; make that first call outside a
 * stream capture. */
int kve_greedy_accept_noalloc_max_batch(void);
int kve_greedy_accept_noalloc(const void* logits, int dtype, int64_t row_stride, const int32_t* drafts,
                              int64_t draft_stride_b, int64_t draft_stride_j, int batch, int k, int vocab,
                              int32_t* out_preds, int32_t* out_n_accepted, int32_t* out_emitted,
                              cudaStream_t stream);

/* Row argmax. Replaces the draft's `int(torch.argmax(logits[-1]))`
 * (kvengine/speculative.py:155) and greedy decoding's argmax (kvengine/decode.py:303).
 * x: [rows, cols] with `row_stride`; out: [rows] int32. Same tie/NaN rule as above. */
int kve_argmax_rows(const void* x, int dtype, int rows, int cols, int64_t row_stride,
                    int32_t* out, cudaStream_t stream);

/* kve_argmax_rows that also writes row i's result to scatter_out[scatter_idx[i]]
 * (0 <= scatter_idx[i] < scatter_len; an index outside that range is skipped and
 * KVE_ERR_BOUNDS is recorded in *dev_status, which may be NULL). Replaces the
 * reference's host-side assembly of the verify feed `unseen + drafts`
 * (kvengine/speculative.py:155,160-162): each draft lands in its slot of the
 * verify pass's token ids on the device. */
int kve_argmax_rows_scatter(const void* x, int dtype, int rows, int cols, int64_t row_stride, int32_t* out,
                            const int32_t* scatter_idx, int32_t* scatter_out, int64_t scatter_len, int* dev_status,
                            cudaStream_t stream);

/* KV append: pool[slot_ids[t]] = new[t] for the K and V of one layer.
 * Replaces `pool.k_flat[layer].index_copy_(0, slots, k_src)` and the V twin,
 * kvengine/paged.py:310-311. k_new, v_new: [n_tokens, num_kv_heads, head_dim];
 * pool_k, pool_v: the layer's flat view [num_slots, num_kv_heads, head_dim]
 * (num_slots = num_blocks * block_size). Slots outside [0, num_slots) are skipped
 * and reported as KVE_ERR_BOUNDS. */
int kve_kv_append(const void* k_new, const void* v_new, int dtype, const int64_t* slot_ids,
                  int n_tokens, int num_kv_heads, int head_dim, void* pool_k, void* pool_v,
                  int64_t num_slots, int* dev_status, cudaStream_t stream);

/* Fused rotary embedding + KV append for one layer.
 * Replaces kvengine/forward.py:193-201: splitting the q/k/v projection output,
 * `apply_rope` (forward.py:55-69, rotate-half pairing with cos/sin cast to the
 * model dtype) and `cache.write`'s scatter (paged.py:310-311).
 * qkv: [n_tokens, (num_heads + 2*num_kv_heads) * head_dim] (bias already added);
 * positions, slots: [n_tokens] int32; rope_cos/sin: [rope_len, head_dim/2] fp32;
 * q_out: [n_tokens, num_heads, head_dim]; pool_k/v as for kve_kv_append. */
int kve_qkv_rope_append(const void* qkv, int dtype, int n_tokens, int num_heads, int num_kv_heads,
                        int head_dim, const int32_t* positions, const int32_t* slots,
                        const float* rope_cos, const float* rope_sin, int rope_len, void* q_out,
                        void* pool_k, void* pool_v, int64_t num_slots, int* dev_status,
                        cudaStream_t stream);

/* Paged multi-query GQA verify attention, reading K/V blocks in place.
 * Replaces the gather kvengine/paged.py:315-331 plus kvengine/forward.py:72-144
 * (`repeat_kv`, `causal_mask`, `attend`): query row i of sequence b sits at
 * position ctx_lens[b] - q_lens[b] + i and attends keys [0, position].
 * q: [sum(q_lens), num_heads, head_dim] with sequence b's rows at q_offsets[b];
 * pool_k/v: the layer's [num_blocks, block_size, num_kv_heads, head_dim];
 * block_tables: [batch, table_stride] int32; out like q. head_dim in {64, 128}.
 * Long contexts are split into fixed 512-key chunks combined in a fixed order
 * (the result for a query depends only on its own keys, not on the batch). */
size_t kve_paged_attn_workspace_bytes(int batch, int max_q_len, int max_ctx, int num_heads,
                                      int num_kv_heads, int head_dim);
int kve_paged_verify_attn(const void* q, int dtype, const void* pool_k, const void* pool_v,
                          const int32_t* block_tables, int table_stride, const int32_t* ctx_lens,
                          const int32_t* q_lens, const int32_t* q_offsets, int batch, int max_q_len,
                          int max_ctx, int num_heads, int num_kv_heads, int head_dim, int block_size,
                          int64_t num_blocks, float scale, void* out, void* workspace,
                          size_t workspace_bytes, int* dev_status, cudaStream_t stream);

/* Contiguous K/V history of one sequence: out[h, t, :] = pool[table[t / bs], t % bs, h, :]
 * for t < length. Replaces kvengine/paged.py:315-331 (`_gather`) where a caller
 * still wants the materialised history (the KVCacheLike `write` return value). */
int kve_gather_kv(const void* pool, int dtype, const int32_t* block_table, int length,
                  int num_kv_heads, int head_dim, int block_size, int64_t num_blocks, void* out,
                  int* dev_status, cudaStream_t stream);

/* Token embedding gather. Replaces `inner.embed_tokens(input_ids)`, kvengine/forward.py:176. */
int kve_embed(const int32_t* ids, int n_tokens, const void* table, int dtype, int hidden, int vocab,
              void* out, int* dev_status, cudaStream_t stream);

/* RMSNorm (Qwen2RMSNorm): out = w * round(x * rsqrt(mean(x^2) + eps)), computed in fp32.
 * Replaces input_layernorm / post_attention_layernorm / model.norm,
 * kvengine/forward.py:191,207,212. Optional row_index [rows] gathers input rows
 * (the final norm runs only on the rows whose logits are needed). */
int kve_rmsnorm(const void* x, int dtype, const float* weight, int rows, int hidden, float eps,
                const int32_t* row_index, void* out, cudaStream_t stream);

/* Linear layer y = x w^T with a fused epilogue (see KVE_EPI_*).
 * Replaces the nn.Linear calls of kvengine/forward.py:194-196 (q/k/v), :204 (o_proj),
 * :207 (Qwen2MLP gate/up/down) and :215 (lm_head).
 * x: [m, k]; w: [n, k] (row-major, k contiguous); out: [m, n] (or [m, n/2] for
 * SILU_MUL) in out_dtype. bf16 runs on tcgen05 tensor cores (fp32 accumulate in
 * TMEM), fp32 on a CUDA-core kernel whose per-element reduction order does not
 * depend on m (draft and verify passes of the same model agree bit for bit). */
size_t kve_gemm_workspace_bytes(int m, int n, int k, int dtype);
int kve_gemm(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue,
             const float* bias, const void* residual, void* out, int out_dtype, void* workspace,
             size_t workspace_bytes, int* dev_status, cudaStream_t stream);
int kve_gemm_ex(const void* x, const void* w, int dtype, int m, int n, int k, int epilogue,
                const float* bias, const void* residual, void* out, int out_dtype, void* workspace,
                size_t workspace_bytes, int* dev_status, int algo, cudaStream_t stream);

/* Tuning and test hook (no kvengine counterpart): force the tcgen05 GEMM's launch
 * shape for later calls in this process: token_tiles (tiles the tokens are cut
 * into), weight_halves (1 or 2 blocks of 128 weight rows per CTA) and k_chunks
 * (1, 2 or 4 64-wide k-chunks per pipeline stage); 0 restores the model's choice
 * for that parameter. A forced value applies only where it is valid for a given
 * GEMM. The split-K factor is never forced, so results are bit-identical under
 * every shape; only speed changes. */
int kve_gemm_force_shape(int token_tiles, int weight_halves, int k_chunks);

/* Tuning hook (no kvengine counterpart): force the tcgen05 GEMM's split-K factor
 * (1..8; 0 restores the model's choice, a function of (n, k) only) for later
 * calls in this process. Unlike the other shape hooks this changes the summation
 * order, hence the low bits of results; it exists for measuring launch shapes. */
int kve_gemm_force_splits(int splits);

/* Tuning and test hook (no kvengine counterpart): whether later tcgen05 GEMMs
 * without split-K, or with split-K inside the CTA, run as CTA pairs (2-CTA MMA on
 * 256-row tiles): 0 = the cost model's choice, 1 = never, 2 = wherever the shape
 * allows. Results are bit-identical either way. */
int kve_gemm_force_pair(int mode);

/* Tuning and test hook (no kvengine counterpart): whether later tcgen05 GEMMs
 * that run one tile per CTA may use 64-row MMA tiles: 0 = only where a CTA's
 * 128-row weight slab would overflow its stage ring and a 64-row one fits
 * (the default), 64 = wherever the shape allows, 128 = never. Results are
 * bit-identical either way. */
int kve_gemm_force_rows(int rows);

/* Tuning and test hook (no kvengine counterpart): whether later tcgen05 GEMMs
 * with split-K compute all of a tile's k-ranges in one CTA or CTA pair (one TMEM
 * accumulator per range, summed in the epilogue) instead of over a cluster of CTAs
 * that exchange their partials: 0 = for prompt-sized batches (m >= 2048, the
 * default), 1 = never, 2 = wherever the shape allows. The ranges and the order
 * of their sum are the same either way, so results are bit-identical. */
int kve_gemm_force_local_split(int mode);

/* Self-test of the device-side timeout path (no kvengine counterpart). Every
 * spin-wait of this library is bounded (2 s) and, when it gives up, records
 * KVE_ERR_TIMEOUT in *dev_status and lets its kernel return instead of hanging the
 * GPU. This launches one thread that waits, through that same bounded mbarrier
 * wait with its limit cut to limit_ns (0 .. 2e9), on a barrier nothing arrives
 * at: afterwards *dev_status holds KVE_ERR_TIMEOUT (if it was 0) and the context
 * is usable. */
int kve_selftest_mbar_timeout(int* dev_status, int64_t limit_ns, cudaStream_t stream);

/* The tcgen05 GEMM's launch plan for an [m, k] x [n, k]^T product with a bf16
 * output (no kvengine counterpart): out[0..12] = split-K factor, token tiles,
 * token groups per tile, tokens per group, weight halves, k-chunks per stage,
 * pipeline stages, 3-D tensor maps (0/1), tiles along the features (of 128 x
 * weight halves rows, or 256 rows for CTA pairs), CTAs launched (fewer than the
 * tiles when CTAs walk several tiles), TMEM accumulators per CTA, CTA pairs (0/1),
 * weight rows per MMA tile (128 or 64). */
int kve_gemm_plan_info(int m, int n, int k, int* out);

/* ------------------------------------------------------------------------
 * Whole forward pass (one call launches every kernel of one model pass).
 * Replaces kvengine/forward.py:147-215 (`forward_with_own_cache`) generalised
 * to a ragged batch: sequence b feeds q_lens[b] new tokens that occupy
 * positions [ctx_lens[b] - q_lens[b], ctx_lens[b]) of its paged cache.
 * Order per layer: rmsnorm -> qkv GEMM (+bias) -> rope + KV append ->
 * paged attention -> o_proj GEMM (+residual) -> rmsnorm -> gate/up GEMM
 * (SwiGLU epilogue) -> down GEMM (+residual); then the final rmsnorm over the
 * `out_rows` rows and the lm_head GEMM into `logits`.
 * ------------------------------------------------------------------------ */
typedef struct {
  const void* w_qkv;   /* [q+2kv, hidden] */
  const float* b_qkv;  /* [q+2kv] */
  const void* w_o;     /* [hidden, q] */
  const void* w_gu;    /* [2*inter, hidden], gate/up rows interleaved */
  const void* w_down;  /* [hidden, inter] */
  const float* ln1;    /* [hidden] */
  const float* ln2;    /* [hidden] */
  void* pool_k;        /* this layer's [num_blocks, block_size, kv_heads, head_dim] */
  void* pool_v;
} kve_layer_t;

typedef struct {
  int dtype;  /* KVE_F32 or KVE_BF16: weights, activations and cache */
  int num_layers, hidden, num_heads, num_kv_heads, head_dim, intermediate, vocab;
  float rms_eps;
  const kve_layer_t* layers; /* host array [num_layers] */
  const void* embed;         /* [vocab, hidden] */
  const void* lm_head;       /* [vocab, hidden] */
  const float* final_norm;   /* [hidden] */
  const float* rope_cos;     /* [rope_len, head_dim/2] */
  const float* rope_sin;
  int rope_len;
  int64_t num_blocks;
  int block_size;
} kve_model_t;

typedef struct {
  int n_tokens, n_seqs, max_q_len, max_ctx;
  const int32_t* ids;        /* [n_tokens] */
  const int32_t* positions;  /* [n_tokens] */
  const int32_t* slots;      /* [n_tokens] flat slot = block * block_size + offset */
  const int32_t* q_lens;     /* [n_seqs] */
  const int32_t* q_offsets;  /* [n_seqs + 1] */
  const int32_t* ctx_lens;   /* [n_seqs] */
  const int32_t* block_tables; /* [n_seqs, table_stride] */
  int table_stride;
  int n_out;                 /* rows whose logits are computed */
  const int32_t* out_rows;   /* [n_out] token rows, or NULL for rows 0..n_out-1 */
  void* logits;              /* [n_out, vocab] in logits_dtype */
  int logits_dtype;
} kve_batch_t;

typedef struct {
  void* hidden;   /* [n_tokens, hidden] residual stream */
  void* normed;   /* [n_tokens, hidden] */
  void* qkv;      /* [n_tokens, q+2kv] */
  void* q;        /* [n_tokens, q] */
  void* attn;     /* [n_tokens, q] */
  void* act;      /* [n_tokens, inter] */
  void* out_normed; /* [n_out, hidden] */
  void* gemm_ws; size_t gemm_ws_bytes;
  void* attn_ws; size_t attn_ws_bytes;
  int* dev_status;
} kve_scratch_t;

/* Bytes the two workspaces of kve_forward need for a batch of this size. */
size_t kve_forward_gemm_ws_bytes(const kve_model_t* model, int n_tokens, int n_out);
size_t kve_forward_attn_ws_bytes(const kve_model_t* model, int n_seqs, int max_q_len, int max_ctx);
int kve_forward(const kve_model_t* model, const kve_batch_t* batch, const kve_scratch_t* scratch,
                cudaStream_t stream);

/* kve_forward recorded into a CUDA graph and launched as one graph (no kvengine
 * counterpart; same results, fewer launch costs on the GPU). *graph_slot is an
 * opaque handle owned by the caller: NULL before the first call, then the library's
 * record of the executable graph, which later calls update in place when they
 * record the same kernels (same functions, block, shared-memory and cluster
 * shapes; new pointers, sizes and grids) and rebuild otherwise. The stream must not
 * be the legacy default stream (it cannot be captured). Free the handle with
 * kve_forward_graph_free. */
int kve_forward_graphed(const kve_model_t* model, const kve_batch_t* batch, const kve_scratch_t* scratch,
                        void** graph_slot, cudaStream_t stream);
int kve_forward_graph_free(void* graph_slot);

/* Layers [l0, l1) of a kve_forward pass, as stream launches or recorded into a graph
 * (no kvengine counterpart): l0 == 0 includes the embedding, l1 == num_layers the
 * final norm and vocabulary projection. A pass split in two ranges, run in order on
 * one stream, computes exactly what kve_forward computes; the split lets a caller
 * start the first layers at once while it records the rest. */
int kve_forward_layers(const kve_model_t* model, const kve_batch_t* batch, const kve_scratch_t* scratch, int l0,
                       int l1, cudaStream_t stream);
int kve_forward_layers_graphed(const kve_model_t* model, const kve_batch_t* batch, const kve_scratch_t* scratch,
                               int l0, int l1, void** graph_slot, cudaStream_t stream);

/* The next speculative step's first draft pass, planned on the device from this
 * step's acceptance result (no kvengine counterpart as a kernel: it moves to the
 * device the host bookkeeping between two iterations of kvengine/speculative.py,
 * the rollback to the accepted prefix at :199-214 and the next
 * `feed(draft, unseen)` at :147-158), so that the pass can be queued before the
 * accept readback.
 * Inputs per sequence s of this step: start_lens[s] = T0, its token count at the
 * start of the step; last_tokens[s] = its token at position T0 - 1 (rows == 2
 * only); n_blocks[s] and tables [n_seqs, width] its draft block count and block
 * table (width >= max block count + 2); n_accepted [n_seqs] and emitted
 * [n_seqs, k+1] as kve_greedy_accept writes them; dump_block: a pool block no
 * sequence holds (a free block: later owners write it after this pass).
 * rows == 1: one row per sequence, (position T0 + n, bonus emitted[s][n]); exact
 * when n < k; a sequence with n == k gets position T0 + k - 1 (its first
 * uncommitted draft position) and the caller must discard the pass.
 * rows == 2: two rows per sequence, exact for every n: (T0 + n - 1, the token
 * there) and (T0 + n, bonus); for n < k the first row rewrites a committed
 * position with the same token and context, i.e. the same K/V bits.
 * A row at a position past the sequence's n_blocks blocks reads and writes
 * dump_block (table entries from n_blocks on are set to it); the caller must then
 * discard the pass.
 * Writes plan_out in the kve_batch_t layout, packed as positions [M] | slots [M] |
 * q_lens [S] | q_offsets [S+1] | ctx_lens [S] | out_rows [S] | tables [S * width]
 * (M = rows * S, logits row = the last row of each sequence), ids_out [M] (the
 * rows' tokens) and verify_ids_out[s * (k+1)] (the bonus: row 0 of the next
 * verify feed, whose other k rows the draft argmax kernels fill). */
int kve_spec_next_draft_plan(const int32_t* start_lens, const int32_t* last_tokens, const int32_t* n_blocks,
                             const int32_t* tables, int n_seqs, int width, int block_size, int k, int rows,
                             int dump_block, const int32_t* n_accepted, const int32_t* emitted, int32_t* plan_out,
                             int32_t* ids_out, int32_t* verify_ids_out, int* dev_status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KVENGINE_B200_H */
