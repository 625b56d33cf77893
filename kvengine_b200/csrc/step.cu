// Device-side planning of the next speculative step's first draft pass.
//
// After the verify pass and the acceptance kernel of step i, the host would
// read the accepted lengths back, roll both caches back to the accepted prefix
// and build the plan of step i+1's first draft pass (kvengine/speculative.py:
// 199-214, then the next iteration's `feed(draft, unseen)` at :147-158). In the
// steady state every quantity of that plan follows on the device from the
// acceptance result, so the pass can be queued before the readback and run
// while the host does its bookkeeping. For sequence s with T0 tokens at the
// start of step i and n = n_accepted[s] (0 <= n <= k):
//
//   the draft keeps min(T0 + k - 1, T0 + n) tokens and its next feed ends with
//   the bonus token emitted[s][n] at position T0 + n.
//
// rows == 1: one row per sequence, (T0 + n, bonus). Exact when n < k. When
//   n == k the draft never fed draft k (its feed would be two rows): the row
//   goes to T0 + k - 1, the first position the draft has not committed, where
//   the correct pass rewrites it, and the caller discards the pass.
// rows == 2: two rows per sequence, exact for every n: (T0 + n - 1, the token
//   there) and (T0 + n, bonus). For n < k the first row recomputes a committed
//   position with the same token and context, which rewrites the same K/V bits
//   (a row's result does not depend on the batch it runs in).
//
// A row past the sequence's reserved blocks (the next step reserves them) maps
// to `dump_block`, a block no sequence holds: table entries from the block
// count on are set to it, so such a row's K/V writes and reads touch no one's
// cache, and the caller discards the pass.
#include "kve_common.cuh"

namespace kve {
namespace {

// One thread per (sequence, table entry) in a grid-stride loop; entry 0 of a
// sequence also writes the per-sequence arrays.
__global__ void spec_next_draft_plan_kernel(const int32_t* start_len, const int32_t* last_tok, const int32_t* n_blocks,
                                            const int32_t* tables_in,
                                            int n_seqs, int width, int bs, int k, int rows, int dump_block,
                                            const int32_t* n_acc, const int32_t* emitted,
                                            int32_t* __restrict__ plan, int32_t* __restrict__ ids,
                                            int32_t* __restrict__ verify_ids, int* status) {
  grid_dep_wait();
  grid_dep_launch();
  const int S = n_seqs, M = rows * n_seqs;
  int32_t* positions = plan;
  int32_t* slots = positions + M;
  int32_t* q_lens = slots + M;
  int32_t* q_offsets = q_lens + S;
  int32_t* ctx_lens = q_offsets + S + 1;
  int32_t* out_rows = ctx_lens + S;
  int32_t* tables = out_rows + S;
  const long long total = (long long)S * width;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int s = (int)(i / width), j = (int)(i % width);
    const int nb = n_blocks[s];
    const int32_t* row = tables_in + (size_t)s * width;
    tables[i] = j < nb ? row[j] : dump_block;
    if (j != 0) continue;
    int n = n_acc[s];
    if (n < 0 || n > k) {
      report(status, KVE_ERR_BOUNDS);
      n = 0;
    }
    const int32_t* em = emitted + (size_t)s * (k + 1);
    const int t0 = start_len[s];
    int pos[2], tok[2];
    if (rows == 1) {
      pos[0] = t0 + (n < k ? n : k - 1);
      tok[0] = em[n];
    } else {
      pos[0] = t0 + n - 1;
      tok[0] = n > 0 ? em[n - 1] : last_tok[s];
      pos[1] = t0 + n;
      tok[1] = em[n];
    }
    for (int r = 0; r < rows; ++r) {
      const int blk = pos[r] / bs;
      int slot = -1;
      if (pos[r] < 0 || blk >= width) report(status, KVE_ERR_BOUNDS);
      else slot = (blk < nb ? row[blk] : dump_block) * bs + pos[r] % bs;
      positions[rows * s + r] = pos[r];
      slots[rows * s + r] = slot;
      ids[rows * s + r] = tok[r];
    }
    q_lens[s] = rows;
    q_offsets[s] = rows * s;
    if (s == S - 1) q_offsets[S] = M;
    ctx_lens[s] = pos[rows - 1] + 1;
    out_rows[s] = rows * s + rows - 1;
    verify_ids[(size_t)s * (k + 1)] = em[n];
  }
}

}  // namespace
}  // namespace kve

using namespace kve;

extern "C" int kve_spec_next_draft_plan(const int32_t* start_lens, const int32_t* last_tokens,
                                        const int32_t* n_blocks, const int32_t* tables, int n_seqs, int width,
                                        int block_size, int k, int rows, int dump_block, const int32_t* n_accepted,
                                        const int32_t* emitted, int32_t* plan_out, int32_t* ids_out,
                                        int32_t* verify_ids_out, int* dev_status, cudaStream_t stream) {
  if (n_seqs < 0 || width < 1 || block_size < 1 || k < 1 || (rows != 1 && rows != 2) || dump_block < 0)
    return set_error(KVE_ERR_ARG, "kve_spec_next_draft_plan: bad sizes");
  if (n_seqs == 0) return KVE_OK;
  if (!start_lens || !n_blocks || !tables || !n_accepted || !emitted || !plan_out || !ids_out || !verify_ids_out ||
      (rows == 2 && !last_tokens))
    return set_error(KVE_ERR_ARG, "kve_spec_next_draft_plan: null pointer");
  const long long total = (long long)n_seqs * width;
  const int threads = 256;
  const long long want = (total + threads - 1) / threads;
  const int blocks = (int)(want < 148 ? want : 148);
  launch_kernel(spec_next_draft_plan_kernel, dim3(blocks), dim3(threads), 0, stream, start_lens, last_tokens,
                n_blocks, tables, n_seqs, width, block_size, k, rows, dump_block, n_accepted, emitted, plan_out,
                ids_out, verify_ids_out, dev_status);
  return check_launch("kve_spec_next_draft_plan");
}
