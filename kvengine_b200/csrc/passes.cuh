// Internal entry points kve_forward uses in place of the public C ABI ones,
// with hints that hold inside a model pass and let kernels start their loads of
// constant data before the previous kernel in the stream has finished.
#pragma once

#include "kve_common.cuh"

namespace kve {

// kve_paged_verify_attn; hist_static: the keys before ctx - q_len of every
// sequence, the block tables and the length arrays are not written by any
// kernel that may still be running.
int paged_attn_run(const void* q, int dtype, const void* pool_k, const void* pool_v, const int32_t* block_tables,
                   int table_stride, const int32_t* ctx_lens, const int32_t* q_lens, const int32_t* q_offsets,
                   int batch, int max_q_len, int max_ctx, int num_heads, int num_kv_heads, int head_dim,
                   int block_size, int64_t num_blocks, float scale, void* out, void* workspace,
                   size_t workspace_bytes, int* dev_status, bool hist_static, cudaStream_t stream);

// kve_rmsnorm; w_static: the weight vector is written by no kernel that may
// still be running, so it is read before the dependency wait.
int rmsnorm_run(const void* x, int dtype, const float* weight, int rows, int hidden, float eps,
                const int32_t* row_index, void* out, bool w_static, cudaStream_t stream);

}  // namespace kve
