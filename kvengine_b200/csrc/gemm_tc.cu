// bf16 GEMM y[m, n] = x[m, k] w[n, k]^T on the 5th-generation tensor cores.
//
// Weight-streaming shape (m = batch * (k+1) tokens is small, n = features is
// large), so the MMA's M dimension runs over FEATURES: one CTA owns 128 weight
// rows x `nt` tokens (nt <= 256) and accumulates D^T[128, nt] in TMEM.
// Weights are read from HBM once per token tile; CTAs of the same feature tile
// are adjacent in launch order, so a second token tile re-reads them from L2.
//
//   warp 0      TMA producer: 128x64 weight tile + nt x 64 token tile per
//               stage (SWIZZLE_128B, K-major), mbarrier expect-tx
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (kind::f16, bf16 x bf16 -> fp32), tcgen05.commit frees stages
//   warps 2-5   epilogue: tcgen05.ld 32x32b (one feature row per thread),
//               fused bias / residual / SwiGLU, store
//
// Small grids split K across CTAs. The split count depends only on (n, k), and
// the last-arriving CTA of a tile sums the fp32 partials in split order, so a
// row's result never depends on m (draft and verify passes agree bit for bit).
// Every mbarrier wait is bounded; a timeout is reported through `status`.
#include <cuda.h>
#include <math.h>

#include <mutex>

#include "gemm_epilogue.cuh"

namespace kve {
namespace {

constexpr int BM = 128;          // features per tile (MMA M)
constexpr int BK = 64;           // K per stage: one 128-byte swizzle row of bf16
constexpr int UMMA_K = 16;       // K per tcgen05.mma for 16-bit inputs
constexpr int kThreads = 192;    // 6 warps
constexpr int kMaxNT = 256;
constexpr int kMaxStages = 8;
constexpr size_t kSmemLimit = 232448;  // 227 KB opt-in

struct TcArgs {
  int m, n, k;
  int nt, k_blocks, splits, stages;
  uint32_t stage_bytes;
  EpiArgs e;
  float* ws;        // [splits, m, n] fp32 partials (splits > 1)
  int* counters;    // [tiles] arrival counters (splits > 1)
  int* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and KVE_ERR_TIMEOUT in status) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      report(status, KVE_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, rows of 128 bytes,
// 8-row groups 1024 bytes apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // SBO
  d |= (uint64_t)1 << 46;            // version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major, M=128, N=nt.
__device__ __forceinline__ uint32_t umma_idesc(int nt) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// One accumulator value for (token row, feature col): final epilogue. SwiGLU
// pairs live in adjacent lanes (features 2j, 2j+1), so every lane calls this.
__device__ __forceinline__ void finish(const TcArgs& a, int row, int col, float v, bool valid) {
  if (a.e.mode == KVE_EPI_SILU_MUL) {
    float other = __shfl_xor_sync(0xffffffffu, v, 1);
    if (valid && (col & 1) == 0 && col + 1 < a.n) epi_silu_mul(a.e, row, col >> 1, v, other);
  } else if (valid) {
    epi_store(a.e, row, col, v);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Stage buffers need 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * a.stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* tmem_full = bars + 2 * kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 1);
  int& s_last = *reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * a.nt;
  const int feat0 = blockIdx.y * BM;
  const int split = blockIdx.z;
  const int kb0 = (int)((long long)split * a.k_blocks / a.splits);
  const int kb1 = (int)((long long)(split + 1) * a.k_blocks / a.splits);
  // After a timeout anywhere in this launch, later CTAs skip their work instead
  // of each waiting out the limit again.
  const bool aborted = a.status && *reinterpret_cast<volatile int*>(a.status) == KVE_ERR_TIMEOUT;
  const int n_iter = aborted ? 0 : kb1 - kb0;
  uint32_t tmem_cols = 32;
  while ((int)tmem_cols < a.nt) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(tmem_full), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- producer
      const uint32_t tx_bytes = a.stage_bytes;
      int issued = 0;
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.stages;
        const uint32_t ph = (uint32_t)(it / a.stages) & 1u;
        if (it >= a.stages && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, a.status)) break;
        uint8_t* sa = smem + (size_t)s * a.stage_bytes;
        uint8_t* sb = sa + BM * BK * 2;
        mbar_expect_tx(smem_u32(&full[s]), tx_bytes);
        tma_load_2d(smem_u32(sa), &map_w, (kb0 + it) * BK, feat0, smem_u32(&full[s]));
        tma_load_2d(smem_u32(sb), &map_x, (kb0 + it) * BK, tok0, smem_u32(&full[s]));
        ++issued;
      }
      // Do not leave while a bulk copy may still be writing this CTA's shared memory.
      for (int it = issued - a.stages < 0 ? 0 : issued - a.stages; it < issued; ++it)
        mbar_wait(smem_u32(&full[it % a.stages]), (uint32_t)(it / a.stages) & 1u, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      const uint32_t idesc = umma_idesc(a.nt);
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.stages;
        const uint32_t ph = (uint32_t)(it / a.stages) & 1u;
        if (!mbar_wait(smem_u32(&full[s]), ph, a.status)) break;
        fence_after();
        const uint32_t sa = smem_u32(smem + (size_t)s * a.stage_bytes);
        const uint32_t sb = sa + BM * BK * 2;
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          umma_bf16(tmem_base, umma_desc(sa + kk * UMMA_K * 2), umma_desc(sb + kk * UMMA_K * 2), idesc,
                    (it > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(&empty[s]));
      }
      umma_commit(smem_u32(tmem_full));  // fires once every issued MMA has completed
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quarter this warp may access
    const int col_feat = feat0 + quad * 32 + lane;
    const bool feat_ok = col_feat < a.n;
    const bool waited = !aborted && mbar_wait(smem_u32(tmem_full), 0, a.status);
    fence_after();
    const uint32_t t_lane = tmem_base + ((uint32_t)(quad * 32) << 16);
    if (a.splits == 1) {
      if (waited) {
        for (int c0 = 0; c0 < a.nt; c0 += 16) {
          float v[16];
          tmem_ld16(t_lane + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = tok0 + c0 + j;
            finish(a, row, col_feat, v[j], feat_ok && row < a.m);
          }
        }
      }
    } else {
      if (waited) {
        for (int c0 = 0; c0 < a.nt; c0 += 16) {
          float v[16];
          tmem_ld16(t_lane + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = tok0 + c0 + j;
            if (feat_ok && row < a.m) a.ws[((size_t)split * a.m + row) * a.n + col_feat] = v[j];
          }
        }
      }
      __threadfence();
      epi_bar();
      if (threadIdx.x == 64) {
        int* ctr = a.counters + (blockIdx.y * gridDim.x + blockIdx.x);
        int prev = atomicAdd(ctr, 1);
        s_last = (prev == a.splits - 1);
        if (s_last) *ctr = 0;
      }
      epi_bar();
      if (s_last) {
        __threadfence();
        for (int c0 = 0; c0 < a.nt; c0 += 16) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int row = tok0 + c0 + j;
            const bool valid = feat_ok && row < a.m;
            float acc = 0.f;
            if (valid) {
              const float* p = a.ws + (size_t)row * a.n + col_feat;
              for (int s = 0; s < a.splits; ++s) acc += __ldcg(p + (size_t)s * a.m * a.n);
            }
            finish(a, row, col_feat, acc, valid);
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_map(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KVE_OK;
}

struct Plan {
  int nt, token_tiles, feat_tiles, k_blocks, splits, stages;
  uint32_t stage_bytes;
};

Plan make_plan(int m, int n, int k) {
  Plan p{};
  p.token_tiles = (m + kMaxNT - 1) / kMaxNT;
  if (p.token_tiles < 1) p.token_tiles = 1;
  int per = (m + p.token_tiles - 1) / p.token_tiles;
  p.nt = ((per + 15) / 16) * 16;
  if (p.nt < 16) p.nt = 16;
  p.feat_tiles = (n + BM - 1) / BM;
  p.k_blocks = (k + BK - 1) / BK;
  // Split K only to fill the machine; depends on (n, k) alone.
  int want = (148 + p.feat_tiles - 1) / p.feat_tiles;
  int max_splits = p.k_blocks / 4;
  if (max_splits < 1) max_splits = 1;
  p.splits = want < max_splits ? want : max_splits;
  if (p.splits < 1) p.splits = 1;
  p.stage_bytes = (uint32_t)(BM * BK * 2 + p.nt * BK * 2);
  size_t avail = kSmemLimit - 2048 /*align slack + barriers + margin*/;
  p.stages = (int)(avail / p.stage_bytes);
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  return p;
}

}  // namespace

size_t gemm_tc_workspace_bytes(int m, int n, int k) {
  Plan p = make_plan(m, n, k);
  if (p.splits <= 1) return 0;
  size_t part = (size_t)p.splits * m * n * sizeof(float);
  size_t ctr = (size_t)p.token_tiles * p.feat_tiles * sizeof(int);
  return ((ctr + 255) / 256) * 256 + part;
}

int gemm_tc(const void* x, const void* w, int m, int n, int k, const EpiArgs& e, void* workspace,
            size_t workspace_bytes, int* status, cudaStream_t stream) {
  if (k % 8) return set_error(KVE_ERR_SHAPE, "kve_gemm(tcgen05): k=%d must be a multiple of 8", k);
  if ((uintptr_t)x % 16 || (uintptr_t)w % 16)
    return set_error(KVE_ERR_ARG, "kve_gemm(tcgen05): x and w must be 16-byte aligned");
  if (e.mode == KVE_EPI_SILU_MUL && (n % 2))
    return set_error(KVE_ERR_SHAPE, "kve_gemm: SILU_MUL needs an even n");
  Plan p = make_plan(m, n, k);
  if (p.stages < 2) return set_error(KVE_ERR_SHAPE, "kve_gemm(tcgen05): tile does not fit shared memory");
  TcArgs a{};
  a.m = m; a.n = n; a.k = k; a.nt = p.nt; a.k_blocks = p.k_blocks; a.splits = p.splits; a.stages = p.stages;
  a.stage_bytes = p.stage_bytes; a.e = e; a.status = status;
  if (p.splits > 1) {
    size_t need = gemm_tc_workspace_bytes(m, n, k);
    if (!workspace || workspace_bytes < need)
      return set_error(KVE_ERR_WORKSPACE, "kve_gemm(tcgen05): workspace needs %zu bytes", need);
    size_t ctr = (size_t)p.token_tiles * p.feat_tiles * sizeof(int);
    a.counters = static_cast<int*>(workspace);
    a.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((ctr + 255) / 256) * 256);
  }
  CUtensorMap mw, mx;
  int rc = make_map(&mw, w, n, k, BM);
  if (rc) return rc;
  rc = make_map(&mx, x, m, k, p.nt);
  if (rc) return rc;
  size_t smem = (size_t)p.stages * p.stage_bytes + 1024 + 512;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
    configured = true;
  }
  dim3 grid(p.token_tiles, p.feat_tiles, p.splits);
  gemm_tc_kernel<<<grid, kThreads, smem, stream>>>(mw, mx, a);
  return check_launch("kve_gemm(tcgen05)");
}

}  // namespace kve
