// bf16 GEMM y[m, n] = x[m, k] w[n, k]^T on the 5th-generation tensor cores.
//
// Weight-streaming shape (m = batch * (k+1) tokens is small, n = features is
// large), so the MMA's M dimension runs over FEATURES: one CTA owns 128 weight
// rows x `mt` tokens and accumulates D^T[128, mt] in TMEM. Weights are read
// from HBM once per token tile; CTAs of the same feature tile are adjacent in
// launch order, so further token tiles re-read them from L2.
//
//   warp 0      TMA producer: 128x64 weight tile + nt x 64 token tile per
//               stage (SWIZZLE_128B, K-major), mbarrier expect-tx
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (kind::f16, bf16 x bf16 -> fp32), tcgen05.commit frees stages
//   warps 2-5   epilogue: tcgen05.ld 32x32b (one feature row per thread),
//               fused bias / residual / SwiGLU, staged 16-byte stores
//
// Up to 384 tokens share one CTA (two MMAs per k-step into two TMEM column
// ranges); larger batches tile tokens by 256. Small grids split K over a thread-
// block cluster of up to 8 CTAs: each CTA parks its fp32 partial in its own
// shared memory and the cluster sums them in rank order through distributed
// shared memory, each CTA finishing a slice of the tokens (no global
// workspace). The split count depends only on (n, k), so a row's result never
// depends on m (draft and verify passes agree bit for bit). Launches without
// split-K that have more tiles than SMs may instead run persistent CTAs that walk
// several tiles with two TMEM accumulators (gemm_tc_persistent_kernel), where the
// cost model prices that cheaper (the vocabulary projection of small batches). The epilogue stages
// each 64-token chunk in shared memory and writes whole rows with 16-byte
// stores. Every mbarrier wait is bounded; a timeout is reported via `status`.
#include <cuda.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <unordered_map>
#include <type_traits>

#include "gemm_epilogue.cuh"
#include "tma.cuh"

namespace kve {
namespace {

constexpr int BM = 128;          // features per tile (MMA M)
constexpr int BK = 64;           // K per stage: one 128-byte swizzle row of bf16
constexpr int UMMA_K = 16;       // K per tcgen05.mma for 16-bit inputs
constexpr int kEpiGroups = 2;    // epilogue warpgroups (each covers all 128 TMEM lanes)
constexpr int kThreads = 64 + 128 * kEpiGroups;  // producer warp, MMA warp, epilogue warps
constexpr int kMaxNG = 256;      // tokens per MMA (N of one tcgen05.mma)
constexpr int kMaxStages = 12;
constexpr int kMaxSplits = 8;    // portable cluster size
constexpr int kRows = 32;                    // tokens per staged output chunk
constexpr int kStageBytes = 2 * kRows * 128 * 4;  // double-buffered output staging (fp32 worst case)
constexpr size_t kSmemLimit = 232448;       // 227 KB opt-in

struct TcArgs {
  int m, n, k;
  int mt, ng, n_g;       // tokens per CTA = ng groups of n_g tokens (one MMA each)
  int k_blocks, splits, stages;
  uint32_t stage_bytes;
  int rch;               // split-K: tokens reduced per round (the receive buffer holds rch tokens)
  int stg_off;           // byte offset of the output staging buffer in the drained stage area
  int out_vec_ok;        // output rows start on 16-byte boundaries
  int w_static;          // weight tiles may be requested before the previous kernel completes
  int kc;                // 64-wide k-chunks per pipeline stage (one 3-D box each for W and X)
  int tma3d;             // tensor maps are 3-D (64, rows, k/64): box {64, rows, kc}
  uint32_t w_bytes;      // weight bytes per stage (MH x 128 rows x kc chunks)
  int token_tiles;       // tiles along tokens (tile t: token tile t % token_tiles)
  int feat_ctas;         // tiles along features (128 x MH weight rows each)
  int acc_bufs;          // TMEM accumulators per CTA (2: the epilogue overlaps the next tile)
  int stg_bytes;         // output staging after the stage ring (CTAs that walk several tiles), else 0
  int lsplit;            // 1: one CTA computes all `splits` k-ranges into its own TMEM accumulators
  EpiArgs e;
  int* status;
};

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

// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major, M=128, N=n.
__device__ __forceinline__ uint32_t umma_idesc(int n, int m = BM) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
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
// Named barrier of one epilogue warpgroup (ids 1 and up; 0 is __syncthreads).
__device__ __forceinline__ void epi_bar(int group) { asm volatile("bar.sync %0, 128;" ::"r"(group + 1) : "memory"); }
// Named barrier of both epilogue warpgroups.
__device__ __forceinline__ void epi_bar_all() { asm volatile("bar.sync %0, %1;" ::"r"(kEpiGroups + 1), "r"(128 * kEpiGroups) : "memory"); }
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Up to 32 TMEM columns (n is 16 or 32) of this thread's lane into v.
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, int n, bool have, float* v) {
  if (!have) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    return;
  }
  if (n == 32) {
    tmem_ld32(taddr, v);
  } else {
    float h[16];
    tmem_ld16(taddr, h);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = h[i];
  }
}

// BMT: weight rows per tile (128, or 64 for the 64-row one-tile kernel).
template <int MODE, bool BF, int BMT = BM>
struct Epi {
  using T = typename std::conditional<BF, __nv_bfloat16, float>::type;
  static constexpr int ES = BF ? 2 : 4;
  static constexpr int W = MODE == KVE_EPI_SILU_MUL ? BMT / 2 : BMT;  // output columns per tile
  static constexpr int VE = 16 / ES;                                 // elements per 16-byte vector
  static constexpr int VPR = W / VE;                                 // vectors per staged row

  static __device__ __forceinline__ float rnd(float v) { return BF ? __bfloat162float(__float2bfloat16_rn(v)) : v; }
  static __device__ __forceinline__ T cvt(float v) {
    if constexpr (BF) return __float2bfloat16_rn(v);
    else return v;
  }

  // Stage values v[0..CNT) of this thread's feature for tokens r0 .. r0+CNT-1 into
  // the dense [kRows][W] buffer (rows >= nr are skipped). Every lane of the warp
  // calls this. SwiGLU pairs sit in adjacent lanes (gate 2j, up 2j+1): the pair
  // trades one value per two tokens, so the even lane finishes token r and the
  // odd lane token r+1 and no lane idles.
  template <int CNT>
  static __device__ __forceinline__ void stage(uint8_t* buf, int r0, int nr, int f_local, const float* v,
                                               float bias_f) {
    T* b = reinterpret_cast<T*>(buf);
    if constexpr (MODE == KVE_EPI_SILU_MUL) {
      const int odd = f_local & 1;
      T* col = b + (f_local >> 1);
      // All exchanges first, then the arithmetic: the shuffles are warp-synchronous
      // and would otherwise serialise the independent SwiGLU evaluations.
      float gs[CNT / 2], us[CNT / 2];
#pragma unroll
      for (int i = 0; i < CNT / 2; ++i) {
        const float recv = __shfl_xor_sync(0xffffffffu, odd ? v[2 * i] : v[2 * i + 1], 1);
        gs[i] = rnd(odd ? recv : v[2 * i]);
        us[i] = rnd(odd ? v[2 * i + 1] : recv);
      }
#pragma unroll
      for (int i = 0; i < CNT / 2; ++i) {
        const int r = r0 + 2 * i + odd;
        const T y = cvt(__fmul_rn(rnd(silu_fast(gs[i])), us[i]));
        if (r < nr) col[r * W] = y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < CNT; ++j) {
        const int r = r0 + j;
        if (r < nr) {
          if constexpr (MODE == KVE_EPI_BIAS || MODE == kEpiQkvRope) b[r * W + f_local] = cvt(__fadd_rn(v[j], bias_f));
          else b[r * W + f_local] = cvt(v[j]);  // RESIDUAL adds the residual while copying out
        }
      }
    }
  }

  // Per-row inputs of copy_out for rows [0, nr), loaded ahead so that they are
  // in flight together (and, for a tile's first chunk, during the main loop):
  // RESIDUAL - the residual vectors (out may alias the residual: each element is
  // read and then written by the same thread); qkv+RoPE - the token's position
  // and pool slot, with the cos/sin lines prefetched into L1.
  static constexpr int RPP = 128 / VPR;       // rows per copy_out pass
  static constexpr int NPASS = kRows / RPP;   // passes per staged chunk
  static __device__ __forceinline__ void load_res(const TcArgs& a, int tok_base, int nr, int col0, int etid,
                                                  uint4 (&res)[NPASS]) {
    if constexpr (MODE == kEpiQkvRope) {
      const int c = (etid % VPR) * VE;
      const int r_first = etid / VPR;
      const int f = col0 + c;
      if (f >= a.n) return;
      const int hd = a.e.hd, half = hd >> 1;
      const int d = f % hd;
      const int dd = d < half ? d : d - half;
      const bool rot = f < (a.e.nq + a.e.nkv) * hd;
#pragma unroll
      for (int i = 0; i < NPASS; ++i) {
        const int r = r_first + i * RPP;
        const int t = tok_base + r;
        if (r < nr && t < a.m) {
          const int pos = a.e.positions[t];
          const int64_t slot = a.e.slots[t];
          res[i] = make_uint4((uint32_t)pos, (uint32_t)slot, (uint32_t)((uint64_t)slot >> 32), 0u);
          if (rot && pos >= 0 && pos < a.e.rope_len) {
            asm volatile("prefetch.global.L1 [%0];" ::"l"(a.e.rope_cos + (size_t)pos * half + dd));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(a.e.rope_sin + (size_t)pos * half + dd));
          }
        }
      }
    }
    if constexpr (MODE == KVE_EPI_RESIDUAL) {
      const int nvalid = min(W, a.e.ld_out - col0);
      const int c = (etid % VPR) * VE;
      const int r_first = etid / VPR;
      const bool vec = a.out_vec_ok && c + VE <= nvalid;
      const T* res0 = static_cast<const T*>(a.e.residual) + (size_t)col0 + c;
#pragma unroll
      for (int i = 0; i < NPASS; ++i) {
        const int r = r_first + i * RPP;
        const int t = tok_base + r;
        if (vec && r < nr && t < a.m) res[i] = *reinterpret_cast<const uint4*>(res0 + (size_t)t * a.e.ld_out);
      }
    }
  }

  // Write staged rows [0, nr) (tokens tok_base ...) with 16-byte stores. Thread
  // etid always handles the same column vector; RPP rows per pass.
  static __device__ __forceinline__ void copy_out(const TcArgs& a, const uint8_t* buf, int tok_base, int nr,
                                                  int col0, int etid, const uint4 (&res)[NPASS]) {
    if constexpr (MODE == kEpiQkvRope) {
      // The staged row holds round(acc + bias) for features col0 .. col0 + 127.
      // A 16-byte vector (8 features) never straddles a head (hd % 8 == 0) and a
      // head never straddles a tile (128 % hd == 0), so the RoPE partner vector
      // (d +- hd/2) is in the same staged row.
      const int c = (etid % VPR) * VE;
      const int r_first = etid / VPR;
      const int f = col0 + c;
      if (f >= a.n) return;
      const int hd = a.e.hd, half = hd >> 1;
      const int q_end = a.e.nq * hd, rot_end = (a.e.nq + a.e.nkv) * hd, kv_w = a.e.nkv * hd;
      const int d = f % hd;
      const bool rot = f < rot_end, lo = d < half;
      const int dd = lo ? d : d - half;
      const int cp = lo ? c + half : c - half;
#pragma unroll
      for (int i = 0; i < NPASS; ++i) {
        const int r = r_first + i * RPP;
        const int t = tok_base + r;
        if (r >= nr || t >= a.m) break;
        const T* srow = reinterpret_cast<const T*>(buf) + r * W;
        uint4 val = *reinterpret_cast<const uint4*>(srow + c);
        if (rot) {
          int pos = (int)res[i].x;
          if (pos < 0 || pos >= a.e.rope_len) {
            report(a.e.status, KVE_ERR_BOUNDS);
            pos = 0;
          }
          // Read-only path: the tables are constant during the kernel, so these loads
          // may be issued ahead of the previous rows' stores.
          const float4* cs = reinterpret_cast<const float4*>(a.e.rope_cos + (size_t)pos * half + dd);
          const float4* sn = reinterpret_cast<const float4*>(a.e.rope_sin + (size_t)pos * half + dd);
          const float4 c0 = __ldg(cs), c1 = __ldg(cs + 1), s0 = __ldg(sn), s1 = __ldg(sn + 1);
          const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
          const uint4 pv = *reinterpret_cast<const uint4*>(srow + cp);
          T* y = reinterpret_cast<T*>(&val);
          const T* o = reinterpret_cast<const T*>(&pv);
          // One branch-free form of both halves: the first half is x1 c - x2 s
          // (rope_first), the second x2 c + x1 s (rope_second); with `self` the
          // element and `other` its partner that is round(self c) + round(+-other s),
          // the same roundings in the same order, without a divergent branch.
          const float sgn = lo ? -1.f : 1.f;
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float self = (float)y[e], other = (float)o[e];
            const float cb = Elem<T>::round(cv[e]), sb = Elem<T>::round(sv[e]);
            y[e] = cvt(__fadd_rn(Elem<T>::round(__fmul_rn(self, cb)), Elem<T>::round(__fmul_rn(sgn * other, sb))));
          }
        }
        T* dst;
        if (f < q_end) {
          dst = static_cast<T*>(a.e.q_out) + (size_t)t * q_end + f;
        } else {
          const int64_t slot = (int64_t)(((uint64_t)res[i].z << 32) | res[i].y);
          if (slot < 0 || slot >= a.e.num_slots) {
            report(a.e.status, KVE_ERR_BOUNDS);
            continue;
          }
          dst = rot ? static_cast<T*>(a.e.pool_k) + slot * kv_w + (f - q_end)
                    : static_cast<T*>(a.e.pool_v) + slot * kv_w + (f - rot_end);
        }
        *reinterpret_cast<uint4*>(dst) = val;
      }
      return;
    } else {
    const int nvalid = min(W, a.e.ld_out - col0);
    const int c = (etid % VPR) * VE;
    const int r_first = etid / VPR;
    if (c >= nvalid) return;
    const bool vec = a.out_vec_ok && c + VE <= nvalid;
    const T* src0 = reinterpret_cast<const T*>(buf) + c;
    T* dst0 = static_cast<T*>(a.e.out) + (size_t)col0 + c;
    const T* res0 = static_cast<const T*>(a.e.residual) + (size_t)col0 + c;
#pragma unroll
    for (int i = 0; i < NPASS; ++i) {
      const int r = r_first + i * RPP;
      const int t = tok_base + r;
      if (r >= nr || t >= a.m) break;
      const T* src = src0 + r * W;
      T* dst = dst0 + (size_t)t * a.e.ld_out;
      if (vec) {
        uint4 val = *reinterpret_cast<const uint4*>(src);
        if constexpr (MODE == KVE_EPI_RESIDUAL) {
          T* y = reinterpret_cast<T*>(&val);
          const T* q = reinterpret_cast<const T*>(&res[i]);
#pragma unroll
          for (int j = 0; j < VE; ++j) y[j] = cvt(__fadd_rn((float)q[j], (float)y[j]));
        }
        *reinterpret_cast<uint4*>(dst) = val;
      } else {
        for (int j = 0; j < VE && c + j < nvalid; ++j) {
          float y = (float)src[j];
          if constexpr (MODE == KVE_EPI_RESIDUAL) y = __fadd_rn((float)res0[(size_t)t * a.e.ld_out + j], y);
          dst[j] = cvt(y);
        }
      }
    }
    }
  }
};

__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t mbar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
               : "memory");
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t map_to(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// Split-K over the cluster, general form: each CTA writes its fp32 partial,
// grouped by the CTA that owns each token (contiguous slices of the round), and
// sends every peer its group with one bulk shared-memory copy; the owner then sums
// the S partials of its tokens in rank order from its own shared memory.
template <int MODE, bool BF, int MH, int BMT>
__device__ __forceinline__ void splitk_exchange(const TcArgs& a, uint8_t* smem, uint32_t t_lane, bool have, bool epi,
                                                int egrp, int f_local, int etid, int tok0, int col0, float bias_f,
                                                const uint4 (&res_first)[Epi<MODE, BF, BMT>::NPASS],
                                                uint64_t* recv_bar) {
  using E = Epi<MODE, BF, BMT>;
  const int S = a.splits;
  uint8_t* stg = smem + a.stg_off;
    const uint32_t rank = cluster_rank();
    const int slm = (a.rch + S - 1) / S;               // max tokens per slice
    float* pout = reinterpret_cast<float*>(smem);      // [rch][128] this CTA's partial, token-major
    float* recv = pout + (size_t)a.rch * BM;           // [S][slm][128] received slices, by sender
    int round = 0;
    for (int r0 = 0; r0 < a.mt; r0 += a.rch, ++round) {
      const int ch = min(a.rch, a.mt - r0);
      // Peers write into this CTA's drained stage buffers: wait until every CTA of
      // the cluster has finished its main loop (and, in later rounds, its reads).
      cluster_sync();
      const int my_lo = (int)rank * ch / S, my_hi = ((int)rank + 1) * ch / S;  // 32-bit: ch <= 512, S <= 8
      if (epi) {
        // Both warpgroups drain alternate 32-token chunks; owner u's tokens
        // [lo_u, hi_u) are contiguous rows of pout.
        float* prow = pout + f_local;
        for (int c = egrp * kRows; c < ch; c += kEpiGroups * kRows) {
          const int n = min(kRows, ch - c);
          float v[32];
          tmem_load_cols(t_lane + r0 + c, n, have, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < n) prow[(c + j) * BM] = v[j];
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        epi_bar_all();
        // Thread u of the first warpgroup sends peer u its slice (one bulk copy each,
        // issued in parallel: one thread issuing them in turn spent ~0.3 us per copy);
        // thread `rank` arms this CTA's receive barrier for the S - 1 incoming slices.
        if (egrp == 0 && etid < S) {
          const int u = etid;
          if (u == (int)rank) {
            mbar_expect_tx(smem_u32(recv_bar), (uint32_t)(S - 1) * (uint32_t)(my_hi - my_lo) * BM * 4);
          } else {
            const int lo = u * ch / S, hi = (u + 1) * ch / S;
            if (hi > lo)
              bulk_copy_to_peer(map_to(smem_u32(recv + (size_t)rank * slm * BM), (uint32_t)u),
                                smem_u32(pout + (size_t)lo * BM), (uint32_t)(hi - lo) * BM * 4,
                                map_to(smem_u32(recv_bar), (uint32_t)u));
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
        mbar_wait(smem_u32(recv_bar), (uint32_t)(round & 1), a.status);
        // Sum the S partials of each owned token in rank order (own slice from
        // pout), 32-token chunks alternating between the warpgroups when both
        // groups' double-buffered staging fits (16-bit outputs).
        constexpr int kStgBufC = kRows * E::W * E::ES;
        constexpr int kSumGroups = 2 * kEpiGroups * kStgBufC <= kStageBytes ? kEpiGroups : 1;
        const float* src[kMaxSplits];
#pragma unroll
        for (int u = 0; u < kMaxSplits; ++u)
          src[u] = (u == (int)rank ? pout + (size_t)my_lo * BM : recv + (size_t)u * slm * BM) + f_local;
        const int mine = my_hi - my_lo;
        int it = 0;
        for (int t0 = egrp * kRows; egrp < kSumGroups && t0 < mine; t0 += kSumGroups * kRows, ++it) {
          const int n = min(kRows, mine - t0);
          uint8_t* buf = stg + (egrp * 2 + (it & 1)) * kStgBufC;
          uint4 res[E::NPASS];
          if (round == 0 && it == 0) {
#pragma unroll
            for (int i = 0; i < E::NPASS; ++i) res[i] = res_first[i];
          } else {
            E::load_res(a, tok0 + r0 + my_lo + t0, n, col0, etid, res);
          }
          for (int j0 = 0; j0 < n; j0 += 4) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int u = 0; u < kMaxSplits; ++u) {
              if (u < S) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  if (j0 + q < n) acc[q] += src[u][(t0 + j0 + q) * BM];
              }
            }
            E::template stage<4>(buf, j0, n, f_local, acc, bias_f);
          }
          epi_bar(egrp);
          E::copy_out(a, buf, tok0 + r0 + my_lo + t0, n, col0, etid, res);
        }
        if (egrp == 0 && etid < S && etid != (int)rank) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        epi_bar_all();
      }
    }
  }

// Split-K over the cluster for 16-bit RESIDUAL / STORE tiles whose partials fit
// the drained stage area in one round: every CTA drains its fp32 partial to its
// own shared memory and, after a cluster barrier, the owner of each token reads
// the S partials of that token straight from the peers' shared memory (16-byte
// distributed loads, all issued before the sums) and sums them in rank order -
// the same additions, in the same order, as splitk_exchange, without the bulk
// copies, receive buffers and staging. A third barrier keeps every partial alive
// until its readers are done.
__device__ __forceinline__ void splitk_direct(const TcArgs& a, uint8_t* smem, uint32_t t_lane, bool have, bool epi,
                                              int egrp, int f_local, int tok0, int col0) {
  using T = __nv_bfloat16;
  constexpr int B = 4;  // tokens per thread per batch
  const int S = a.splits;
  const uint32_t rank = cluster_rank();
  float* pout = reinterpret_cast<float*>(smem);  // [mt][128] this CTA's partial, token-major
  const int my_lo = (int)rank * a.mt / S, my_hi = ((int)rank + 1) * a.mt / S;  // 32-bit: mt <= 512, S <= 8
  const int tid = (int)threadIdx.x - 64;  // epilogue thread 0 .. 255
  const int fq = tid & 31;                 // features 4 fq .. 4 fq + 3 of the tile
  const int tsub = tid >> 5;               // token offset within a pass of 8
  const T* res_base = static_cast<const T*>(a.e.residual) + col0 + 4 * fq;
  T* out_base = static_cast<T*>(a.e.out) + col0 + 4 * fq;
  const bool residual = a.e.mode == KVE_EPI_RESIDUAL;
  // The first batch's residual rows load while the partials drain and the cluster syncs.
  uint2 res[B];
#pragma unroll
  for (int b = 0; b < B; ++b) {
    res[b] = make_uint2(0u, 0u);
    const int t = my_lo + tsub + 8 * b;
    if (epi && residual && t < my_hi && tok0 + t < a.m)
      res[b] = *reinterpret_cast<const uint2*>(res_base + (size_t)(tok0 + t) * a.e.ld_out);
  }
  // Peers read this CTA's stage buffers: wait until every CTA has finished its main loop.
  cluster_sync();
  if (epi) {
    float* prow = pout + f_local;
    for (int c = egrp * kRows; c < a.mt; c += kEpiGroups * kRows) {
      const int n = min(kRows, a.mt - c);
      float v[32];
      tmem_load_cols(t_lane + c, n, have, v);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < n) prow[(c + j) * BM] = v[j];
    }
  }
  cluster_sync();  // every partial is in its CTA's shared memory
  if (epi) {
    uint32_t peer[kMaxSplits];
#pragma unroll
    for (int u = 0; u < kMaxSplits; ++u) peer[u] = u < S ? map_to(smem_u32(pout + 4 * fq), (uint32_t)u) : 0u;
    for (int t_b = my_lo + tsub; t_b < my_hi; t_b += 8 * B) {
      float4 acc[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        acc[b] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int t = t_b + 8 * b;
        if (t_b != my_lo + tsub && residual && t < my_hi && tok0 + t < a.m)
          res[b] = *reinterpret_cast<const uint2*>(res_base + (size_t)(tok0 + t) * a.e.ld_out);
      }
      float4 part[kMaxSplits][B];
#pragma unroll
      for (int u = 0; u < kMaxSplits; ++u)
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const int t = t_b + 8 * b;
          part[u][b] = u < S && t < my_hi ? ld_cluster_f4(peer[u] + (uint32_t)(t * BM * 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < kMaxSplits; ++u)
#pragma unroll
        for (int b = 0; b < B; ++b)
          if (u < S) {
            acc[b].x += part[u][b].x;
            acc[b].y += part[u][b].y;
            acc[b].z += part[u][b].z;
            acc[b].w += part[u][b].w;
          }
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const int t = t_b + 8 * b;
        if (t >= my_hi || tok0 + t >= a.m) continue;
        const float sv[4] = {acc[b].x, acc[b].y, acc[b].z, acc[b].w};
        const T* rv = reinterpret_cast<const T*>(&res[b]);
        uint2 outv;
        T* ov = reinterpret_cast<T*>(&outv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const T y = __float2bfloat16_rn(sv[j]);
          ov[j] = residual ? __float2bfloat16_rn(__fadd_rn(__bfloat162float(rv[j]), __bfloat162float(y))) : y;
        }
        *reinterpret_cast<uint2*>(out_base + (size_t)(tok0 + t) * a.e.ld_out) = outv;
      }
    }
  }
  cluster_sync();  // no CTA leaves (or reuses its partial) while a peer may still read it
}

// Rows of weights per CTA: MH halves of 128 (one MMA M-tile each) sharing the
// activation tile, so each activation byte a CTA loads serves 128 * MH features.
//
// BMT = 64 (one weight half, no split-K): 64-row MMA tiles (M = 64), for GEMMs
// whose 128-row weight slab per CTA would overflow the stage ring while a 64-row
// slab fits, so all of a CTA's weights can be requested before the dependency
// wait. The accumulator's 64 rows sit in TMEM lanes 0-15 of each 32-lane
// quarter: epilogue threads 0-15 of each warp own a row, 16-31 write nothing.
//
// LSP (a.lsplit): split-K inside the CTA - it computes all a.splits k-ranges of
// its tile, range r into its own TMEM accumulator, and sums them in the epilogue.
template <int MODE, bool BF, int NG, int MH, int BMT = BM, bool LSP = false>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, TcArgs a) {
  static_assert(BMT == BM || (BMT == 64 && MH == 1), "64-row tiles carry one weight half");
  static_assert(!LSP || (BMT == BM && MH == 1 && NG == 1), "in-CTA split-K tiles are one 128-row half, one group");
  using E = Epi<MODE, BF, BMT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Stage buffers need 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * a.stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* tmem_full = bars + 2 * kMaxStages;
  uint64_t* epi_done = bars + 2 * kMaxStages + 1;
  uint64_t* recv_bar = bars + 2 * kMaxStages + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 3);
  // After the main loop the drained stage buffers hold the split-K exchange
  // buffers (offset 0) and the output staging (offset stg_off).

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // LSP grids run the feature tiles fastest: the CTAs of a wave share a few token
  // tiles and all the weights, which stay in L2, so each activation row comes from
  // DRAM once (prompt-sized activations overflow L2: 186 MB for the 3B down).
  const int tok0 = (LSP ? blockIdx.y : blockIdx.x) * a.mt;
  const int feat0 = (LSP ? blockIdx.x : blockIdx.y) * BMT * MH;
  // Split-K: k-range r is k-blocks [range_lo(r), range_lo(r + 1)). Over a cluster
  // (CS CTAs) this CTA computes range blockIdx.z; with lsplit it computes all LS
  // ranges itself, range r into its own TMEM accumulator, and sums them in the
  // epilogue exactly as the cluster's owner sums its peers' partials.
  const int LS = LSP ? a.splits : 1;
  const int CS = LSP ? 1 : a.splits;
  // (r * k_blocks fits 32 bits: k_blocks = k / 64 < 2^25 and r <= kMaxSplits.)
  auto range_lo = [&](int r) { return r * a.k_blocks / a.splits; };
  const int r_first = LSP ? 0 : (int)blockIdx.z;
  const int kb0 = range_lo(r_first), kb1 = range_lo(r_first + 1);
  // Pipeline stages of kc k-blocks, a range's last one possibly partial.
  int n_stages_work = (kb1 - kb0 + a.kc - 1) / a.kc;
  if constexpr (LSP)
    for (int r = 1; r < LS; ++r) n_stages_work += (range_lo(r + 1) - range_lo(r) + a.kc - 1) / a.kc;
  uint32_t tmem_cols = 32;
  while ((int)tmem_cols < MH * a.mt * LS) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(tmem_full), 1);
    mbar_init(smem_u32(epi_done), 4 * kEpiGroups);  // one arrival per epilogue warp
    mbar_init(smem_u32(recv_bar), 1);  // this CTA's expect-tx arrival per split-K round
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
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
  // Weights no kernel writes (w_static): the first stages' weight tiles are
  // requested before waiting on the previous kernel, so their latency overlaps
  // its tail. Their full barriers expect the bytes now and get the arrival (with
  // the activation bytes) once the activations may be read.
  // Stage layout: weights [kc][128 * MH rows][64] then, per token group,
  // activations [kc][n_g rows][64]; every [rows][64] slab is one SW128 K-major tile.
  auto load_w = [&](uint8_t* dst, int chunk, uint32_t fb) {
    if (a.tma3d) tma_load_3d(smem_u32(dst), &map_w, 0, feat0, chunk, fb);
    else tma_load_2d(smem_u32(dst), &map_w, chunk * BK, feat0, fb);
  };
  auto load_x = [&](uint8_t* dst, int chunk, uint32_t fb) {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      uint8_t* d = dst + (size_t)g * a.kc * a.n_g * BK * 2;
      if (a.tma3d) tma_load_3d(smem_u32(d), &map_x, 0, tok0 + g * a.n_g, chunk, fb);
      else tma_load_2d(smem_u32(d), &map_x, chunk * BK, tok0 + g * a.n_g, fb);
    }
  };
  // Walk to the next stage: `chunk` is its first k-block, in range r = [rlo, rhi).
  auto next_stage = [&](int& r, int& chunk, int& rlo, int& rhi) {
    chunk += a.kc;
    if (LSP && chunk >= rhi) {
      ++r;
      rlo = chunk = rhi;
      rhi = range_lo(r + 1);
    }
  };
  const int pre = a.w_static ? min(n_stages_work, a.stages) : 0;
  if (warp == 0 && lane == 0) {
    prefetch_map(&map_w);
    prefetch_map(&map_x);
    uint8_t* sa = smem;
    int r = r_first, chunk = kb0, rlo = kb0, rhi = kb1;
    for (int it = 0; it < pre; ++it, sa += a.stage_bytes) {
      const uint32_t fb = smem_u32(&full[it]);
      mbar_add_tx(fb, a.w_bytes);
      load_w(sa, chunk, fb);
      next_stage(r, chunk, rlo, rhi);
    }
  }
  // After a timeout anywhere in this launch, later CTAs skip their work instead
  // of each waiting out the limit again. The flag is read before the dependency
  // wait, so its latency overlaps the previous kernel's tail instead of delaying
  // the first loads (the CTAs whose timeout it reports run alongside this one; a
  // timeout of an earlier kernel is seen by the launches after this one).
  const bool aborted = a.status && *reinterpret_cast<volatile int*>(a.status) == KVE_ERR_TIMEOUT;
  // Everything else touches global memory only after the previous kernel has
  // completed.
  grid_dep_wait();
  grid_dep_launch();
  const int n_iter = aborted ? 0 : n_stages_work;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- producer
      int issued = 0, s = 0;
      uint32_t ph = 0;
      uint8_t* sa = smem;
      int r = r_first, chunk = kb0, rlo = kb0, rhi = kb1;
      for (int it = 0; it < n_iter; ++it) {
        if (it >= a.stages && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, a.status)) break;
        const uint32_t fb = smem_u32(&full[s]);
        if (it < pre) {
          mbar_expect_tx(fb, a.stage_bytes - a.w_bytes);  // weight tile already requested
        } else {
          mbar_expect_tx(fb, a.stage_bytes);
          load_w(sa, chunk, fb);
        }
        load_x(sa + a.w_bytes, chunk, fb);
        ++issued;
        next_stage(r, chunk, rlo, rhi);
        if (++s == a.stages) {
          s = 0;
          ph ^= 1u;
          sa = smem;
        } else {
          sa += a.stage_bytes;
        }
      }
      // Early weight loads of stages the loop never reached (abort): arrive so
      // their phase completes once those bytes land.
      for (int it = issued; it < pre; ++it) mbar_arrive(smem_u32(&full[it]));
      if (issued < pre) issued = pre;
      // Do not leave while a bulk copy may still be writing this CTA's shared memory.
      for (int it = issued - a.stages < 0 ? 0 : issued - a.stages; it < issued; ++it)
        mbar_wait(smem_u32(&full[it % a.stages]), (uint32_t)(it / a.stages) & 1u, a.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // One thread issues every MMA; its ALU latency is fully exposed, so the
    // loop only adds precomputed descriptor deltas (the 14-bit start-address
    // field counts 16-byte units; stages, k-steps and N groups are offsets).
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(a.n_g, BMT);
      const uint64_t a0 = umma_desc(smem_u32(smem));
      const uint64_t b0 = umma_desc(smem_u32(smem) + a.w_bytes);
      const uint64_t stage_step = (uint64_t)(a.stage_bytes >> 4);
      constexpr uint64_t half_step = (uint64_t)((BMT * BK * 2) >> 4);            // next 128 weight rows
      const uint64_t a_chunk = (uint64_t)((MH * BMT * BK * 2) >> 4);             // next k-chunk of weights
      const uint64_t b_chunk = (uint64_t)((a.n_g * BK * 2) >> 4);                // next k-chunk of a group
      const uint64_t grp_step = (uint64_t)((a.kc * a.n_g * BK * 2) >> 4);        // next token group
      constexpr uint64_t kstep = (UMMA_K * 2) >> 4;  // 32 bytes along K
      int s = 0;
      uint32_t ph = 0;
      uint64_t soff = 0;
      int r = r_first, chunk = kb0, rlo = kb0, rhi = kb1;
      for (int it = 0; it < n_iter; ++it) {
        if (!mbar_wait(smem_u32(&full[s]), ph, a.status)) break;
        fence_after();
        const int nch = min(a.kc, rhi - chunk);  // a range's partial last stage multiplies only its own chunks
        const uint32_t acc_base = tmem_base + (LSP ? (uint32_t)(r * a.mt) : 0u);
        for (int j = 0; j < nch; ++j) {
          const uint64_t ad = a0 + soff + j * a_chunk, bd = b0 + soff + j * b_chunk;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint32_t acc = (chunk > rlo || j > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < MH; ++h)
#pragma unroll
              for (int g = 0; g < NG; ++g)
                umma_bf16(acc_base + h * a.mt + g * a.n_g, ad + h * half_step + kk * kstep,
                          bd + g * grp_step + kk * kstep, idesc, acc);
          }
        }
        next_stage(r, chunk, rlo, rhi);
        umma_commit(smem_u32(&empty[s]));
        if (++s == a.stages) {
          s = 0;
          ph ^= 1u;
          soff = 0;
        } else {
          soff += stage_step;
        }
      }
      umma_commit(smem_u32(tmem_full));  // fires once every issued MMA has completed
    }
    __syncwarp();
  }

  // ---------------------------------------------------------------- epilogue
  // Epilogue warps 2.. own TMEM lane quarters (warp w reads lanes 32*(w%4) ...),
  // i.e. feature rows; tokens are TMEM columns. With one weight half (MH == 1)
  // each warpgroup takes every kEpiGroups-th chunk of 32 tokens; with two, each
  // warpgroup drains one half. A chunk is staged in a dense [32][W] buffer of the
  // warpgroup's own (double-buffered) and written as whole rows.
  static_assert(MH == 1 || MH == kEpiGroups, "one epilogue warpgroup per weight half");
  const bool epi = warp >= 2;
  const int egrp = epi ? (warp - 2) / 4 : 0;
  const int half = MH == 1 ? 0 : egrp;
  const int quad = warp & 3;
  const int f_local = BMT == BM ? quad * 32 + lane : quad * 16 + (lane & 15);
  const bool live = BMT == BM || lane < 16;  // this thread's TMEM lane holds a row of the tile
  const int fbase = feat0 + half * BMT;  // first feature of this warpgroup's rows
  const int feat = fbase + f_local;
  const int col0 = MODE == KVE_EPI_SILU_MUL ? fbase / 2 : fbase;
  const uint32_t t_lane = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * a.mt);
  const int etid = (threadIdx.x - 64) & 127;  // thread index within its warpgroup
  const float bias_f = ((MODE == KVE_EPI_BIAS || MODE == kEpiQkvRope) && epi && feat < a.n) ? a.e.bias[feat] : 0.f;
  // The first chunk's per-row inputs load while the main loop runs.
  const int first_c0 = MH == 1 ? egrp * kRows : 0;
  uint4 res_first[E::NPASS];
  if (epi && CS == 1 && first_c0 < a.mt)
    E::load_res(a, tok0 + first_c0, min(kRows, a.mt - first_c0), col0, etid, res_first);
  if constexpr (BMT == BM) {
    // Split-K: the first chunk of tokens this CTA owns in the first round.
    constexpr int kSumGroupsP = 2 * kEpiGroups * (kRows * E::W * E::ES) <= kStageBytes ? kEpiGroups : 1;
    if (epi && CS > 1 && egrp < kSumGroupsP) {
      const int ch0 = min(a.rch, a.mt);
      const uint32_t rk = cluster_rank();
      const int lo = (int)rk * ch0 / a.splits, hi = ((int)rk + 1) * ch0 / a.splits;
      const int t0 = egrp * kRows;
      if (t0 < hi - lo) E::load_res(a, tok0 + lo + t0, min(kRows, hi - lo - t0), col0, etid, res_first);
    }
  }
  bool have = false;
  if (epi) {
    have = !aborted && mbar_wait(smem_u32(tmem_full), 0, a.status);
    fence_after();
  }
  uint8_t* stg = smem + a.stg_off;
  constexpr int kStgBuf = kRows * BM * 4;  // one staging buffer (fp32 worst case)
  if (CS == 1) {
    if (epi) {
      int it = 0;
      constexpr int kChunkStride = (MH == 1 ? kEpiGroups : 1) * kRows;
      for (int c0 = first_c0; c0 < a.mt; c0 += kChunkStride, ++it) {
        const int n = min(kRows, a.mt - c0);
        uint8_t* buf = stg + (egrp * 2 + (it & 1)) * kStgBuf;
        uint4 res[E::NPASS];
        if (it == 0) {
#pragma unroll
          for (int i = 0; i < E::NPASS; ++i) res[i] = res_first[i];
        } else {
          E::load_res(a, tok0 + c0, n, col0, etid, res);
        }
        float v[32];
        if constexpr (!LSP) {
          tmem_load_cols(t_lane + c0, n, have, v);
        } else {
          // The LS partials summed from zero in range order: the additions of the
          // cluster split-K reductions (splitk_exchange, splitk_direct).
          // 16 columns per load keeps the second operand to 16 registers.
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
          for (int u = 0; u < LS; ++u) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (h == 1 && n <= 16) break;
              float p[16];
              if (have) {
                tmem_ld16(t_lane + (uint32_t)(u * a.mt) + c0 + 16 * h, p);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) p[i] = 0.f;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) v[16 * h + i] += p[i];
            }
          }
        }
        E::template stage<32>(buf, 0, live ? n : 0, f_local, v, bias_f);
        epi_bar(egrp);
        E::copy_out(a, buf, tok0 + c0, n, col0, etid, res);
      }
    }
  } else if constexpr (BMT == BM && MH == 1 && BF &&
                       (MODE == KVE_EPI_RESIDUAL || MODE == KVE_EPI_STORE)) {
    if ((size_t)a.mt * BM * 4 <= (size_t)a.stages * a.stage_bytes && a.out_vec_ok && col0 + BM <= a.e.ld_out) {
      splitk_direct(a, smem, t_lane, have, epi, egrp, f_local, tok0, col0);
    } else {
      splitk_exchange<MODE, BF, MH, BMT>(a, smem, t_lane, have, epi, egrp, f_local, etid, tok0, col0, bias_f,
                                         res_first, recv_bar);
    }
  } else if constexpr (BMT == BM) {
    splitk_exchange<MODE, BF, MH, BMT>(a, smem, t_lane, have, epi, egrp, f_local, etid, tok0, col0, bias_f,
                                       res_first, recv_bar);
  }

  if (epi) {
    // Every tcgen05.ld of this warp has completed (wait::ld); tell warp 1 it may free TMEM.
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(epi_done));
  } else if (warp == 1) {
    // Free TMEM only after the epilogue is done with it (bounded wait; freed either way
    // so a later CTA on this SM can always allocate).
    mbar_wait(smem_u32(epi_done), 0, a.status);
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// Persistent variant of gemm_tc_kernel for launches without split-K that have
// more tiles than resident CTAs. Tile t covers tokens [(t % token_tiles) * mt,
// +mt) and weight rows [(t / token_tiles) * 128 * MH, +128 * MH); CTA b walks
// tiles b, b + gridDim.x, ..., so the CTAs running at the same time share weight
// tiles through L2. The stage ring runs on across tiles (the producer loads the
// next tile while the MMAs of this one drain), and with two TMEM accumulators the
// epilogue of one tile overlaps the main loop of the next. The output staging sits
// after the ring, since the ring is never drained between tiles. Each tile's
// arithmetic is exactly gemm_tc_kernel's, so results are the same bits.
template <int MODE, bool BF, int NG, int MH>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                          TcArgs a) {
  using E = Epi<MODE, BF>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stages][stage_bytes] | output staging [stg_bytes] | barriers
  uint8_t* stg = smem + (size_t)a.stages * a.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + a.stg_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* acc_full = bars + 2 * kMaxStages;       // [2] accumulator ready (MMA -> epilogue)
  uint64_t* acc_empty = bars + 2 * kMaxStages + 2;  // [2] accumulator drained (epilogue -> MMA)
  uint64_t* epi_done = bars + 2 * kMaxStages + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = a.token_tiles * a.feat_ctas;
  const int n_stages_work = (a.k_blocks + a.kc - 1) / a.kc;  // pipeline stages of kc k-blocks per tile
  const int acc_cols = MH * a.mt;                            // TMEM columns of one accumulator
  uint32_t tmem_cols = 32;
  while ((int)tmem_cols < a.acc_bufs * acc_cols) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 4 * kEpiGroups);  // one arrival per epilogue warp
    }
    mbar_init(smem_u32(epi_done), 4 * kEpiGroups);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
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
  auto tile_tok0 = [&](int t) { return (t % a.token_tiles) * a.mt; };
  auto tile_feat0 = [&](int t) { return (t / a.token_tiles) * BM * MH; };
  // Stage layout as in gemm_tc_kernel.
  auto load_w = [&](uint8_t* dst, int chunk, int feat0, uint32_t fb) {
    if (a.tma3d) tma_load_3d(smem_u32(dst), &map_w, 0, feat0, chunk, fb);
    else tma_load_2d(smem_u32(dst), &map_w, chunk * BK, feat0, fb);
  };
  auto load_x = [&](uint8_t* dst, int chunk, int tok0, uint32_t fb) {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      uint8_t* d = dst + (size_t)g * a.kc * a.n_g * BK * 2;
      if (a.tma3d) tma_load_3d(smem_u32(d), &map_x, 0, tok0 + g * a.n_g, chunk, fb);
      else tma_load_2d(smem_u32(d), &map_x, chunk * BK, tok0 + g * a.n_g, fb);
    }
  };
  // Constant weights (w_static): the first tile's first stages of weights are
  // requested before waiting on the previous kernel.
  const int pre = a.w_static ? min(n_stages_work, a.stages) : 0;
  if (warp == 0 && lane == 0) {
    prefetch_map(&map_w);
    prefetch_map(&map_x);
    uint8_t* sa = smem;
    for (int it = 0; it < pre; ++it, sa += a.stage_bytes) {
      const uint32_t fb = smem_u32(&full[it]);
      mbar_add_tx(fb, a.w_bytes);
      load_w(sa, it * a.kc, tile_feat0(blockIdx.x), fb);
    }
  }
  // After a timeout anywhere in this launch every CTA that starts later skips
  // all of its tiles (read before the dependency wait, as in gemm_tc_kernel).
  const bool aborted = a.status && *reinterpret_cast<volatile int*>(a.status) == KVE_ERR_TIMEOUT;
  grid_dep_wait();
  grid_dep_launch();
  const int tile_first = aborted ? n_tiles : (int)blockIdx.x;
  const int tile_step = (int)gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- producer
      int issued = 0, s = 0;
      uint32_t ph = 0;
      uint8_t* sa = smem;
      bool ok = true;
      for (int tile = tile_first, ti = 0; ok && tile < n_tiles; tile += tile_step, ++ti) {
        const int tok0 = tile_tok0(tile), feat0 = tile_feat0(tile);
        int chunk = 0;
        for (int it = 0; it < n_stages_work; ++it) {
          if (issued >= a.stages && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, a.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[s]);
          if (ti == 0 && it < pre) {
            mbar_expect_tx(fb, a.stage_bytes - a.w_bytes);  // weight tile already requested
          } else {
            mbar_expect_tx(fb, a.stage_bytes);
            load_w(sa, chunk, feat0, fb);
          }
          load_x(sa + a.w_bytes, chunk, tok0, fb);
          ++issued;
          chunk += a.kc;
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
            sa = smem;
          } else {
            sa += a.stage_bytes;
          }
        }
      }
      // Early weight loads of stages the loop never reached (abort): arrive so
      // their phase completes once those bytes land.
      for (int it = issued; it < pre; ++it) mbar_arrive(smem_u32(&full[it]));
      if (issued < pre) issued = pre;
      // Do not leave while a bulk copy may still be writing this CTA's shared memory.
      for (int it = issued - a.stages < 0 ? 0 : issued - a.stages; it < issued; ++it)
        mbar_wait(smem_u32(&full[it % a.stages]), (uint32_t)(it / a.stages) & 1u, a.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(a.n_g);
      const uint64_t a0 = umma_desc(smem_u32(smem));
      const uint64_t b0 = umma_desc(smem_u32(smem) + a.w_bytes);
      const uint64_t stage_step = (uint64_t)(a.stage_bytes >> 4);
      constexpr uint64_t half_step = (uint64_t)((BM * BK * 2) >> 4);
      const uint64_t a_chunk = (uint64_t)((MH * BM * BK * 2) >> 4);
      const uint64_t b_chunk = (uint64_t)((a.n_g * BK * 2) >> 4);
      const uint64_t grp_step = (uint64_t)((a.kc * a.n_g * BK * 2) >> 4);
      constexpr uint64_t kstep = (UMMA_K * 2) >> 4;
      int s = 0;
      uint32_t ph = 0;
      uint64_t soff = 0;
      bool ok = true;
      for (int tile = tile_first, ti = 0; ok && tile < n_tiles; tile += tile_step, ++ti) {
        const int ab = a.acc_bufs == 2 ? (ti & 1) : 0;
        const int use = a.acc_bufs == 2 ? (ti >> 1) : ti;  // earlier tiles in this accumulator
        if (use > 0) {
          // The epilogue has drained this accumulator's previous tile.
          if (!mbar_wait(smem_u32(&acc_empty[ab]), (uint32_t)(use - 1) & 1u, a.status)) break;
          fence_after();
        }
        const uint32_t tacc = tmem_base + (uint32_t)(ab * acc_cols);
        int chunk = 0;
        for (int it = 0; it < n_stages_work; ++it) {
          if (!mbar_wait(smem_u32(&full[s]), ph, a.status)) {
            ok = false;
            break;
          }
          fence_after();
          const int nch = min(a.kc, a.k_blocks - chunk);  // a partial last stage multiplies only real chunks
          for (int j = 0; j < nch; ++j) {
            const uint64_t ad = a0 + soff + j * a_chunk, bd = b0 + soff + j * b_chunk;
#pragma unroll
            for (int kk = 0; kk < BK / UMMA_K; ++kk) {
              const uint32_t acc = (it > 0 || j > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
              for (int h = 0; h < MH; ++h)
#pragma unroll
                for (int g = 0; g < NG; ++g)
                  umma_bf16(tacc + h * a.mt + g * a.n_g, ad + h * half_step + kk * kstep,
                            bd + g * grp_step + kk * kstep, idesc, acc);
            }
          }
          chunk += a.kc;
          umma_commit(smem_u32(&empty[s]));
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
            soff = 0;
          } else {
            soff += stage_step;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&acc_full[ab]));  // fires once every issued MMA has completed
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    // As gemm_tc_kernel's, per tile, from accumulator ab; then the accumulator is
    // released to the MMA warp.
    static_assert(MH == 1 || MH == kEpiGroups, "one epilogue warpgroup per weight half");
    const int egrp = (warp - 2) / 4;
    const int half = MH == 1 ? 0 : egrp;
    const int quad = warp & 3;
    const int f_local = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(half * a.mt);
    const int etid = (threadIdx.x - 64) & 127;
    const int first_c0 = MH == 1 ? egrp * kRows : 0;
    constexpr int kStgBufE = kRows * E::W * E::ES;  // one staging buffer
    constexpr int kChunkStride = (MH == 1 ? kEpiGroups : 1) * kRows;
    int it = 0;  // chunks staged so far by this warpgroup (alternates its two buffers)
    for (int tile = tile_first, ti = 0; tile < n_tiles; tile += tile_step, ++ti) {
      const int tok0 = tile_tok0(tile);
      const int fbase = tile_feat0(tile) + half * BM;
      const int feat = fbase + f_local;
      const int col0 = MODE == KVE_EPI_SILU_MUL ? fbase / 2 : fbase;
      const float bias_f = ((MODE == KVE_EPI_BIAS || MODE == kEpiQkvRope) && feat < a.n) ? a.e.bias[feat] : 0.f;
      uint4 res_first[E::NPASS];  // the first chunk's per-row inputs load while the main loop runs
      if (first_c0 < a.mt) E::load_res(a, tok0 + first_c0, min(kRows, a.mt - first_c0), col0, etid, res_first);
      const int ab = a.acc_bufs == 2 ? (ti & 1) : 0;
      const int use = a.acc_bufs == 2 ? (ti >> 1) : ti;
      const bool have = mbar_wait(smem_u32(&acc_full[ab]), (uint32_t)use & 1u, a.status);
      fence_after();
      const uint32_t t_acc = t_lane + (uint32_t)(ab * acc_cols);
      bool first = true;
      for (int c0 = first_c0; c0 < a.mt; c0 += kChunkStride, ++it) {
        const int n = min(kRows, a.mt - c0);
        uint8_t* buf = stg + (egrp * 2 + (it & 1)) * kStgBufE;
        uint4 res[E::NPASS];
        if (first) {
#pragma unroll
          for (int i = 0; i < E::NPASS; ++i) res[i] = res_first[i];
          first = false;
        } else {
          E::load_res(a, tok0 + c0, n, col0, etid, res);
        }
        float v[32];
        tmem_load_cols(t_acc + c0, n, have, v);
        E::template stage<32>(buf, 0, n, f_local, v, bias_f);
        epi_bar(egrp);
        E::copy_out(a, buf, tok0 + c0, n, col0, etid, res);
      }
      // Every tcgen05.ld of this warp has completed (wait::ld): release the accumulator.
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[ab]));
      if (!have) break;
    }
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(epi_done));
  }
  if (warp == 1) {
    // Free TMEM only after the epilogue is done with it (bounded wait; freed either way).
    mbar_wait(smem_u32(epi_done), 0, a.status);
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// ---------------------------------------------------------- CTA-pair variant
// 2-CTA MMA (tcgen05 cta_group::2): the two CTAs of a cluster pair compute one
// 256-weight-row tile. Each holds its own 128 weight rows and HALF of the tile's
// tokens in shared memory; one MMA of M = 256 reads both CTAs' operands, and each
// CTA's TMEM receives its 128 rows x all tokens. Per SM this loads half the
// activation bytes of gemm_tc_kernel for the same work, which is what bounds the
// wide projections (gate_up, the vocabulary projection) at verify batches.
// Protocol: both CTAs' TMA loads signal the leader's (rank 0) full barriers, for
// which the leader expects both CTAs' bytes; the leader's single MMA thread issues
// every MMA and commits each stage's release and each tile's completion to the
// barriers of both CTAs (two commits, one per CTA); both epilogues drain their
// own TMEM and arrive on the leader's accumulator-empty barrier. Tiles are walked
// as in gemm_tc_persistent_kernel; a tile's arithmetic per output element is the
// same K-ordered MMA chain as gemm_tc_kernel's.
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                               uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive (once the issuing thread's earlier MMAs complete) on an mbarrier of
// either CTA of the pair, given by its shared::cluster address.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
// TMA into this CTA's shared memory, completing bytes on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// Instruction descriptor, kind::f16: D fp32, A/B bf16, both K-major, M = 256 (pair), N = n.
__device__ __forceinline__ uint32_t umma_idesc_pair(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
}

// LSP (a.lsplit): split-K inside the pair, as in gemm_tc_kernel - every tile's
// a.splits k-ranges accumulate into their own TMEM accumulators (one buffer).
template <int MODE, bool BF, int NG, bool LSP = false>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, TcArgs a) {
  static_assert(!LSP || NG == 1, "in-CTA split-K pair tiles are one token group");
  using E = Epi<MODE, BF>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [stages][stage_bytes] | output staging [stg_bytes] | barriers; the same offsets in both CTAs.
  uint8_t* stg = smem + (size_t)a.stages * a.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + a.stg_bytes);
  uint64_t* full = bars;                            // leader's: both CTAs' bytes of a stage
  uint64_t* empty = bars + kMaxStages;              // each CTA's own: stage consumed
  uint64_t* acc_full = bars + 2 * kMaxStages;       // [2] each CTA's own: accumulator ready
  uint64_t* acc_empty = bars + 2 * kMaxStages + 2;  // [2] leader's: drained by both epilogues
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kMaxStages + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int half_n = a.n_g >> 1;                             // tokens of a group held by each CTA
  const int n_tiles = a.token_tiles * a.feat_ctas;           // pair tiles of 256 weight rows
  // k-range r = k-blocks [range_lo(r), range_lo(r + 1)); one range without LSP.
  const int LS = LSP ? a.splits : 1;
  auto range_lo = [&](int r) { return LSP ? r * a.k_blocks / a.splits : (r ? a.k_blocks : 0); };
  int n_stages_work = (range_lo(1) + a.kc - 1) / a.kc;  // per tile
  if constexpr (LSP)
    for (int r = 1; r < LS; ++r) n_stages_work += (range_lo(r + 1) - range_lo(r) + a.kc - 1) / a.kc;
  // Walk to the next stage of a tile: `chunk` is its first k-block, in range r = [rlo, rhi).
  auto next_stage = [&](int& r, int& chunk, int& rlo, int& rhi) {
    chunk += a.kc;
    if (LSP && chunk >= rhi) {
      ++r;
      rlo = chunk = rhi;
      rhi = range_lo(r + 1);
    }
  };
  const int kb1_0 = range_lo(1);
  const int acc_cols = a.mt * LS;
  uint32_t tmem_cols = 32;
  while ((int)tmem_cols < a.acc_bufs * acc_cols) tmem_cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), 2 * 4 * kEpiGroups);  // every epilogue warp of both CTAs
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  // Both CTAs' barriers are initialised (and TMEM allocated) before either CTA
  // signals the other's.
  fence_before();
  cluster_sync();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t lead_full = map_to(smem_u32(full), 0);  // leader's full[0]; entries 8 bytes apart
  const uint32_t lead_acc_empty = map_to(smem_u32(acc_empty), 0);
  const uint32_t peer_empty = map_to(smem_u32(empty), rank ^ 1u);
  const uint32_t peer_acc_full = map_to(smem_u32(acc_full), rank ^ 1u);
  // Tile t: token tiles fastest (the pairs of a round share the weight tiles), or
  // with LSP feature tiles fastest (they share the token tiles, as in gemm_tc_kernel).
  auto tile_tok0 = [&](int t) { return (LSP ? t / a.feat_ctas : t % a.token_tiles) * a.mt; };
  auto tile_feat0 = [&](int t) {  // this CTA's rows
    return (LSP ? t % a.feat_ctas : t / a.token_tiles) * 2 * BM + (int)rank * BM;
  };
  // Stage layout: weights [kc][128][64], then per token group this CTA's half
  // [kc][n_g / 2][64] (SW128 K-major slabs).
  auto load_w = [&](uint8_t* dst, int chunk, int feat0, uint32_t fb) {
    if (a.tma3d) tma_load_3d_pair(smem_u32(dst), &map_w, 0, feat0, chunk, fb);
    else tma_load_2d_pair(smem_u32(dst), &map_w, chunk * BK, feat0, fb);
  };
  auto load_x = [&](uint8_t* dst, int chunk, int tok0, uint32_t fb) {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      uint8_t* d = dst + (size_t)g * a.kc * half_n * BK * 2;
      const int row = tok0 + g * a.n_g + (int)rank * half_n;
      if (a.tma3d) tma_load_3d_pair(smem_u32(d), &map_x, 0, row, chunk, fb);
      else tma_load_2d_pair(smem_u32(d), &map_x, chunk * BK, row, fb);
    }
  };
  const int pre = a.w_static ? min(n_stages_work, a.stages) : 0;
  const int pair_idx = (int)(blockIdx.x >> 1);
  if (warp == 0 && lane == 0) {
    prefetch_map(&map_w);
    prefetch_map(&map_x);
    uint8_t* sa = smem;
    int r = 0, chunk = 0, rlo = 0, rhi = kb1_0;
    for (int it = 0; it < pre; ++it, sa += a.stage_bytes) {
      if (leader) mbar_add_tx(smem_u32(&full[it]), 2 * a.w_bytes);
      load_w(sa, chunk, tile_feat0(pair_idx), lead_full + 8u * it);
      next_stage(r, chunk, rlo, rhi);
    }
  }
  // Read before the dependency wait, as in gemm_tc_kernel.
  const bool aborted = a.status && *reinterpret_cast<volatile int*>(a.status) == KVE_ERR_TIMEOUT;
  grid_dep_wait();
  grid_dep_launch();
  const int tile_first = aborted ? n_tiles : pair_idx;
  const int tile_step = (int)(gridDim.x >> 1);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- producer
      int issued = 0, s = 0;
      uint32_t ph = 0;
      uint8_t* sa = smem;
      bool ok = true;
      for (int tile = tile_first, ti = 0; ok && tile < n_tiles; tile += tile_step, ++ti) {
        const int tok0 = tile_tok0(tile), feat0 = tile_feat0(tile);
        int r = 0, chunk = 0, rlo = 0, rhi = kb1_0;
        for (int it = 0; it < n_stages_work; ++it) {
          if (issued >= a.stages && !mbar_wait(smem_u32(&empty[s]), ph ^ 1u, a.status)) {
            ok = false;
            break;
          }
          const uint32_t fb = lead_full + 8u * s;
          if (ti == 0 && it < pre) {
            if (leader) mbar_expect_tx(smem_u32(&full[s]), 2 * (a.stage_bytes - a.w_bytes));
          } else {
            if (leader) mbar_expect_tx(smem_u32(&full[s]), 2 * a.stage_bytes);
            load_w(sa, chunk, feat0, fb);
          }
          load_x(sa + a.w_bytes, chunk, tok0, fb);
          ++issued;
          next_stage(r, chunk, rlo, rhi);
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
            sa = smem;
          } else {
            sa += a.stage_bytes;
          }
        }
      }
      if (leader) {
        // Early weight loads of stages the loop never reached (abort): arrive so
        // their phase completes once the bytes land. Then wait for the bytes of
        // the last stages of both CTAs, so that neither leaves with a copy in flight.
        for (int it = issued; it < pre; ++it) mbar_arrive(smem_u32(&full[it]));
        if (issued < pre) issued = pre;
        for (int it = issued - a.stages < 0 ? 0 : issued - a.stages; it < issued; ++it)
          mbar_wait(smem_u32(&full[it % a.stages]), (uint32_t)(it / a.stages) & 1u, a.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (leader)
    if (leader && lane == 0) {
      const uint32_t idesc = umma_idesc_pair(a.n_g);
      const uint64_t a0 = umma_desc(smem_u32(smem));
      const uint64_t b0 = umma_desc(smem_u32(smem) + a.w_bytes);
      const uint64_t stage_step = (uint64_t)(a.stage_bytes >> 4);
      const uint64_t a_chunk = (uint64_t)((BM * BK * 2) >> 4);
      const uint64_t b_chunk = (uint64_t)((half_n * BK * 2) >> 4);
      const uint64_t grp_step = (uint64_t)((a.kc * half_n * BK * 2) >> 4);
      constexpr uint64_t kstep = (UMMA_K * 2) >> 4;
      int s = 0;
      uint32_t ph = 0;
      uint64_t soff = 0;
      bool ok = true;
      for (int tile = tile_first, ti = 0; ok && tile < n_tiles; tile += tile_step, ++ti) {
        const int ab = a.acc_bufs == 2 ? (ti & 1) : 0;
        const int use = a.acc_bufs == 2 ? (ti >> 1) : ti;
        if (use > 0) {
          if (!mbar_wait(smem_u32(&acc_empty[ab]), (uint32_t)(use - 1) & 1u, a.status)) break;
          fence_after();
        }
        const uint32_t tacc0 = tmem_base + (uint32_t)(ab * acc_cols);
        int r = 0, chunk = 0, rlo = 0, rhi = kb1_0;
        for (int it = 0; it < n_stages_work; ++it) {
          if (!mbar_wait(smem_u32(&full[s]), ph, a.status)) {
            ok = false;
            break;
          }
          fence_after();
          const int nch = min(a.kc, rhi - chunk);  // a range's partial last stage multiplies only its own chunks
          const uint32_t tacc = tacc0 + (LSP ? (uint32_t)(r * a.mt) : 0u);
          for (int j = 0; j < nch; ++j) {
            const uint64_t ad = a0 + soff + j * a_chunk, bd = b0 + soff + j * b_chunk;
#pragma unroll
            for (int kk = 0; kk < BK / UMMA_K; ++kk) {
              const uint32_t acc = (chunk > rlo || j > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
              for (int g = 0; g < NG; ++g)
                umma_bf16_pair(tacc + g * a.n_g, ad + kk * kstep, bd + g * grp_step + kk * kstep, idesc, acc);
            }
          }
          next_stage(r, chunk, rlo, rhi);
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(peer_empty + 8u * s);
          if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
            soff = 0;
          } else {
            soff += stage_step;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[ab]));
        umma_commit_pair(peer_acc_full + 8u * ab);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int egrp = (warp - 2) / 4;
    const int quad = warp & 3;
    const int f_local = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(quad * 32) << 16);
    const int etid = (threadIdx.x - 64) & 127;
    const int first_c0 = egrp * kRows;
    constexpr int kStgBufE = kRows * E::W * E::ES;
    constexpr int kChunkStride = kEpiGroups * kRows;
    int it = 0;
    for (int tile = tile_first, ti = 0; tile < n_tiles; tile += tile_step, ++ti) {
      const int tok0 = tile_tok0(tile);
      const int fbase = tile_feat0(tile);
      const int feat = fbase + f_local;
      const int col0 = MODE == KVE_EPI_SILU_MUL ? fbase / 2 : fbase;
      const float bias_f = ((MODE == KVE_EPI_BIAS || MODE == kEpiQkvRope) && feat < a.n) ? a.e.bias[feat] : 0.f;
      uint4 res_first[E::NPASS];
      if (first_c0 < a.mt) E::load_res(a, tok0 + first_c0, min(kRows, a.mt - first_c0), col0, etid, res_first);
      const int ab = a.acc_bufs == 2 ? (ti & 1) : 0;
      const int use = a.acc_bufs == 2 ? (ti >> 1) : ti;
      const bool have = mbar_wait(smem_u32(&acc_full[ab]), (uint32_t)use & 1u, a.status);
      fence_after();
      const uint32_t t_acc = t_lane + (uint32_t)(ab * acc_cols);
      bool first = true;
      for (int c0 = first_c0; c0 < a.mt; c0 += kChunkStride, ++it) {
        const int n = min(kRows, a.mt - c0);
        uint8_t* buf = stg + (egrp * 2 + (it & 1)) * kStgBufE;
        uint4 res[E::NPASS];
        if (first) {
#pragma unroll
          for (int i = 0; i < E::NPASS; ++i) res[i] = res_first[i];
          first = false;
        } else {
          E::load_res(a, tok0 + c0, n, col0, etid, res);
        }
        float v[32];
        if constexpr (!LSP) {
          tmem_load_cols(t_acc + c0, n, have, v);
        } else {
          // The LS partials summed from zero in range order (as in gemm_tc_kernel).
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
          for (int u = 0; u < LS; ++u) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (h == 1 && n <= 16) break;
              float p[16];
              if (have) {
                tmem_ld16(t_acc + (uint32_t)(u * a.mt) + c0 + 16 * h, p);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) p[i] = 0.f;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) v[16 * h + i] += p[i];
            }
          }
        }
        E::template stage<32>(buf, 0, n, f_local, v, bias_f);
        epi_bar(egrp);
        E::copy_out(a, buf, tok0 + c0, n, col0, etid, res);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead_acc_empty + 8u * ab);
      if (!have) break;
    }
  }
  // Both CTAs are done with every MMA, copy and barrier of the pair before TMEM
  // is released and either CTA exits.
  fence_before();
  cluster_sync();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host
int make_map(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled unavailable");
  CUresult r = CUDA_SUCCESS;
  auto encode = [&](CUtensorMap* m) {
    cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
  };
  // key: rows (24 bits) | k (20) | box rows (9)
  const bool packable = rows >= 0 && rows < (1 << 24) && k >= 0 && k < (1 << 20) && box_rows >= 0 && box_rows < 512;
  const bool ok = packable ? cached_map(map, ptr, (uint64_t)rows | (uint64_t)k << 24 | (uint64_t)box_rows << 44, encode)
                           : encode(map);
  if (!ok) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KVE_OK;
}

// The same [rows, k] matrix as a 3-D tensor (64, rows, k / 64) whose third
// dimension steps 128 bytes along k: one box {64, box_rows, kc} brings kc
// consecutive 64-wide k-chunks, each landing as its own SW128 [box_rows][64]
// tile. Needs k % 64 == 0 (a partial chunk would read the next row).
int make_map3(CUtensorMap* map, const void* ptr, int rows, int k, int box_rows, int kc) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled unavailable");
  CUresult r = CUDA_SUCCESS;
  auto encode = [&](CUtensorMap* m) {
    cuuint64_t dims[3] = {(cuuint64_t)BK, (cuuint64_t)rows, (cuuint64_t)(k / BK)};
    cuuint64_t strides[2] = {(cuuint64_t)k * 2, (cuuint64_t)BK * 2};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, (cuuint32_t)kc};
    cuuint32_t estr[3] = {1, 1, 1};
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
  };
  // key: rows (24 bits) | k (20) | box rows (9) | k-chunks per box (3)
  const bool packable = rows >= 0 && rows < (1 << 24) && k >= 0 && k < (1 << 20) && box_rows >= 0 &&
                        box_rows < 512 && kc >= 0 && kc < 8;
  const bool ok = packable ? cached_map(map, ptr,
                                        (uint64_t)rows | (uint64_t)k << 24 | (uint64_t)box_rows << 44 |
                                            (uint64_t)kc << 53,
                                        encode)
                           : encode(map);
  if (!ok) return set_error(KVE_ERR_CUDA, "kve_gemm: cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return KVE_OK;
}

struct Plan {
  int mt, ng, n_g, token_tiles, feat_tiles, k_blocks, splits, stages, rch, stg_off;
  int mh, kc, tma3d;  // weight halves per CTA, k-chunks per stage, 3-D tensor maps
  uint32_t stage_bytes, w_bytes;
  int grid_x;         // CTAs without split-K (fewer than the tiles when persistent)
  int acc_bufs, stg_bytes;
  bool pair;          // CTA pairs with the 2-CTA MMA (gemm_tc_pair_kernel)
  int bmt;            // weight rows per MMA tile: 128, or 64 (rows64)
  bool lsplit;        // split-K ranges summed inside one CTA (no cluster exchange)
};

typedef void (*GemmKernel)(CUtensorMap, CUtensorMap, TcArgs);

template <int MODE, bool BF, int NG, int MH, bool P>
GemmKernel kernel_of() {
  if constexpr (P) return gemm_tc_persistent_kernel<MODE, BF, NG, MH>;
  else return gemm_tc_kernel<MODE, BF, NG, MH>;
}

// The in-CTA split-K kernels (one token group): one-tile (one 128-row half) and CTA pairs.
GemmKernel lsplit_pair_kernel_for(int mode, int out_dtype) {
  const bool bf = out_dtype == KVE_BF16;
  switch (mode) {
    case KVE_EPI_STORE:
      return bf ? gemm_tc_pair_kernel<KVE_EPI_STORE, true, 1, true> : gemm_tc_pair_kernel<KVE_EPI_STORE, false, 1, true>;
    case KVE_EPI_BIAS:
      return bf ? gemm_tc_pair_kernel<KVE_EPI_BIAS, true, 1, true> : gemm_tc_pair_kernel<KVE_EPI_BIAS, false, 1, true>;
    case KVE_EPI_RESIDUAL:
      return bf ? gemm_tc_pair_kernel<KVE_EPI_RESIDUAL, true, 1, true>
                : gemm_tc_pair_kernel<KVE_EPI_RESIDUAL, false, 1, true>;
    case KVE_EPI_SILU_MUL:
      return bf ? gemm_tc_pair_kernel<KVE_EPI_SILU_MUL, true, 1, true>
                : gemm_tc_pair_kernel<KVE_EPI_SILU_MUL, false, 1, true>;
    case kEpiQkvRope:
      return bf ? gemm_tc_pair_kernel<kEpiQkvRope, true, 1, true> : nullptr;
    default:
      return nullptr;
  }
}
GemmKernel lsplit_kernel_for(int mode, int out_dtype) {
  const bool bf = out_dtype == KVE_BF16;
  switch (mode) {
    case KVE_EPI_STORE:
      return bf ? gemm_tc_kernel<KVE_EPI_STORE, true, 1, 1, BM, true> : gemm_tc_kernel<KVE_EPI_STORE, false, 1, 1, BM, true>;
    case KVE_EPI_BIAS:
      return bf ? gemm_tc_kernel<KVE_EPI_BIAS, true, 1, 1, BM, true> : gemm_tc_kernel<KVE_EPI_BIAS, false, 1, 1, BM, true>;
    case KVE_EPI_RESIDUAL:
      return bf ? gemm_tc_kernel<KVE_EPI_RESIDUAL, true, 1, 1, BM, true>
                : gemm_tc_kernel<KVE_EPI_RESIDUAL, false, 1, 1, BM, true>;
    case KVE_EPI_SILU_MUL:
      return bf ? gemm_tc_kernel<KVE_EPI_SILU_MUL, true, 1, 1, BM, true>
                : gemm_tc_kernel<KVE_EPI_SILU_MUL, false, 1, 1, BM, true>;
    case kEpiQkvRope:
      return bf ? gemm_tc_kernel<kEpiQkvRope, true, 1, 1, BM, true> : nullptr;
    default:
      return nullptr;
  }
}

template <int NG, int MH, bool P>
GemmKernel kernel_for_shape(int mode, bool bf) {
  switch (mode) {
    case KVE_EPI_BIAS:
      return bf ? kernel_of<KVE_EPI_BIAS, true, NG, MH, P>() : kernel_of<KVE_EPI_BIAS, false, NG, MH, P>();
    case KVE_EPI_RESIDUAL:
      return bf ? kernel_of<KVE_EPI_RESIDUAL, true, NG, MH, P>() : kernel_of<KVE_EPI_RESIDUAL, false, NG, MH, P>();
    case KVE_EPI_SILU_MUL:
      return bf ? kernel_of<KVE_EPI_SILU_MUL, true, NG, MH, P>() : kernel_of<KVE_EPI_SILU_MUL, false, NG, MH, P>();
    case kEpiQkvRope: return bf ? kernel_of<kEpiQkvRope, true, NG, MH, P>() : nullptr;  // bf16 only
    default: return bf ? kernel_of<KVE_EPI_STORE, true, NG, MH, P>() : kernel_of<KVE_EPI_STORE, false, NG, MH, P>();
  }
}

template <int MODE, bool BF>
GemmKernel pair_kernel_of(int ng) {
  return ng == 2 ? gemm_tc_pair_kernel<MODE, BF, 2> : gemm_tc_pair_kernel<MODE, BF, 1>;
}
GemmKernel pair_kernel_for(int mode, int out_dtype, int ng) {
  const bool bf = out_dtype == KVE_BF16;
  switch (mode) {
    case KVE_EPI_BIAS: return bf ? pair_kernel_of<KVE_EPI_BIAS, true>(ng) : pair_kernel_of<KVE_EPI_BIAS, false>(ng);
    case KVE_EPI_RESIDUAL:
      return bf ? pair_kernel_of<KVE_EPI_RESIDUAL, true>(ng) : pair_kernel_of<KVE_EPI_RESIDUAL, false>(ng);
    case KVE_EPI_SILU_MUL:
      return bf ? pair_kernel_of<KVE_EPI_SILU_MUL, true>(ng) : pair_kernel_of<KVE_EPI_SILU_MUL, false>(ng);
    case kEpiQkvRope: return bf ? pair_kernel_of<kEpiQkvRope, true>(ng) : nullptr;
    default: return bf ? pair_kernel_of<KVE_EPI_STORE, true>(ng) : pair_kernel_of<KVE_EPI_STORE, false>(ng);
  }
}

// 64-row one-tile kernels (bf16 output, one token group, one weight half).
GemmKernel rows64_kernel_for(int mode, int out_dtype) {
  if (out_dtype != KVE_BF16) return nullptr;
  switch (mode) {
    case KVE_EPI_BIAS: return gemm_tc_kernel<KVE_EPI_BIAS, true, 1, 1, 64>;
    case KVE_EPI_RESIDUAL: return gemm_tc_kernel<KVE_EPI_RESIDUAL, true, 1, 1, 64>;
    case KVE_EPI_SILU_MUL: return gemm_tc_kernel<KVE_EPI_SILU_MUL, true, 1, 1, 64>;
    case kEpiQkvRope: return gemm_tc_kernel<kEpiQkvRope, true, 1, 1, 64>;
    default: return gemm_tc_kernel<KVE_EPI_STORE, true, 1, 1, 64>;
  }
}

// Token groups x weight halves: (1, 1), (2, 1) for tiles above 256 tokens, (1, 2);
// one tile per CTA or persistent.
GemmKernel kernel_for(int mode, int out_dtype, int ng, int mh, bool persist) {
  const bool bf = out_dtype == KVE_BF16;
  if (persist) {
    if (mh == 2) return kernel_for_shape<1, 2, true>(mode, bf);
    return ng == 2 ? kernel_for_shape<2, 1, true>(mode, bf) : kernel_for_shape<1, 1, true>(mode, bf);
  }
  if (mh == 2) return kernel_for_shape<1, 2, false>(mode, bf);
  return ng == 2 ? kernel_for_shape<2, 1, false>(mode, bf) : kernel_for_shape<1, 1, false>(mode, bf);
}

void configure_kernel() {
  static std::once_flag once;
  std::call_once(once, [] {
    for (int mode = KVE_EPI_STORE; mode <= kEpiQkvRope; ++mode)
      for (int dt : {KVE_F32, KVE_BF16})
        for (int shape = 0; shape < 3; ++shape)
          for (bool persist : {false, true}) {
            GemmKernel kern = kernel_for(mode, dt, shape == 1 ? 2 : 1, shape == 2 ? 2 : 1, persist);
            if (kern) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
            if (shape < 2 && persist) {
              GemmKernel pk = pair_kernel_for(mode, dt, shape == 1 ? 2 : 1);
              if (pk) cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
            }
            if (shape == 0 && !persist) {
              GemmKernel rk = rows64_kernel_for(mode, dt);
              if (rk) cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
              GemmKernel lk = lsplit_kernel_for(mode, dt);
              if (lk) cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
              GemmKernel lp = lsplit_pair_kernel_for(mode, dt);
              if (lp) cudaFuncSetAttribute(lp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kSmemLimit - 512));
            }
          }
  });
}

// Concurrent CTAs for each cluster size with one CTA per SM (queried once).
const int* cluster_capacity() {
  static int cap[kMaxSplits + 1];
  static std::once_flag once;
  std::call_once(once, [] {
    configure_kernel();
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    for (int s = 1; s <= kMaxSplits; ++s) {
      cap[s] = (sms / s) * s;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, s);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmemLimit - 512;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 1;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = s;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kernel_for(KVE_EPI_STORE, KVE_BF16, 1, 1, false), &cfg) == cudaSuccess && n > 0)
        cap[s] = n * s;
    }
    cudaGetLastError();
  });
  return cap;
}

// Launch-time model (microseconds) used to pick split-K, token tiling, weight
// halves per CTA and k-chunks per stage, fitted to B200 measurements of this
// kernel and of TMA streaming alone:
// * a pipeline stage costs the largest of its TMA issue time (about 0.12 us plus
//   0.1 us per box and k-chunk), the load latency spread over the stages in
//   flight, and its MMAs;
// * a cluster exchange costs a fixed part plus a part per token of the tile;
// * the epilogue costs a fixed part plus a part per token each warpgroup drains.
constexpr double kLoadLatencyUs = 2.0;
constexpr size_t kAvail = kSmemLimit - 2048;  // stage ring budget (alignment slack, barriers, margin)
// Output staging a CTA that walks several tiles keeps beside its stage ring (the
// ring is never drained between tiles): two buffers of kRows staged output rows
// per epilogue warpgroup; row_bytes is one staged row (128 outputs, 64 for SwiGLU).
size_t persist_staging(int row_bytes) { return (size_t)kEpiGroups * 2 * kRows * row_bytes; }
// A CTA's fixed cost outside its main loop: barrier and TMEM set-up and the first
// load round trip (measured: a persistent walk over 9 tiles saved about 2.3 us per
// tile against nine waves of one-tile CTAs with the same stages).
constexpr double kStartUs = 2.0;
// x_rows: activation rows a CTA stages per k-chunk (all mt tokens, or half of
// them in a CTA pair); the MMA term is this SM's share (mh x 128 rows x mt).
double stage_us(int mh, int ng, int mt, int kc, size_t avail, int x_rows);
double stage_us(int mh, int ng, int mt, int kc, size_t avail) { return stage_us(mh, ng, mt, kc, avail, mt); }
double stage_us(int mh, int ng, int mt, int kc, size_t avail, int x_rows) {
  const size_t bytes = (size_t)(mh * BM + x_rows) * BK * 2 * kc;
  int stages = (int)(avail / bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return 1e9;
  const double issue = 0.12 + 0.10 * (1 + ng) * kc;
  const double lat = kLoadLatencyUs / stages;
  const double mma = (double)mh * BM * mt * BK * kc * 2 / (7.7e3 * 1.9e3);  // 7.7k flop/clk/SM at 1.9 GHz
  return fmax(issue, fmax(lat, mma));
}
double exchange_us(int m_cta, int s) { return s > 1 ? 2.5 + 0.25 * s + 0.04 * m_cta : 0.0; }
double epilogue_us(int tokens_per_group) { return 0.5 + 0.03 * tokens_per_group; }

inline int round16(int x) { return (x + 15) / 16 * 16; }

// One launch shape: token_tiles tiles of ng x n_g tokens, mh weight halves of
// 128 rows per CTA, kc k-chunks of 64 per pipeline stage.
struct TileConfig {
  int token_tiles, ng, n_g, mh, kc;
  bool persist;  // CTAs walk several tiles (no split-K, more tiles than resident CTAs)
  bool pair;     // CTA pairs (2-CTA MMA) on 256-row tiles; always tile-walking
  double us;
};

// Pair forcing through kve_gemm_force_pair: 0 = the model's choice, 1 = never, 2 = where valid.
std::atomic<int> g_force_pair{0};

// Launch of CTA pairs: pair tiles of 256 weight rows x mt tokens walked by the
// resident pairs; per SM a stage holds 128 weight rows and mt / 2 token rows.
constexpr double kPairStartUs = 0.5;  // cluster barrier after set-up
double pair_us(int feat_tiles, int k_blocks, const TileConfig& c, int row_bytes) {
  const int* cap = cluster_capacity();
  const long long tiles = (long long)((feat_tiles + 1) / 2) * c.token_tiles;
  const long long pairs = cap[2] / 2 > 0 ? cap[2] / 2 : 1;
  const long long rounds = (tiles + pairs - 1) / pairs;
  const int mt = c.ng * c.n_g;
  const int iters = (k_blocks + c.kc - 1) / c.kc;
  const double main = iters * stage_us(1, c.ng, mt, c.kc, kAvail - persist_staging(row_bytes), mt / 2);
  const double epi = epilogue_us((mt + kEpiGroups - 1) / kEpiGroups);
  return kStartUs + kPairStartUs + (2 * mt <= 512 ? rounds * fmax(main, epi) + epi : rounds * (main + epi));
}

// A persistent launch: each CTA walks ceil(tiles / CTAs) tiles with its stage ring
// running on across tiles; the epilogue overlaps the next tile's main loop when
// two TMEM accumulators fit, else it follows every tile. The staging it keeps
// beside the ring leaves fewer stages in flight. `legacy` prices the one-tile-per-
// CTA launches only, without start costs (the model the split factor is chosen by).
double config_us(int feat_tiles, int k_blocks, int s, const TileConfig& c, int row_bytes, bool legacy) {
  const int* cap = cluster_capacity();
  const long long ctas = (long long)((feat_tiles + c.mh - 1) / c.mh) * c.token_tiles * s;
  const long long waves = (ctas + cap[s] - 1) / cap[s];
  const int mt = c.ng * c.n_g;
  const int iters = ((k_blocks + s - 1) / s + c.kc - 1) / c.kc;
  const int per_group = c.mh == 1 ? (mt + kEpiGroups - 1) / kEpiGroups : mt;
  const double epi = epilogue_us(per_group);
  if (c.persist) {
    const double main = iters * stage_us(c.mh, c.ng, mt, c.kc, kAvail - persist_staging(row_bytes));
    return kStartUs + (2 * c.mh * mt <= 512 ? waves * fmax(main, epi) + epi : waves * (main + epi));
  }
  const double per_wave = iters * stage_us(c.mh, c.ng, mt, c.kc, kAvail) + exchange_us(mt, s) + epi;
  return waves * (per_wave + (legacy ? 0.0 : kStartUs));
}

TileConfig token_tiling(int m, int t) {
  TileConfig tt{};
  const int per = (m + t - 1) / t;
  tt.token_tiles = t;
  if (per <= kMaxNG) {
    tt.ng = 1;
    tt.n_g = round16(per < 16 ? 16 : per);
  } else {
    tt.ng = 2;
    tt.n_g = round16((per + 1) / 2);
  }
  tt.mh = 1;
  tt.kc = 1;
  return tt;
}

// The cheapest token tiling by the model, preferring fewer tiles unless more
// are clearly faster. Each tiling takes the most k-chunks per stage that still
// leave two pipeline stages (fewer, larger TMA boxes measured faster than more
// stages in flight); several k-chunks are single-split shapes on the 3-D maps
// (k % 64 == 0). Two weight halves per CTA (256 weight rows sharing each
// activation tile) measured faster only for prompt-sized batches (m >= kLargeM).
// None of these choices changes a row's reduction order.
constexpr int kLargeM = 2048;
int chunks_for(int mh, int mt, int s, bool tma3d, size_t avail) {
  if (s > 1 || !tma3d) return 1;
  for (int kc = 4; kc > 1; kc /= 2)
    if ((size_t)(mh * BM + mt) * BK * 2 * kc * 2 <= avail) return kc;
  return 1;
}

// A pair tile needs an even number of tokens per group on each CTA's 8-row
// swizzle atoms: n_g a multiple of 16 (always) and at least 16.
bool pair_ok(const TileConfig& c, int s, int feat_tiles) {
  return s == 1 && c.mh == 1 && feat_tiles >= 2 && c.n_g >= 16 && c.n_g % 16 == 0;
}

TileConfig best_config(int m, int feat_tiles, int k_blocks, int s, bool tma3d, int row_bytes, bool legacy) {
  int t_min = (m + 383) / 384;
  if (t_min < 1) t_min = 1;
  // The best one-tile-per-CTA shape (by the model without start costs, which
  // ranks those shapes as measured) and the best persistent shape.
  TileConfig best = token_tiling(m, t_min), best_p = best;
  best.us = best_p.us = 1e30;
  for (int t = t_min; t <= (m + 15) / 16; ++t) {
    TileConfig c = token_tiling(m, t);
    const int mt = c.ng * c.n_g;
    if ((long long)(t - 1) * mt >= m) continue;  // an empty trailing tile
    for (int mh = 1; mh <= (m >= kLargeM ? 2 : 1); ++mh) {
      if (mh == 2 && (s > 1 || c.ng == 2 || mt > 256 || feat_tiles < 2)) continue;
      c.mh = mh;
      c.persist = false;
      c.kc = chunks_for(mh, mt, s, tma3d, kAvail);
      c.us = config_us(feat_tiles, k_blocks, s, c, row_bytes, true);
      if (c.us < best.us * 0.97) best = c;
      const long long ctas = (long long)((feat_tiles + mh - 1) / mh) * t * s;
      if (!legacy && s == 1 && ctas > cluster_capacity()[1]) {
        c.persist = true;
        c.kc = chunks_for(mh, mt, s, tma3d, kAvail - persist_staging(row_bytes));
        c.us = config_us(feat_tiles, k_blocks, s, c, row_bytes, false);
        if (c.us < best_p.us * 0.97) best_p = c;
      }
      c.persist = false;
      const int fp = g_force_pair.load();
      if (!legacy && fp != 1 && pair_ok(c, s, feat_tiles)) {
        TileConfig q = c;
        q.pair = true;
        q.kc = chunks_for(1, mt / 2, s, tma3d, kAvail - persist_staging(row_bytes));
        q.us = pair_us(feat_tiles, k_blocks, q, row_bytes) * (fp == 2 ? 0.0 : 1.0);
        if (q.us < best_p.us * 0.97) best_p = q;
      }
    }
  }
  if (legacy) return best;
  best.us = config_us(feat_tiles, k_blocks, s, best, row_bytes, false);  // with its start costs
  return best_p.us < best.us * 0.97 ? best_p : best;
}

// Split-K factor: a function of (n, k) only, so a row's reduction order never
// depends on how many tokens are processed together (draft and verify passes
// agree bit for bit whatever the batch, prompts included - a draft identical to
// the target is accepted in full under continuous batching). It minimises the
// modelled time summed over small, medium and large decode batches, each with
// its best shape.
int choose_splits(int feat_tiles, int k_blocks, bool tma3d) {
  int best = 1;
  double best_t = 1e30;
  for (int s = 1; s <= kMaxSplits; ++s) {
    if (s > 1 && k_blocks / s < 2) break;
    double t = 0;
    for (int m_ref : {16, 64, 256}) t += best_config(m_ref, feat_tiles, k_blocks, s, tma3d, 256, true).us;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

// Shape forced through kve_gemm_force_shape (0 = the model's choice).
std::atomic<int> g_force_t{0}, g_force_mh{0}, g_force_kc{0};
// Split-K factor forced through kve_gemm_force_splits (0 = the function of (n, k)).
std::atomic<int> g_force_s{0};
// In-CTA split-K through kve_gemm_force_local_split: 0 = the rule, 1 = never, 2 = where valid.
std::atomic<int> g_force_local{0};

// In-CTA split-K for prompt-sized batches. The split factor S is a function of
// (n, k) only, so a prompt-sized batch splits K like a decode batch does; over a
// cluster that costs an exchange of fp32 partials about as long as the main loop
// (three rounds of 128 x 384 partials per tile for the 3B down projection). With
// many tiles to spread over the SMs, one CTA can instead compute all S ranges of
// its tile, range r into its own TMEM accumulator (S x mt <= 512 columns), and sum
// them in the epilogue in the same order from the same zero start: the same bits
// as the cluster reduction, without the exchange. Where the features allow, the
// tiles run on CTA pairs (2-CTA MMA, 256 weight rows; each SM stages half of the
// tokens, so 85 instead of 64 FLOP per staged byte at 128 tokens), walked by the
// resident pairs with one accumulator set per pair. Both forms run the feature
// tiles fastest: 3B down over 8448 rows 0.56 ms over a cluster, 0.50 ms on one-CTA
// tiles in token order (1.45 GB read from DRAM per launch), 0.41 ms on pairs in
// feature order (0.52 GB).
void try_local_split(Plan& p, int m, int row_bytes) {
  const int force = g_force_local.load();
  if (force == 1 || p.splits < 2 || !p.tma3d) return;
  if (force != 2 && m < kLargeM) return;
  int mt = 512 / p.splits / 16 * 16;  // tokens per tile: S accumulators fill at most the 512 TMEM columns
  if (mt > kMaxNG) mt = kMaxNG;
  if (mt < 16) return;
  const int per = round16(m < mt ? (m < 16 ? 16 : m) : mt);
  const int kc = chunks_for(1, per, 1, true, kAvail);
  const uint32_t w_bytes = (uint32_t)(BM * BK * 2 * kc);
  const uint32_t stage_bytes = w_bytes + (uint32_t)(per * BK * 2 * kc);
  const int stages = (int)std::min<size_t>(kMaxStages, kAvail / stage_bytes);
  // Two stages, and the drained ring must hold the epilogue's four output staging buffers.
  if (stages < 2 || (size_t)stages * stage_bytes < 4 * (size_t)kRows * BM * 4) return;
  p.lsplit = true;
  p.mt = p.n_g = per;
  p.ng = 1;
  p.mh = 1;
  p.pair = false;
  p.token_tiles = (m + per - 1) / per;
  p.kc = kc;
  p.w_bytes = w_bytes;
  p.stage_bytes = stage_bytes;
  p.stages = stages;
  p.stg_bytes = 0;
  p.acc_bufs = 1;
  p.rch = per;
  p.stg_off = 0;
  p.grid_x = p.token_tiles * p.feat_tiles;
  // Pairs only for an even number of 128-row feature tiles: an odd one leaves half of
  // every last pair tile idle (the 0.5B down, 7 tiles: 0.158 ms as pairs against
  // 0.145-0.150 ms on one-CTA tiles over 8192 rows).
  const int fp = g_force_pair.load();
  if (fp == 1 || p.feat_tiles < 2 || (fp != 2 && p.feat_tiles % 2) || per < 32 || per % 16) return;
  const size_t stg = persist_staging(row_bytes);
  const int kc2 = chunks_for(1, per / 2, 1, true, kAvail - stg);
  const uint32_t w2 = (uint32_t)(BM * BK * 2 * kc2);
  const uint32_t sb2 = w2 + (uint32_t)(per / 2 * BK * 2 * kc2);
  const int st2 = (int)std::min<size_t>(kMaxStages, (kAvail - stg) / sb2);
  if (st2 < 2) return;
  p.pair = true;
  p.kc = kc2;
  p.w_bytes = w2;
  p.stage_bytes = sb2;
  p.stages = st2;
  p.stg_bytes = (int)stg;
  const long long tiles = (long long)((p.feat_tiles + 1) / 2) * p.token_tiles;
  const long long pairs = cluster_capacity()[2] / 2 > 0 ? cluster_capacity()[2] / 2 : 1;
  const long long rounds = (tiles + pairs - 1) / pairs;
  p.grid_x = (int)(2 * ((tiles + rounds - 1) / rounds));  // CTAs: two per pair
}

Plan make_plan_uncached(int m, int n, int k, int row_bytes) {
  Plan p{};
  p.feat_tiles = (n + BM - 1) / BM;
  p.k_blocks = (k + BK - 1) / BK;
  p.tma3d = k % BK == 0;
  p.splits = choose_splits(p.feat_tiles, p.k_blocks, p.tma3d);
  if (const int fs = g_force_s.load()) p.splits = std::min(fs, std::max(1, p.k_blocks / 2));
  TileConfig c = best_config(m, p.feat_tiles, p.k_blocks, p.splits, p.tma3d, row_bytes, false);
  // Split-K stages carry several k-chunks too (the split factor itself is chosen
  // with one-chunk stages): fewer, larger TMA boxes measured 15 % faster for the
  // split-K down projections. A stage's last box may run past the split's range;
  // only its own chunks are multiplied.
  if (p.splits > 1 && !c.pair && p.tma3d) c.kc = chunks_for(c.mh, c.ng * c.n_g, 1, true, kAvail);
  // A forced shape applies where it is valid for this GEMM; it never touches the
  // split factor, so results are the same bits either way.
  const int ft = g_force_t.load(), fmh = g_force_mh.load(), fkc = g_force_kc.load();
  if (ft > 0) {
    TileConfig f = token_tiling(m, ft < (m + 15) / 16 ? ft : (m + 15) / 16);
    f.mh = c.mh;
    f.kc = c.kc;
    f.persist = c.persist;
    f.pair = c.pair;
    if (f.ng == 2 || (long long)f.ng * f.n_g > 256) f.mh = 1;
    c = f;
  }
  if (fmh == 1) c.mh = 1;
  if (fmh == 2 && p.splits == 1 && c.ng == 1 && c.n_g <= 256 && p.feat_tiles >= 2) c.mh = 2;
  if (fkc > 0 && (fkc == 1 || p.tma3d)) c.kc = fkc;
  // ... and is shrunk until two pipeline stages fit in shared memory.
  // A forced shape with no more tiles than resident CTAs runs one tile per CTA;
  // a pair launch stays a pair launch where its tiling allows.
  if (c.pair && !pair_ok(c, p.splits, p.feat_tiles)) c.pair = false;
  auto tiles_of = [&](const TileConfig& t) {
    return t.pair ? (long long)((p.feat_tiles + 1) / 2) * t.token_tiles
                  : (long long)((p.feat_tiles + t.mh - 1) / t.mh) * t.token_tiles;
  };
  auto persist_of = [&](const TileConfig& t) {
    return t.pair || (t.persist && p.splits == 1 && tiles_of(t) > cluster_capacity()[1]);
  };
  auto avail_of = [&](const TileConfig& t) { return kAvail - (persist_of(t) ? persist_staging(row_bytes) : 0); };
  auto fits = [&](const TileConfig& t) {
    const int x_rows = t.pair ? t.ng * t.n_g / 2 : t.ng * t.n_g;
    return (size_t)(t.mh * BM + x_rows) * BK * 2 * t.kc * 2 <= avail_of(t);
  };
  while (!fits(c) && c.kc > 1) c.kc /= 2;
  if (!fits(c)) {
    c.mh = 1;
    while (!fits(c) && c.kc > 1) c.kc /= 2;
  }
  p.bmt = BM;
  p.token_tiles = c.token_tiles;
  p.ng = c.ng;
  p.n_g = c.n_g;
  p.mh = c.mh;
  p.kc = c.kc;
  p.mt = p.ng * p.n_g;
  p.pair = c.pair;
  p.w_bytes = (uint32_t)(p.mh * BM * BK * 2 * p.kc);
  p.stage_bytes = (uint32_t)(p.w_bytes + (p.pair ? p.mt / 2 : p.mt) * BK * 2 * p.kc);
  const long long tiles = tiles_of(c);
  const bool persist = persist_of(c);
  size_t avail = avail_of(c);
  p.stg_bytes = persist ? (int)persist_staging(row_bytes) : 0;
  p.acc_bufs = persist && 2 * p.mh * p.mt <= 512 ? 2 : 1;
  if (p.pair) {
    const long long pairs = cluster_capacity()[2] / 2 > 0 ? cluster_capacity()[2] / 2 : 1;
    const long long rounds = (tiles + pairs - 1) / pairs;
    p.grid_x = (int)(2 * ((tiles + rounds - 1) / rounds));  // CTAs: two per pair
  } else if (persist) {
    const long long cap = cluster_capacity()[1];
    const long long rounds = (tiles + cap - 1) / cap;
    p.grid_x = (int)((tiles + rounds - 1) / rounds);  // balanced: every CTA walks rounds or rounds - 1 tiles
  } else {
    p.grid_x = (int)tiles;
  }
  p.stages = (int)(avail / p.stage_bytes);
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  p.rch = p.mt;
  p.stg_off = 0;
  if (p.splits > 1) {
    // Largest round whose exchange buffers (outgoing [rch][128] + incoming
    // [S][ceil(rch/S)][128] fp32) fit in the drained stage area next to the staging.
    const size_t area = (size_t)p.stages * p.stage_bytes;
    p.rch = 0;
    for (int ch = p.mt; ch >= 16; ch -= 16) {
      size_t slm = (ch + p.splits - 1) / p.splits;
      size_t xbuf = ((size_t)ch + (size_t)p.splits * slm) * BM * 4;
      size_t off = (xbuf + 1023) / 1024 * 1024;
      if (off + kStageBytes <= area) {
        p.rch = ch;
        p.stg_off = (int)off;
        break;
      }
    }
  }
  try_local_split(p, m, row_bytes);
  return p;
}

// Plans are cached per (m, n, k): a forward pass asks for the same few shapes on
// every layer.
std::mutex g_plan_mu;
std::unordered_map<uint64_t, Plan> g_plan_cache;

Plan make_plan(int m, int n, int k, int row_bytes) {
  std::mutex& mu = g_plan_mu;
  std::unordered_map<uint64_t, Plan>& cache = g_plan_cache;
  const bool key_ok = m < (1 << 18) && n < (1 << 24) && k < (1 << 20) && row_bytes >= 128 && row_bytes <= 512;
  const uint64_t rb_code = row_bytes == 128 ? 1 : row_bytes == 256 ? 2 : 3;  // 128 / 256 / 512
  const uint64_t key = (rb_code << 62) | ((uint64_t)m << 44) | ((uint64_t)n << 20) | (uint64_t)k;
  if (key_ok) {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  Plan p = make_plan_uncached(m, n, k, row_bytes);
  if (key_ok) {
    std::lock_guard<std::mutex> g(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, p);
  }
  return p;
}

// 64-row tiles through kve_gemm_force_rows: 0 = the rule below, 128 = never, 64 = where valid.
std::atomic<int> g_force_rows{0};

// A one-tile, single-group plan whose 128-row weight slab per CTA (plus its
// tokens) overflows the stage ring, while a 64-row slab fits whole, in one wave
// of CTAs: with 64-row tiles every weight byte of a CTA can be requested before
// the dependency wait (the draft's K = 896 projections at decode batches).
// Results are the same bits: each output is the same K-ordered MMA chain.
void try_rows64(Plan& p, int m, int n, int k, int mode, int out_dtype, int hd) {
  const int force = g_force_rows.load();
  if (force == 128) return;
  if (p.splits != 1 || p.pair || p.stg_bytes || p.mh != 1 || p.ng != 1 || !p.tma3d || out_dtype != KVE_BF16) return;
  if (mode == kEpiQkvRope && (hd <= 0 || 64 % hd)) return;
  const size_t x_row = (size_t)p.mt * BK * 2;  // token bytes per k-chunk
  int kc = 0, stages = 0;
  for (int c = 4; c >= 1; c /= 2) {
    const size_t bytes = (64 * (size_t)BK * 2 + x_row) * c;
    const int st = (int)std::min<size_t>(kMaxStages, kAvail / bytes);
    if (st >= 2) {
      kc = c;
      stages = st;
      break;
    }
  }
  if (!kc) return;
  const bool whole64 = (long long)stages * kc >= p.k_blocks;
  const bool over128 = ((size_t)BM * BK * 2 + x_row) * (size_t)p.k_blocks > kAvail;
  const long long ctas = (long long)((n + 63) / 64) * p.token_tiles;
  if (force != 64 && !(whole64 && over128 && ctas <= cluster_capacity()[1])) return;
  p.bmt = 64;
  p.kc = kc;
  p.stages = stages;
  p.w_bytes = (uint32_t)(64 * BK * 2 * kc);
  p.stage_bytes = (uint32_t)(p.w_bytes + x_row * kc);
  p.grid_x = (int)ctas;
  (void)m;
}

}  // namespace

size_t gemm_tc_workspace_bytes(int, int, int) { return 0; }

int gemm_tc(const void* x, const void* w, int m, int n, int k, const EpiArgs& e, void*, size_t, int* status,
            cudaStream_t stream) {
  if (k % 8) return set_error(KVE_ERR_SHAPE, "kve_gemm(tcgen05): k=%d must be a multiple of 8", k);
  if ((uintptr_t)x % 16 || (uintptr_t)w % 16)
    return set_error(KVE_ERR_ARG, "kve_gemm(tcgen05): x and w must be 16-byte aligned");
  if (e.mode == KVE_EPI_SILU_MUL && (n % 2))
    return set_error(KVE_ERR_SHAPE, "kve_gemm: SILU_MUL needs an even n");
  configure_kernel();
  // Bytes of one staged output row: 128 outputs (64 for SwiGLU) of the output type.
  const int row_bytes = (e.mode == KVE_EPI_SILU_MUL ? BM / 2 : BM) * (e.out_dtype == KVE_BF16 ? 2 : 4);
  Plan p = make_plan(m, n, k, row_bytes);
  try_rows64(p, m, n, k, e.mode, e.out_dtype, e.hd);
  if (p.stages < 2 || (p.splits > 1 && !p.lsplit && p.rch == 0))
    return set_error(KVE_ERR_SHAPE, "kve_gemm(tcgen05): tile does not fit shared memory");
  TcArgs a{};
  a.m = m; a.n = n; a.k = k; a.mt = p.mt; a.ng = p.ng; a.n_g = p.n_g; a.k_blocks = p.k_blocks;
  a.splits = p.splits; a.stages = p.stages; a.stage_bytes = p.stage_bytes; a.e = e; a.status = status;
  a.rch = p.rch; a.stg_off = p.stg_off;
  a.w_static = e.w_static;
  a.kc = p.kc; a.tma3d = p.tma3d; a.w_bytes = p.w_bytes;
  a.token_tiles = p.token_tiles;
  a.feat_ctas = p.bmt == 64 ? (n + 63) / 64 : p.pair ? (p.feat_tiles + 1) / 2 : (p.feat_tiles + p.mh - 1) / p.mh;
  a.acc_bufs = p.acc_bufs; a.stg_bytes = p.stg_bytes;
  a.lsplit = p.lsplit ? 1 : 0;
  const int es = e.out_dtype == KVE_BF16 ? 2 : 4;
  a.out_vec_ok = ((uintptr_t)e.out % 16 == 0) && ((size_t)e.ld_out * es % 16 == 0) &&
                 (e.mode != KVE_EPI_RESIDUAL || (uintptr_t)e.residual % 16 == 0);
  const bool persist = p.stg_bytes > 0;
  GemmKernel kern = p.bmt == 64 ? rows64_kernel_for(e.mode, e.out_dtype)
                  : p.lsplit ? (p.pair ? lsplit_pair_kernel_for(e.mode, e.out_dtype) : lsplit_kernel_for(e.mode, e.out_dtype))
                  : p.pair ? pair_kernel_for(e.mode, e.out_dtype, p.ng) : kernel_for(e.mode, e.out_dtype, p.ng, p.mh, persist);
  if (!kern) return set_error(KVE_ERR_DTYPE, "kve_gemm(tcgen05): epilogue %d needs bf16 output", e.mode);
  CUtensorMap mw, mx;
  int rc = p.tma3d ? make_map3(&mw, w, n, k, p.bmt * p.mh, p.kc) : make_map(&mw, w, n, k, p.bmt * p.mh);
  if (rc) return rc;
  const int x_box = p.pair ? p.n_g / 2 : p.n_g;  // a pair CTA stages half of each token group
  rc = p.tma3d ? make_map3(&mx, x, m, k, x_box, p.kc) : make_map(&mx, x, m, k, x_box);
  if (rc) return rc;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = p.pair ? 2 : 1;  // a CTA pair, or the split-K CTAs of one tile
  attr.val.clusterDim.y = 1;
  const int cl_splits = p.lsplit ? 1 : p.splits;  // CTAs of a cluster splitting K
  attr.val.clusterDim.z = cl_splits;
  const dim3 grid = persist     ? dim3(p.grid_x, 1, 1)
                    : p.lsplit ? dim3(a.feat_ctas, p.token_tiles, 1)  // feature tiles fastest
                               : dim3(p.token_tiles, a.feat_ctas, cl_splits);
  cudaError_t err = launch_kernel_ex(kern, grid, dim3(kThreads),
                                     (size_t)p.stages * p.stage_bytes + p.stg_bytes + 1024 + 512, stream, &attr,
                                     (cl_splits > 1 || p.pair) ? 1 : 0, mw, mx, a);
  if (err != cudaSuccess) {
    cudaGetLastError();
    count_launch();
    return set_error(KVE_ERR_CUDA, "kve_gemm(tcgen05): launch failed: %s", cudaGetErrorString(err));
  }
  return check_launch("kve_gemm(tcgen05)");
}

int gemm_qkv_rope(const void* x, const void* w, int m, int n, int k, const EpiArgs& e_in, cudaStream_t stream) {
  EpiArgs e = e_in;
  e.mode = kEpiQkvRope;
  e.out_dtype = KVE_BF16;
  e.out = e.q_out;
  e.ld_out = n;
  if (e.hd < 8 || e.hd % 8 || 128 % e.hd || n != (e.nq + 2 * e.nkv) * e.hd || !e.bias || !e.positions ||
      !e.slots || !e.rope_cos || !e.rope_sin || !e.q_out || !e.pool_k || !e.pool_v)
    return set_error(KVE_ERR_ARG, "gemm_qkv_rope: bad head layout or null pointer");
  const void* ptrs[5] = {e.q_out, e.pool_k, e.pool_v, e.rope_cos, e.rope_sin};
  for (const void* q : ptrs)
    if ((uintptr_t)q % 16) return set_error(KVE_ERR_ARG, "gemm_qkv_rope: pointers must be 16-byte aligned");
  return gemm_tc(x, w, m, n, k, e, nullptr, 0, e.status, stream);
}

}  // namespace kve

extern "C" int kve_gemm_force_shape(int token_tiles, int weight_halves, int k_chunks) {
  using namespace kve;
  if (token_tiles < 0 || weight_halves < 0 || weight_halves > 2 ||
      !(k_chunks == 0 || k_chunks == 1 || k_chunks == 2 || k_chunks == 4))
    return set_error(KVE_ERR_ARG, "kve_gemm_force_shape: token_tiles >= 0, weight_halves in 0..2, k_chunks in 0,1,2,4");
  std::lock_guard<std::mutex> g(g_plan_mu);
  g_force_t.store(token_tiles);
  g_force_mh.store(weight_halves);
  g_force_kc.store(k_chunks);
  g_plan_cache.clear();
  return KVE_OK;
}

extern "C" int kve_gemm_force_splits(int splits) {
  using namespace kve;
  if (splits < 0 || splits > kMaxSplits)
    return set_error(KVE_ERR_ARG, "kve_gemm_force_splits: 0 (model) or 1..%d", kMaxSplits);
  std::lock_guard<std::mutex> g(g_plan_mu);
  g_force_s.store(splits);
  g_plan_cache.clear();
  return KVE_OK;
}

extern "C" int kve_gemm_force_local_split(int mode) {
  using namespace kve;
  if (mode < 0 || mode > 2)
    return set_error(KVE_ERR_ARG, "kve_gemm_force_local_split: mode 0 (rule), 1 (never) or 2 (where valid)");
  std::lock_guard<std::mutex> g(g_plan_mu);
  g_force_local.store(mode);
  g_plan_cache.clear();
  return KVE_OK;
}

extern "C" int kve_gemm_force_rows(int rows) {
  using namespace kve;
  if (!(rows == 0 || rows == 64 || rows == 128))
    return set_error(KVE_ERR_ARG, "kve_gemm_force_rows: rows 0 (rule), 64 (where valid) or 128 (never 64)");
  g_force_rows.store(rows);
  return KVE_OK;
}

extern "C" int kve_gemm_force_pair(int mode) {
  using namespace kve;
  if (mode < 0 || mode > 2) return set_error(KVE_ERR_ARG, "kve_gemm_force_pair: mode 0 (model), 1 (never) or 2 (where valid)");
  std::lock_guard<std::mutex> g(g_plan_mu);
  g_force_pair.store(mode);
  g_plan_cache.clear();
  return KVE_OK;
}

extern "C" int kve_gemm_plan_info(int m, int n, int k, int* out) {
  using namespace kve;
  if (m < 1 || n < 1 || k < 1 || !out) return set_error(KVE_ERR_ARG, "kve_gemm_plan_info: bad arguments");
  Plan p = make_plan(m, n, k, BM * 2);
  try_rows64(p, m, n, k, KVE_EPI_STORE, KVE_BF16, 0);
  const int feat_ctas = p.bmt == 64 ? (n + 63) / 64 : p.pair ? (p.feat_tiles + 1) / 2 : (p.feat_tiles + p.mh - 1) / p.mh;
  const int v[13] = {p.splits, p.token_tiles, p.ng, p.n_g, p.mh, p.kc, p.stages, p.tma3d, feat_ctas,
                     p.splits > 1 && !p.lsplit ? p.token_tiles * feat_ctas * p.splits : p.grid_x, p.acc_bufs,
                     p.pair ? 1 : 0,
                     p.bmt};
  for (int i = 0; i < 13; ++i) out[i] = v[i];
  return KVE_OK;
}
