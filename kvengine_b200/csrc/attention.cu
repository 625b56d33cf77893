// Paged multi-query GQA verify attention.
//
// CTA = (context chunk, sequence x kv-head, query tile). All query rows of one
// kv-head group (q tokens x group heads, <= 64 rows) share every K/V tile the
// CTA stages through shared memory, so each K/V byte is read from HBM once per
// query tile. Keys are visited in absolute 32-key tiles; chunks of kChunk keys
// run in parallel and are merged in chunk order (bf16: by the last chunk CTA
// to finish, in the same launch; fp32: by a second kernel). A
// query's result therefore depends only on its own position and keys: the
// draft's 1-row pass and the target's k+1-row pass agree bit for bit.
//
// Softmax is online in fp32 (scores, running max and sum, and the P.V
// accumulator all fp32), masked keys contribute exact zeros.
#include <math.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "kve_common.cuh"
#include "passes.cuh"
#include "tma.cuh"

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
  int* counters;  // split mode (bf16): finished-chunk count per (sequence x kv-head, query tile), left at zero
  int n_chunks, n_qtiles;
  int rb;  // bf16 kernel: row blocks (16 query rows each) per CTA
  int* status;
  // Keys before ctx - q_len of every sequence, the block tables and the
  // length arrays are written by no kernel that may still be running (true in
  // kve_forward: the pass's only K/V writer appends the new tokens): their loads
  // may start before the dependency wait.
  int hist_static;
};

__host__ __device__ inline size_t partial_floats(int hd) { return (size_t)kMaxRows * (hd + 2); }

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnThreads)
paged_attn_kernel(AttnParams p) {
  grid_dep_wait();
  grid_dep_launch();
  constexpr int DPL = HD / 32;  // output dims per lane
  constexpr int VEC = 16 / sizeof(T);
  constexpr int VPR = HD / VEC;  // 16-byte vectors per key row
  extern __shared__ float smem[];
  float* qs = smem;                          // [kMaxRows][HD]
  float* ks = qs + kMaxRows * HD;            // [kKeyTile][HD + 1]
  float* vs = ks + kKeyTile * (HD + 1);      // [kKeyTile][HD]

  const int bh = blockIdx.x, c = blockIdx.y, qtile = blockIdx.z;
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

// ---------------------------------------------------------------------------
// bf16 tensor-core variant (mma.sync m16n8k16, fp32 accumulate). Same CTA
// decomposition, key tiles, chunking and partial format as the kernel above;
// each of the 4 warps owns 16 query rows. K/V tiles of 32 keys are staged with
// 16-byte cp.async (double-buffered, rows padded by 16 bytes so ldmatrix is
// conflict-free); S = Q K^T and O += P V run on the tensor cores, the online
// softmax in registers. Every row's arithmetic depends only on that row and on
// keys at fixed absolute positions, so results do not depend on the batch.
constexpr int kMmaKeyTile = 32;
// Key tile t of a chunk (32 keys at key_lo + 32 t) belongs to key slice
// t % SL (SL = key_slices(head_dim)). The slices of a row block (16 query rows) run in separate warps
// at the same time and their softmax states merge in slice order at the end, so
// a row's arithmetic is the same whatever the number of row blocks in its CTA.
// Slices per row block: 8 for head_dim 64 (a round then covers 256 keys, so a
// decode context of a few hundred keys takes one round), 4 for head_dim 128 (its
// accumulators take twice the registers). A model has one head_dim, so all of
// its passes slice alike. Row blocks per CTA are capped so the CTA stays at 16
// warps.
constexpr int key_slices(int hd) { return hd == 64 ? 8 : 4; }
constexpr int max_row_blocks(int hd) { return hd == 64 ? 2 : 4; }
constexpr int kRoundBufs = 2;  // rounds (one tile per slice each) staged in shared memory

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// 2^x on the special-function unit (ex2.approx: relative error about 2^-22;
// 2^-inf = +0). The bf16 kernel keeps its softmax in log2 units: scores are
// scaled by scale * log2(e), so 2^(s - m) equals e^(scale * (q.k) - m').
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Merge chunk partials in chunk order for the rows of one (sequence x kv-head,
// query tile). A row at position pos reads chunks 0 .. pos / kChunk; with a
// single chunk this reproduces acc / l exactly. Partials are read through L2
// (another CTA of the same launch may have written them).
// LOG2: the partials' running maxima are in log2 units (the bf16 kernel scores
// with scale * log2(e) and exponentiates with 2^x); otherwise natural units.
template <typename T, int HD, int WARPS, bool LOG2>
__device__ __forceinline__ void merge_partials(const AttnParams& p, int bh, int qtile, int h, int rows,
                                               int first_pos, int qoff, int t0) {
  constexpr int DPL = HD / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* base = p.ws + (((size_t)bh * p.n_qtiles + qtile) * p.n_chunks) * partial_floats(HD);
  T* out = static_cast<T*>(p.out);
  for (int r = warp; r < rows; r += WARPS) {
    const int pos = first_pos + r / p.group;
    const int live = pos / kChunk + 1;
    float mx = -INFINITY;
    for (int c = 0; c < live; ++c) mx = fmaxf(mx, __ldcg(base + c * partial_floats(HD) + (size_t)r * (HD + 2) + HD));
    float lsum = 0.f, acc[DPL];
#pragma unroll
    for (int dd = 0; dd < DPL; ++dd) acc[dd] = 0.f;
    for (int c = 0; c < live; ++c) {
      const float* pr = base + c * partial_floats(HD) + (size_t)r * (HD + 2);
      float w = LOG2 ? ex2f(__ldcg(pr + HD) - mx) : expf(__ldcg(pr + HD) - mx);
      lsum += __ldcg(pr + HD + 1) * w;
#pragma unroll
      for (int dd = 0; dd < DPL; ++dd) acc[dd] += __ldcg(pr + lane + dd * 32) * w;
    }
    int t = r / p.group, g = r % p.group;
    T* o = out + ((size_t)(qoff + t0 + t) * p.nq + h * p.group + g) * HD;
#pragma unroll
    for (int dd = 0; dd < DPL; ++dd) o[lane + dd * 32] = Elem<T>::from_f(acc[dd] / lsum);
  }
}

// TMA: block size 16 only. One thread brings each round's K and V with 2 KB
// boxes (16 keys x 64 dims, SWIZZLE_128B) straight from the pool; keys past the
// chunk load from outside the tensor (zero fill) and the tail of the last
// partial block is zeroed in shared memory. Otherwise 16-byte cp.async per thread.
template <int HD, int BS, int RB, bool TMA>
__global__ void __launch_bounds__(RB * key_slices(HD) * 32, 1)
paged_attn_mma_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v,
                      AttnParams p) {
  // With hist_static the wait moves down to the first load of a key written in
  // this pass (or of q); everything before it reads constant inputs only.
  bool waited = !p.hist_static;
  if (waited) grid_dep_wait();
  grid_dep_launch();
  constexpr int SL = key_slices(HD);
  constexpr int NTHR = RB * SL * 32;
  constexpr int ROW = HD * 2 + 16;                  // padded smem row (bytes, cp.async layout)
  constexpr int TILE = TMA ? kMmaKeyTile * HD * 2 : kMmaKeyTile * ROW;  // one K or V tile
  constexpr int ROUND = SL * 2 * TILE;      // K and V of one round (SL tiles)
  constexpr int KSTEPS = HD / 16;                   // k16 steps over the head dim
  constexpr int NT = kMmaKeyTile / 8;               // n8 tiles of keys per tile
  constexpr int DT = HD / 8;                        // n8 tiles of the output
  constexpr int CPR = HD * 2 / 16;                  // 16-byte chunks per key row
  constexpr int TCH = 2 * kMmaKeyTile * CPR;        // 16-byte chunks of one tile (K and V)
  constexpr int TOTAL = SL * TCH;           // 16-byte chunks of one round
  constexpr int SLOTS = (TOTAL + NTHR - 1) / NTHR;  // chunks per thread per round
  extern __shared__ __align__(128) uint8_t smem_dyn[];
  // The 128-byte swizzle repeats every 1024 bytes: TMA tiles start 1024-aligned.
  uint8_t* smem_attn = TMA ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023))
                           : smem_dyn;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem_attn));
  // buffers: [round buffer][slice][K|V] tiles (after the main loop: the slice merge
  // area), then the chunk's block table, then (TMA) the round barriers
  constexpr int XS = HD + 8;  // merge rows (floats), padded so the 8 rows g of a warp hit different banks
  constexpr int MERGE = SL * RB * 16 * (XS + 2) * 4 + RB * 16 * (SL + 2) * 4;
  constexpr int AREA = kRoundBufs * ROUND > MERGE ? kRoundBufs * ROUND : MERGE;
  uint64_t* round_full = reinterpret_cast<uint64_t*>(smem_attn + AREA + kChunk * sizeof(int));
  if constexpr (TMA) {
    if (threadIdx.x == 0) {
      for (int b = 0; b < kRoundBufs; ++b) mbar_init(smem_u32(&round_full[b]), 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
  }

  const int bh = blockIdx.x, c = blockIdx.y, qtile = blockIdx.z;
  const int b = bh / p.nkv, h = bh % p.nkv;
  const int ctx = p.ctx_lens[b], ql = p.q_lens[b], qoff = p.q_offsets[b];
  // Every CTA passes the dependency wait before it exits, so this grid never
  // completes ahead of the kernels before it.
  if (ql < 0 || ctx < ql || ctx > p.table_stride * p.bs) {
    if (!waited) grid_dep_wait();
    if (threadIdx.x == 0 && c == 0 && qtile == 0) report(p.status, KVE_ERR_BOUNDS);
    return;
  }
  const int t0 = qtile * p.qt;
  const int nt = min(p.qt, ql - t0);
  const int rows = nt * p.group;
  const int first_pos = ctx - ql + t0;
  const int last_pos = first_pos + nt - 1;
  const int key_lo = c * kChunk;
  if (t0 >= ql || key_lo > last_pos) {
    if (!waited) grid_dep_wait();
    return;
  }
  const int key_hi = min(min(ctx, key_lo + kChunk), last_pos + 1);
  const int n_tiles = (key_hi - key_lo + kMmaKeyTile - 1) / kMmaKeyTile;
  const int n_rounds = (n_tiles + SL - 1) / SL;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = warp % RB, ks = warp / RB;  // row block, key slice
  const int g = lane >> 2, tq = lane & 3;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q);
  const __nv_bfloat16* pk = static_cast<const __nv_bfloat16*>(p.pool_k);
  const __nv_bfloat16* pv = static_cast<const __nv_bfloat16*>(p.pool_v);
  const int32_t* table = p.tables + (size_t)b * p.table_stride;

  // The chunk's block-table entries, staged once (kChunk keys / block size).
  int* tab = reinterpret_cast<int*>(smem_attn + AREA);
  const int blk_lo = BS > 0 ? key_lo / BS : key_lo / p.bs;
  const int n_blk = (BS > 0 ? (key_hi - 1) / BS : (key_hi - 1) / p.bs) - blk_lo + 1;
  for (int i = threadIdx.x; i < n_blk; i += NTHR) {
    int64_t blk = table[blk_lo + i];
    if (blk < 0 || blk >= p.num_blocks) {
      report(p.status, KVE_ERR_BOUNDS);
      blk = -1;
    }
    tab[i] = (int)blk;
  }
  __syncthreads();

  // Round r holds tiles r*SL .. +SL-1 (tile s of the round at
  // slot s); every thread copies the same slots of every round.
  const size_t head_off = (size_t)h * HD;
  const size_t row_stride = (size_t)p.nkv * HD;  // elements between consecutive tokens
  auto load_round = [&](int r) {
    const uint32_t rbase = sbase + (uint32_t)((r % kRoundBufs) * ROUND);
#pragma unroll
    for (int u = 0; u < SLOTS; ++u) {
      const int i = threadIdx.x + u * NTHR;
      if (TOTAL % NTHR != 0 && i >= TOTAL) break;
      const int s = i / TCH, rem = i % TCH;
      const bool is_v = rem >= kMmaKeyTile * CPR;
      const int j = is_v ? rem - kMmaKeyTile * CPR : rem;
      const int kk = j / CPR, ch = j % CPR;
      const int tile = r * SL + s;
      const int key = key_lo + tile * kMmaKeyTile + kk;
      const __nv_bfloat16* src = pk;
      uint32_t bytes = 0;
      if (tile < n_tiles && key < key_hi) {
        int blk, off;
        if constexpr (BS > 0) {
          blk = tab[key / BS - blk_lo];
          off = key % BS;
        } else {
          blk = tab[key / p.bs - blk_lo];
          off = key % p.bs;
        }
        if (blk >= 0) {
          const int bsz = BS > 0 ? BS : p.bs;
          src = (is_v ? pv : pk) + ((size_t)blk * bsz + off) * row_stride + head_off + ch * 8;
          bytes = 16;
        }
      }
      cp_async16(rbase + (uint32_t)(s * 2 * TILE + (is_v ? TILE : 0) + kk * ROW + ch * 16), src, bytes);
    }
  };

  // TMA: thread 0 asks for the 16-key blocks of round r's tiles in slots [s0, s1);
  // with `arm` it first arms the round's barrier for every tile of the round, so a
  // round may be requested in two parts (history tiles before the dependency wait).
  const int oob_row = (int)(p.num_blocks * 16);  // first row past the pool: loads there fill zeros
  auto tma_tiles = [&](int r, int s0, int s1, bool arm) {
    if constexpr (TMA) {
      if (threadIdx.x != 0) return;
      const uint32_t fb = smem_u32(&round_full[r % kRoundBufs]);
      const uint32_t rbase = sbase + (uint32_t)((r % kRoundBufs) * ROUND);
      if (arm) {
        int tiles = 0;
        for (int s = 0; s < SL; ++s) tiles += r * SL + s < n_tiles;
        mbar_expect_tx(fb, (uint32_t)(tiles * 2 * TILE));  // K and V of every tile of the round
      }
      for (int s = s0; s < s1; ++s) {
        const int tile = r * SL + s;
        if (tile >= n_tiles) break;
#pragma unroll
        for (int jb = 0; jb < 2; ++jb) {
          const int key0 = key_lo + tile * kMmaKeyTile + jb * 16;
          int y = oob_row;
          if (key0 < key_hi) {
            const int blk = tab[key0 / 16 - blk_lo];
            if (blk >= 0) y = blk * 16;
          }
#pragma unroll
          for (int half = 0; half < HD / 64; ++half) {
            const uint32_t off = (uint32_t)(s * 2 * TILE + half * 4096 + jb * 2048);
            tma_load_2d(rbase + off, &map_k, h * HD + half * 64, y, fb);
            tma_load_2d(rbase + off + TILE, &map_v, h * HD + half * 64, y, fb);
          }
        }
      }
    }
  };
  auto tma_round = [&](int r) { tma_tiles(r, 0, SL, true); };

  // Prologue: kRoundBufs rounds in flight. Keys written before this pass (history)
  // may load before the dependency wait: TMA requests every history tile of those
  // rounds first and the rest after the wait; cp.async (one commit group per round,
  // empty groups past the end) goes by whole rounds.
  const int hist_end = ctx - ql;  // keys below this were written before this pass
  if constexpr (TMA) {
    int issued[kRoundBufs];
#pragma unroll
    for (int r = 0; r < kRoundBufs; ++r) {
      issued[r] = 0;
      if (r >= n_rounds) continue;
      int s1 = SL;
      if (!waited) {  // slots whose 32 keys all lie below hist_end
        const int hist_tiles = hist_end > key_lo ? (hist_end - key_lo) / kMmaKeyTile : 0;
        s1 = min(max(hist_tiles - r * SL, 0), SL);
      }
      tma_tiles(r, 0, s1, true);
      issued[r] = s1;
    }
    if (!waited) {
      grid_dep_wait();
      waited = true;
    }
#pragma unroll
    for (int r = 0; r < kRoundBufs; ++r)
      if (r < n_rounds && issued[r] < SL) tma_tiles(r, issued[r], SL, false);
  } else {
#pragma unroll
    for (int r = 0; r < kRoundBufs; ++r) {
      if (r < n_rounds) {
        if (!waited && key_lo + (r + 1) * SL * kMmaKeyTile > hist_end) {
          grid_dep_wait();
          waited = true;
        }
        load_round(r);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  if (!waited) grid_dep_wait();  // before q and the remaining rounds

  // Q fragments for this warp's 16 rows (rows >= `rows` are zero).
  const int r_lo = rb * 16 + g, r_hi = r_lo + 8;
  const bool active = rb * 16 < rows;
  uint32_t qa[KSTEPS][4];
  {
    const __nv_bfloat16* q_lo = nullptr;
    const __nv_bfloat16* q_hi = nullptr;
    if (r_lo < rows) q_lo = q + ((size_t)(qoff + t0 + r_lo / p.group) * p.nq + h * p.group + r_lo % p.group) * HD;
    if (r_hi < rows) q_hi = q + ((size_t)(qoff + t0 + r_hi / p.group) * p.nq + h * p.group + r_hi % p.group) * HD;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int d0 = kk * 16 + 2 * tq;
      qa[kk][0] = q_lo ? *reinterpret_cast<const uint32_t*>(q_lo + d0) : 0u;
      qa[kk][1] = q_hi ? *reinterpret_cast<const uint32_t*>(q_hi + d0) : 0u;
      qa[kk][2] = q_lo ? *reinterpret_cast<const uint32_t*>(q_lo + d0 + 8) : 0u;
      qa[kk][3] = q_hi ? *reinterpret_cast<const uint32_t*>(q_hi + d0 + 8) : 0u;
    }
  }
  const int pos_lo = first_pos + (r_lo < rows ? r_lo / p.group : 0);
  const int pos_hi = first_pos + (r_hi < rows ? r_hi / p.group : 0);

  const float sl2 = p.scale * kLog2e;  // scores in log2 units
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  float acc[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;

  // Shared-memory address of (key row, dim) in a K or V tile; dim is a multiple of 8.
  auto tile_addr = [&](uint32_t base, int key_row, int dim) -> uint32_t {
    if constexpr (TMA)
      return base + (uint32_t)((dim >> 6) * 4096 + key_row * 128 + ((((dim & 63) >> 3) ^ (key_row & 7)) << 4));
    else
      return base + (uint32_t)(key_row * ROW + dim * 2);
  };
  bool failed = false;
  for (int r = 0; r < n_rounds; ++r) {
    if constexpr (TMA) {
      const bool ok = mbar_wait(smem_u32(&round_full[r % kRoundBufs]), (uint32_t)(r / kRoundBufs) & 1u, p.status);
      if (__syncthreads_or(!ok)) {
        // Let the other buffer's loads (if any were issued) land before leaving.
        for (int rr = r + 1; rr < n_rounds && rr < r + kRoundBufs; ++rr)
          mbar_wait(smem_u32(&round_full[rr % kRoundBufs]), (uint32_t)(rr / kRoundBufs) & 1u, p.status);
        failed = true;
        break;
      }
      // Zero the V rows of the last partial block past the chunk's keys (pool contents there are
      // not this sequence's keys; P is 0 for them but 0 * NaN would not be).
      const int t_last = (key_hi - 1 - key_lo) / kMmaKeyTile;
      if (t_last / SL == r) {
        const int first = key_hi - (key_lo + t_last * kMmaKeyTile);
        if (first < kMmaKeyTile) {
          uint8_t* vt = smem_attn + (r % kRoundBufs) * ROUND + (t_last % SL) * 2 * TILE + TILE;
          const int per_half = (kMmaKeyTile - first) * 8;  // 16-byte pieces of one 64-dim half
          for (int i = threadIdx.x; i < per_half * (HD / 64); i += NTHR) {
            const int half = i / per_half, rem = i % per_half;
            reinterpret_cast<uint4*>(vt + half * 4096 + (first + rem / 8) * 128)[rem % 8] = make_uint4(0, 0, 0, 0);
          }
        }
        __syncthreads();
      }
    } else {
      // Round r is the oldest outstanding group once kRoundBufs - 1 newer ones may remain.
      asm volatile("cp.async.wait_group %0;" ::"n"(kRoundBufs - 1) : "memory");
      __syncthreads();
    }
    const int tile = r * SL + ks;
    if (active && tile < n_tiles) {
      const uint32_t kbase = sbase + (uint32_t)((r % kRoundBufs) * ROUND + ks * 2 * TILE);
      const uint32_t vbase = kbase + TILE;
      const int kt = key_lo + tile * kMmaKeyTile;
      // S = Q K^T over this tile's 32 keys.
      float sc[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
        for (int j2 = 0; j2 < NT; j2 += 2) {
          // 4 matrices: keys [8*j2, 8*j2+8) dims k0..k0+7 / k0+8..k0+15, keys [8*j2+8, ...) same dims
          const int mat = lane >> 3, rr = lane & 7;
          const int key_row = 8 * j2 + ((mat >> 1) << 3) + rr;
          const int dim = kk * 16 + ((mat & 1) << 3);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(tile_addr(kbase, key_row, dim), b0, b1, b2, b3);
          mma_bf16_16816(sc[j2], qa[kk], b0, b1);
          mma_bf16_16816(sc[j2 + 1], qa[kk], b2, b3);
        }
      }
      // scale, causal mask, online softmax (rows g and g+8 of this warp)
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = kt + 8 * j + 2 * tq + e;
          const bool ok = key < key_hi;
          sc[j][e] = (ok && key <= pos_lo) ? sc[j][e] * sl2 : -INFINITY;
          sc[j][2 + e] = (ok && key <= pos_hi) ? sc[j][2 + e] * sl2 : -INFINITY;
          mx_lo = fmaxf(mx_lo, sc[j][e]);
          mx_hi = fmaxf(mx_hi, sc[j][2 + e]);
        }
      }
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      // Rows whose tile is fully masked keep their state exactly (factor 1, p = 0).
      const float f_lo = mx_lo == -INFINITY ? 1.f : ex2f(m_lo - mn_lo);
      const float f_hi = mx_hi == -INFINITY ? 1.f : ex2f(m_hi - mn_hi);
      float s_lo = 0.f, s_hi = 0.f;
      uint32_t pa[NT / 2][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const float p0 = sc[j][0] == -INFINITY ? 0.f : ex2f(sc[j][0] - mn_lo);
        const float p1 = sc[j][1] == -INFINITY ? 0.f : ex2f(sc[j][1] - mn_lo);
        const float p2 = sc[j][2] == -INFINITY ? 0.f : ex2f(sc[j][2] - mn_hi);
        const float p3 = sc[j][3] == -INFINITY ? 0.f : ex2f(sc[j][3] - mn_hi);
        s_lo += p0 + p1;
        s_hi += p2 + p3;
        pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16(p0, p1);
        pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
      }
      s_lo += __shfl_xor_sync(0xffffffffu, s_lo, 1);
      s_lo += __shfl_xor_sync(0xffffffffu, s_lo, 2);
      s_hi += __shfl_xor_sync(0xffffffffu, s_hi, 1);
      s_hi += __shfl_xor_sync(0xffffffffu, s_hi, 2);
      if (mx_lo != -INFINITY) { l_lo = l_lo * f_lo + s_lo; m_lo = mn_lo; }
      if (mx_hi != -INFINITY) { l_hi = l_hi * f_hi + s_hi; m_hi = mn_hi; }
#pragma unroll
      for (int j = 0; j < DT; ++j) {
        acc[j][0] *= f_lo; acc[j][1] *= f_lo;
        acc[j][2] *= f_hi; acc[j][3] *= f_hi;
      }
      // O += P V: P (16 x 32 keys) as two k16 A fragments, V via transposed ldmatrix.
#pragma unroll
      for (int s16 = 0; s16 < NT / 2; ++s16) {
        // A fragment order: (row g, keys 2t..), (row g+8, keys 2t..), (row g, keys 8+2t..), (row g+8, keys 8+2t..)
        const uint32_t a[4] = {pa[s16][0], pa[s16][1], pa[s16][2], pa[s16][3]};
#pragma unroll
        for (int j2 = 0; j2 < DT; j2 += 2) {
          const int mat = lane >> 3, rr = lane & 7;
          const int key_row = s16 * 16 + ((mat & 1) << 3) + rr;
          const int dim = 8 * j2 + ((mat >> 1) << 3);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(tile_addr(vbase, key_row, dim), b0, b1, b2, b3);
          mma_bf16_16816(acc[j2], a, b0, b1);
          mma_bf16_16816(acc[j2 + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();  // every slice is done with this round's buffer
    if constexpr (TMA) {
      if (threadIdx.x == 0 && r + kRoundBufs < n_rounds) {
        fence_proxy_async_smem();
        tma_round(r + kRoundBufs);
      }
    } else {
      if (r + kRoundBufs < n_rounds) load_round(r + kRoundBufs);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  if (failed) return;
  if constexpr (!TMA) asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  // Merge the key slices of each row block (the round buffers are free now). Every
  // slice publishes its unnormalised state (acc, m, l) per row; one thread per row
  // turns the slice maxima into weights w_s = 2^(m_s - M) (0 for a slice that saw
  // no key of the row) and the merged sum L = sum_s l_s w_s, in slice order; then
  // each slice's warp finishes a quarter of the head dims: sum_s acc_s w_s in slice
  // order, divided by L (or kept unnormalised as this chunk's partial).
  float* xs = reinterpret_cast<float*>(smem_attn);                  // [slice][rb][16 rows][XS]
  float* xml = xs + (size_t)SL * RB * 16 * XS;              // [slice][rb][16 rows][m, l]
  float* xw = xml + (size_t)SL * RB * 16 * 2;               // [rb][16 rows][w_0..w_S-1, M, L]
  constexpr int WS = SL + 2;
  if (active) {
    float* a = xs + (size_t)(ks * RB + rb) * 16 * XS;
#pragma unroll
    for (int j = 0; j < DT; ++j) {
      *reinterpret_cast<float2*>(a + g * XS + 8 * j + 2 * tq) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(a + (g + 8) * XS + 8 * j + 2 * tq) = make_float2(acc[j][2], acc[j][3]);
    }
    if (tq == 0) {
      float* ml = xml + (size_t)(ks * RB + rb) * 16 * 2;
      ml[g * 2] = m_lo;
      ml[g * 2 + 1] = l_lo;
      ml[(g + 8) * 2] = m_hi;
      ml[(g + 8) * 2 + 1] = l_hi;
    }
  }
  __syncthreads();
  if (active && ks == 0 && lane < 16) {
    float ms[SL];
    float mm = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < SL; ++s2) {
      ms[s2] = xml[(size_t)(s2 * RB + rb) * 32 + lane * 2];
      mm = fmaxf(mm, ms[s2]);
    }
    float lsum = 0.f;
    float* w = xw + (size_t)(rb * 16 + lane) * WS;
#pragma unroll
    for (int s2 = 0; s2 < SL; ++s2) {
      const float ws = ms[s2] == -INFINITY ? 0.f : ex2f(ms[s2] - mm);
      lsum += xml[(size_t)(s2 * RB + rb) * 32 + lane * 2 + 1] * ws;
      w[s2] = ws;
    }
    w[SL] = mm;
    w[SL + 1] = lsum;
  }
  __syncthreads();

  // This warp's quarter of the head dims: QP float pairs per row, 16 rows.
  constexpr int QP = HD / SL / 2;
  constexpr int ITEMS = 16 * QP / 32;  // (row, pair) items per lane
  const int d_base = ks * (HD / SL);
  if (p.ws == nullptr) {
    if (!active) return;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
      const int item = it * 32 + lane;
      const int r = item / QP, d = d_base + 2 * (item % QP);
      const int rr = rb * 16 + r;
      if (rr >= rows) continue;
      const float* w = xw + (size_t)(rb * 16 + r) * WS;
      float o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < SL; ++s2) {
        const float2 x = *reinterpret_cast<const float2*>(xs + (size_t)((s2 * RB + rb) * 16 + r) * XS + d);
        o0 += x.x * w[s2];
        o1 += x.y * w[s2];
      }
      const float l = w[SL + 1];
      __nv_bfloat16* o = out + ((size_t)(qoff + t0 + rr / p.group) * p.nq + h * p.group + rr % p.group) * HD + d;
      *reinterpret_cast<uint32_t*>(o) = pack_bf16(o0 / l, o1 / l);
    }
  } else {
    float* part = p.ws + ((((size_t)bh * p.n_qtiles + qtile) * p.n_chunks) + c) * partial_floats(HD);
    if (active) {
#pragma unroll
      for (int it = 0; it < ITEMS; ++it) {
        const int item = it * 32 + lane;
        const int r = item / QP, d = d_base + 2 * (item % QP);
        const int rr = rb * 16 + r;
        if (rr >= rows) continue;
        const float* w = xw + (size_t)(rb * 16 + r) * WS;
        float o0 = 0.f, o1 = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < SL; ++s2) {
          const float2 x = *reinterpret_cast<const float2*>(xs + (size_t)((s2 * RB + rb) * 16 + r) * XS + d);
          o0 += x.x * w[s2];
          o1 += x.y * w[s2];
        }
        float* pr = part + (size_t)rr * (HD + 2);
        *reinterpret_cast<float2*>(pr + d) = make_float2(o0, o1);
        if (ks == 0 && (item % QP) == 0) {
          pr[HD] = w[SL];
          pr[HD + 1] = w[SL + 1];
        }
      }
    }
    if (!p.counters) return;  // merged by attn_combine_kernel
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) {
      // CTAs c = 0 .. last_pos / kChunk do work for this tile; the others exited early.
      int* cnt = p.counters + (size_t)bh * p.n_qtiles + qtile;
      const int prev = atomicAdd(cnt, 1);
      s_last = prev == last_pos / kChunk;
      if (s_last) *cnt = 0;  // leave the workspace zeroed
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      merge_partials<__nv_bfloat16, HD, NTHR / 32, true>(p, bh, qtile, h, rows, first_pos, qoff, t0);
    }
  }
}

// Separate merge pass for the CUDA-core (fp32) kernel's chunk partials.
template <typename T, int HD>
__global__ void __launch_bounds__(kAttnThreads)
attn_combine_kernel(AttnParams p) {
  grid_dep_wait();
  grid_dep_launch();
  const int bh = blockIdx.x, qtile = blockIdx.y;
  const int b = bh / p.nkv, h = bh % p.nkv;
  const int ctx = p.ctx_lens[b], ql = p.q_lens[b], qoff = p.q_offsets[b];
  if (ql < 0 || ctx < ql || ctx > p.table_stride * p.bs) return;
  const int t0 = qtile * p.qt;
  if (t0 >= ql) return;
  const int nt = min(p.qt, ql - t0);
  merge_partials<T, HD, kWarps, std::is_same<T, __nv_bfloat16>::value>(p, bh, qtile, h, nt * p.group,
                                                                        ctx - ql + t0, qoff, t0);
}

template <int HD, int BS, int RB, bool TMA>
void launch_mma(const AttnParams& p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid, cudaStream_t stream) {
  // round buffers (K + V of SL tiles, twice), then the chunk's block table
  // (<= kChunk entries) and the round barriers; the slice merge reuses the round buffers.
  constexpr int SL = key_slices(HD);
  constexpr size_t kRounds = (size_t)kRoundBufs * SL * 2 * kMmaKeyTile * (TMA ? HD * 2 : HD * 2 + 16);
  constexpr size_t kMerge = (size_t)SL * RB * 16 * (HD + 8 + 2) * sizeof(float) +
                            (size_t)RB * 16 * (SL + 2) * sizeof(float);
  constexpr size_t kArea = kRounds > kMerge ? kRounds : kMerge;
  constexpr size_t smem = kArea + kChunk * sizeof(int) + kRoundBufs * sizeof(uint64_t) + (TMA ? 1024 : 0);
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(paged_attn_mma_kernel<HD, BS, RB, TMA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  });
  launch_kernel(paged_attn_mma_kernel<HD, BS, RB, TMA>, grid, dim3(RB * SL * 32), smem, stream, mk, mv, p);
}

template <int HD, int BS, bool TMA>
void launch_mma_rb(const AttnParams& p, const CUtensorMap& mk, const CUtensorMap& mv, dim3 grid,
                   cudaStream_t stream) {
  if (p.rb == 1) launch_mma<HD, BS, 1, TMA>(p, mk, mv, grid, stream);
  else if constexpr (max_row_blocks(HD) == 2) launch_mma<HD, BS, 2, TMA>(p, mk, mv, grid, stream);
  else if (p.rb == 2) launch_mma<HD, BS, 2, TMA>(p, mk, mv, grid, stream);
  else if (p.rb == 3) launch_mma<HD, BS, 3, TMA>(p, mk, mv, grid, stream);
  else launch_mma<HD, BS, 4, TMA>(p, mk, mv, grid, stream);
}

// 2-D map of one layer's pool as [num_blocks * 16 rows, nkv * hd] bf16, box {64, 16}, SWIZZLE_128B.
bool pool_map(CUtensorMap* map, const void* pool, int64_t rows, int width) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  auto encode = [&](CUtensorMap* m) {
    cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)width * 2};
    cuuint32_t box[2] = {64, 16};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(pool), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  // key: rows (32 bits) | width (24)
  if (rows < 0 || rows >= (1ll << 32) || width < 0 || width >= (1 << 24)) return encode(map);
  return cached_map(map, pool, (uint64_t)rows | (uint64_t)width << 32, encode);
}

template <typename T, int HD>
int launch(AttnParams& p, int batch, cudaStream_t stream) {
  // (sequence x kv-head) fastest: every sequence's chunk-0 CTA is scheduled before any
  // later chunk, and the empty late-chunk CTAs of short sequences come last.
  dim3 grid(batch * p.nkv, p.n_chunks, p.n_qtiles);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    CUtensorMap mk, mv;
    memset(&mk, 0, sizeof(mk));
    memset(&mv, 0, sizeof(mv));
    const int64_t rows = p.num_blocks * 16;
    if (p.bs == 16 && rows < (1ll << 31) && pool_map(&mk, p.pool_k, rows, p.nkv * HD) &&
        pool_map(&mv, p.pool_v, rows, p.nkv * HD))
      launch_mma_rb<HD, 16, true>(p, mk, mv, grid, stream);
    else if (p.bs == 16)
      launch_mma_rb<HD, 16, false>(p, mk, mv, grid, stream);
    else
      launch_mma_rb<HD, 0, false>(p, mk, mv, grid, stream);
  } else {
    const size_t smem = sizeof(float) * ((size_t)kMaxRows * HD + kKeyTile * (HD + 1) + kKeyTile * HD);
    static std::once_flag once;
    std::call_once(once, [smem] {
      cudaFuncSetAttribute(paged_attn_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    launch_kernel(paged_attn_kernel<T, HD>, dim3(grid), dim3(kAttnThreads), smem, stream, p);
  }
  int rc = check_launch("kve_paged_verify_attn");
  if (rc || !p.ws || (std::is_same<T, __nv_bfloat16>::value && p.counters)) return rc;  // merged in-kernel
  launch_kernel(attn_combine_kernel<T, HD>, dim3(batch * p.nkv, p.n_qtiles), dim3(kAttnThreads), 0, stream, p);
  return check_launch("kve_paged_verify_attn(combine)");
}

int qtile_tokens(int group) { return group >= kMaxRows ? 1 : kMaxRows / group; }

// bf16 kernel: row blocks of 16 query rows per CTA, from the largest query tile
// (rows = tokens x group) of the call, at most max_row_blocks(head_dim); a query
// tile holds 16 * rb / group tokens.
int row_blocks(int max_q_len, int group, int hd) {
  const long long rows = (long long)max_q_len * group;
  const int rb = rows <= 16 ? 1 : rows <= 32 ? 2 : rows <= 48 ? 3 : 4;
  return rb < max_row_blocks(hd) ? rb : max_row_blocks(hd);
}
int mma_qtile_tokens(int max_q_len, int group, int hd) { return row_blocks(max_q_len, group, hd) * 16 / group; }

// Split-mode workspace: kCounterSlots int32 chunk counters at offset 0 (always the
// same addresses, so no call's partials ever land on them), then the fp32
// partials [B*nkv][n_qtiles][n_chunks][64 rows][hd + 2]. Tiles beyond
// kCounterSlots merge in a second kernel instead.
constexpr size_t kCounterSlots = 16384;
constexpr size_t kCounterBytes = kCounterSlots * sizeof(int32_t);
size_t partials_bytes(size_t batch, size_t nkv, size_t n_qtiles, size_t n_chunks, int hd) {
  return batch * nkv * n_qtiles * n_chunks * partial_floats(hd) * sizeof(float);
}

}  // namespace
}  // namespace kve

using namespace kve;

extern "C" size_t kve_paged_attn_workspace_bytes(int batch, int max_q_len, int max_ctx, int num_heads,
                                                 int num_kv_heads, int head_dim) {
  if (batch <= 0 || num_kv_heads <= 0 || max_ctx <= kChunk || head_dim <= 0) return 0;
  int group = num_heads / num_kv_heads;
  if (group < 1 || group > kMaxRows) return 0;
  // The bf16 kernel's query tiles are never larger than the fp32 kernel's: size for them.
  int qt = mma_qtile_tokens(max_q_len, group, head_dim);
  if (qt < 1) qt = 1;
  size_t n_qtiles = (max_q_len + qt - 1) / qt;
  size_t n_chunks = (max_ctx + kChunk - 1) / kChunk;
  return kCounterBytes + partials_bytes(batch, num_kv_heads, n_qtiles, n_chunks, head_dim);
}

int kve::paged_attn_run(const void* q, int dtype, const void* pool_k, const void* pool_v,
                        const int32_t* block_tables, int table_stride, const int32_t* ctx_lens,
                        const int32_t* q_lens, const int32_t* q_offsets, int batch, int max_q_len, int max_ctx,
                        int num_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                        float scale, void* out, void* workspace, size_t workspace_bytes, int* dev_status,
                        bool hist_static, cudaStream_t stream) {
  if (batch < 0 || max_q_len < 0 || max_ctx < 0 || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads || block_size < 1 || table_stride < 1 || num_blocks < 1)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: bad sizes");
  if (batch == 0 || max_q_len == 0) return KVE_OK;
  if (head_dim != 64 && head_dim != 128)
    return set_error(KVE_ERR_SHAPE, "kve_paged_verify_attn: head_dim %d (supported: 64, 128)", head_dim);
  int group = num_heads / num_kv_heads;
  if (group > kMaxRows) return set_error(KVE_ERR_SHAPE, "kve_paged_verify_attn: group %d > %d", group, kMaxRows);
  if (dtype == KVE_BF16 && group > 16 * max_row_blocks(head_dim))
    return set_error(KVE_ERR_SHAPE, "kve_paged_verify_attn: bf16 group %d > %d at head_dim %d", group,
                     16 * max_row_blocks(head_dim), head_dim);
  if (!q || !pool_k || !pool_v || !block_tables || !ctx_lens || !q_lens || !q_offsets || !out)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: null pointer");
  if ((uintptr_t)pool_k % 16 || (uintptr_t)pool_v % 16)
    return set_error(KVE_ERR_ARG, "kve_paged_verify_attn: pool pointers must be 16-byte aligned");
  AttnParams p{};
  p.q = q; p.pool_k = pool_k; p.pool_v = pool_v; p.tables = block_tables; p.table_stride = table_stride;
  p.ctx_lens = ctx_lens; p.q_lens = q_lens; p.q_offsets = q_offsets;
  p.nq = num_heads; p.nkv = num_kv_heads; p.group = group;
  p.rb = row_blocks(max_q_len, group, head_dim);
  p.qt = dtype == KVE_BF16 ? mma_qtile_tokens(max_q_len, group, head_dim) : qtile_tokens(group);
  p.bs = block_size; p.num_blocks = num_blocks; p.scale = scale; p.out = out; p.status = dev_status;
  p.hist_static = hist_static ? 1 : 0;
  p.n_qtiles = (max_q_len + p.qt - 1) / p.qt;
  p.n_chunks = (max_ctx + kChunk - 1) / kChunk;
  if (p.n_chunks < 1) p.n_chunks = 1;
  p.ws = nullptr;
  if (p.n_chunks > 1) {
    size_t need = kve_paged_attn_workspace_bytes(batch, max_q_len, max_ctx, num_heads, num_kv_heads, head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(KVE_ERR_WORKSPACE, "kve_paged_verify_attn: workspace needs %zu bytes", need);
    p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
    p.counters = (size_t)batch * num_kv_heads * p.n_qtiles <= kCounterSlots ? static_cast<int*>(workspace)
                                                                             : nullptr;
  }
  if (dtype == KVE_F32) {
    return head_dim == 64 ? launch<float, 64>(p, batch, stream) : launch<float, 128>(p, batch, stream);
  } else if (dtype == KVE_BF16) {
    return head_dim == 64 ? launch<__nv_bfloat16, 64>(p, batch, stream)
                          : launch<__nv_bfloat16, 128>(p, batch, stream);
  }
  return set_error(KVE_ERR_DTYPE, "kve_paged_verify_attn: dtype %d", dtype);
}

extern "C" int kve_paged_verify_attn(const void* q, int dtype, const void* pool_k, const void* pool_v,
                                     const int32_t* block_tables, int table_stride, const int32_t* ctx_lens,
                                     const int32_t* q_lens, const int32_t* q_offsets, int batch,
                                     int max_q_len, int max_ctx, int num_heads, int num_kv_heads,
                                     int head_dim, int block_size, int64_t num_blocks, float scale,
                                     void* out, void* workspace, size_t workspace_bytes, int* dev_status,
                                     cudaStream_t stream) {
  return paged_attn_run(q, dtype, pool_k, pool_v, block_tables, table_stride, ctx_lens, q_lens, q_offsets, batch,
                        max_q_len, max_ctx, num_heads, num_kv_heads, head_dim, block_size, num_blocks, scale, out,
                        workspace, workspace_bytes, dev_status, false, stream);
}
