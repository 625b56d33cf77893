// Shared-memory mbarrier and TMA helpers of the sm_100a kernels (tensor maps
// are built on the host with cuTensorMapEncodeTiled). Every wait is bounded.
#pragma once

#include <cuda.h>

#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "kve_common.cuh"

namespace kve {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Raise the expected transaction bytes of the current phase without arriving.
__device__ __forceinline__ void mbar_add_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// Bounded wait: false (and KVE_ERR_TIMEOUT in status) if the phase never completes
// within limit_ns (the library-wide limit unless a self-test shortens it).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) {
      report(status, KVE_ERR_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before later
// async-proxy (TMA) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

// Encoded tensor maps by their parameters: the forward pass asks for the same few
// (pointer, shape, box) maps on every layer and every pass, and an encoding costs
// host time on the launch path. A map holds only the address, shape, strides and
// box, so a hit is exactly the map the encoder would return. `shape` packs the
// rest of the parameters of one call site (each call site has its own cache).
struct MapCacheKey {
  uint64_t ptr, shape;
  bool operator==(const MapCacheKey& o) const { return ptr == o.ptr && shape == o.shape; }
};
struct MapCacheHash {
  size_t operator()(const MapCacheKey& k) const { return std::hash<uint64_t>()(k.ptr * 0x9E3779B97F4A7C15ull ^ k.shape); }
};
template <typename Encode>
inline bool cached_map(CUtensorMap* map, const void* ptr, uint64_t shape, Encode&& encode) {
  static std::mutex mu;
  static std::unordered_map<MapCacheKey, CUtensorMap, MapCacheHash> cache;
  const MapCacheKey key{reinterpret_cast<uint64_t>(ptr), shape};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *map = it->second;
      return true;
    }
  }
  if (!encode(map)) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 16384) cache.clear();
  cache.emplace(key, *map);
  return true;
}

}  // namespace kve
