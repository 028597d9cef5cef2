// tcgen05 / TMA / mbarrier helpers shared by the tensor-core GEMM kernels.
// Device helpers live in an anonymous namespace (one copy per translation
// unit); every wait is iteration-bounded.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <unordered_map>

namespace aideen {
namespace {

constexpr uint32_t kMaxSpin = 1u << 26;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < kMaxSpin; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Shared-memory matrix descriptor (sm100 version field = 1).  layout 2 =
// 128-byte swizzle (K-major operands), layout 1 = 128-byte swizzle on 32-byte
// atoms, the only layout the tf32 MMA accepts for MN-major operands.
__device__ __forceinline__ uint64_t sdesc(const void *base, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                          uint32_t layout) {
  const uint64_t addr = smem_u32(base);
  return ((addr & 0x3FFFFull) >> 4) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_c, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_c),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}


// Bulk tensor store / reduce-add from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap *map, const void *src, int x, int y,
                                                  int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                              CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

inline EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}


// 3-D fp32 tensor map: dim0 contiguous (extent e0), dim1 stride s1 elements,
// dim2 stride s2 elements (0: packed after dim1).  Encoded maps are kept per
// host thread, keyed by every argument: a training step encodes the same ~80
// maps every time, and a map depends only on the address and the shape.
struct MapKey {
  const void *base;
  uint64_t e0, e1, e2, s1, s2;
  uint32_t box0, box1, sw;
  bool operator==(const MapKey &o) const {
    return base == o.base && e0 == o.e0 && e1 == o.e1 && e2 == o.e2 && s1 == o.s1 && s2 == o.s2 &&
           box0 == o.box0 && box1 == o.box1 && sw == o.sw;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey &k) const {
    uint64_t h = reinterpret_cast<uint64_t>(k.base);
    for (uint64_t v : {k.e0, k.e1, k.e2, k.s1, k.s2, (uint64_t)k.box0 << 32 | k.box1, (uint64_t)k.sw})
      h = (h ^ v) * 0x100000001B3ull;
    return (size_t)h;
  }
};

inline bool make_map_sw(CUtensorMap *m, const float *base, uint64_t e0, uint64_t e1, uint64_t e2,
                        uint64_t s1, uint64_t s2, uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  static thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{base, e0, e1, e2, s1, s2, box0, box1, (uint32_t)sw};
  const auto it = cache.find(key);
  if (it != cache.end()) {
    *m = it->second;
    return true;
  }
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {e0, e1, e2 ? e2 : 1};
  const cuuint64_t strides[2] = {s1 * 4, (s2 ? s2 : s1 * e1) * 4};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const bool ok = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  if (ok) {
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, *m);
  }
  return ok;
}

}  // namespace aideen
