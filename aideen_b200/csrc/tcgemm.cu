// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[b] = alpha * opA(A[b]) * opB(B[b]) + beta * C[b], row-major, the same
// contract as gemm_f32 (kernels.cuh).  One CTA computes a 128 x BN tile
// (BN = 32, 64, 128 or 256):
//
//   * TMA (cp.async.bulk.tensor, no multicast) brings fp32 tiles of A and B
//     into 128-byte-swizzled shared memory, BK = 32 along K per stage, in a
//     ring of as many stages as fit (the stage size depends on the mode);
//   * eight warps convert each staged value x in place: 3xTF32 splits it into
//     x_hi = x with the low 13 mantissa bits cleared (exact in tf32) and
//     x_lo = x - x_hi; single TF32 rounds it to the nearest tf32 value;
//   * one thread issues, per K=8 step, three tcgen05.mma kind::tf32
//     (hi*hi + hi*lo + lo*hi; one in single mode) accumulating in TMEM
//     (fp32), then tcgen05.commit releases the stage to the TMA producer;
//   * the epilogue reads the accumulator with tcgen05.ld (warp w owns TMEM
//     lanes 32w..32w+31 = tile rows), stages 32x32 boxes in the (now idle)
//     stage ring and writes them with bulk tensor stores / reduce-adds.
//
// The shared-memory traffic per K block (TMA writes, the conversion pass,
// the MMA operand reads) bounds this kernel before the tensor pipe does, so
// wide tiles (fewer A re-reads per product) and deep rings pay.
//
// The 3-term split keeps the product error at ~2^-21 relative, i.e. fp32
// level, which the DEQ forward needs (its stop rule compares residuals near
// 1e-4).  Operands may be K-major or MN-major, so transposed views
// (weight gradients A^T B) need no copies.  Every mbarrier wait is bounded;
// on timeout the kernel records an error code and skips the remaining work.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace aideen {
namespace {

// 2 role warps + NCONV converter / epilogue warps
constexpr int BM = 128, BK = 32, MAX_STAGES = 8, NCONV = 8, TC_THREADS = 64 + 32 * NCONV;
constexpr int SMEM_LIMIT = 232448;  // opt-in dynamic shared memory per block on sm_100

__device__ unsigned int g_tc_error;  // first error code seen by any tcgemm CTA

#ifdef AIDEEN_TC_PROF
// Per-CTA timeline of the launches since the last reset (profiling builds
// only), clock64 cycles after the CTA's start: [0] setup done, [1] first stage
// converted, [2] last stage converted, [3] accumulator complete, [4] end,
// [5] converter wait on full (warp 2), [6] MMA wait on conv, [7] producer
// wait on empty.
__device__ unsigned long long g_tc_prof[4096 * 8];
#define TCP(i, v) if (prof_row) prof_row[i] = (v)
#else
#define TCP(i, v)
#endif

// x -> tf32 in place, rounded to nearest (cvt.rna: ties away from zero)
// instead of the truncation the tensor core applies to fp32 bit patterns.
__device__ __forceinline__ float tf32_rn(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void round1(float4 *raw) {
  float4 v = *raw;
  v.x = tf32_rn(v.x);
  v.y = tf32_rn(v.y);
  v.z = tf32_rn(v.z);
  v.w = tf32_rn(v.w);
  *raw = v;
}

// x -> (x_hi, x_lo) in place / alongside: x_hi keeps the 10 tf32 mantissa bits.
__device__ __forceinline__ void split1(float4 *raw, float4 *lo) {
  const float4 v = *raw;
  float4 hv;
  hv.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
  hv.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
  hv.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
  hv.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
  *raw = hv;
  *lo = make_float4(v.x - hv.x, v.y - hv.y, v.z - hv.z, v.w - hv.w);
}

struct TcParams {
  int M, N, K;
  bool a_kmajor, b_kmajor;  // K contiguous in memory (else M/N contiguous)
  float *C;
  long ldc, strideC;
  float alpha, beta;
  int a_batched, b_batched;  // operand map has a batch dimension
  int ksplit, kchunk;        // split-K: blockIdx.z = split index, kchunk K-blocks each
  int tma_epi;               // 1: epilogue through 32x32 shared-memory boxes + bulk tensor
                             //    store (beta 0) or reduce-add (beta 1) on mapC
  int stages;                // depth of the TMA ring (2..MAX_STAGES)
};

constexpr int BOX_BYTES = 32 * 32 * 4;  // one 32x32 fp32 epilogue box

template <int BN, bool SPLIT3>
__host__ __device__ constexpr int stage_bytes() {
  return (SPLIT3 ? 2 : 1) * (BM * BK * 4 + BN * BK * 4);
}
constexpr size_t ring_offset_bytes = 1024;                      // alignment slack
constexpr size_t bar_bytes = 8 * (3 * MAX_STAGES + 1) + 16;  // mbarriers, TMEM slot, error word
size_t tc_smem(int stage_b, int stages) { return ring_offset_bytes + (size_t)stages * stage_b + bar_bytes; }

// Warp roles: warp 0 lane 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer (lane 0), warps 2..2+NCONV-1 = converters and epilogue (warp w reads
// TMEM lanes 32*(w%4)..+31; warps w and w+4 take alternate 32-column chunks).
// Per stage s: full[s] (TMA landed) -> conv[s] (converted, NCONV warp
// arrivals) -> empty[s] (MMAs done, tcgen05.commit) -> producer refills.
template <int BN, bool SPLIT3>
__global__ void __launch_bounds__(TC_THREADS) tcgemm_kernel(const __grid_constant__ CUtensorMap mapA,
                                                            const __grid_constant__ CUtensorMap mapB,
                                                            const __grid_constant__ CUtensorMap mapC,
                                                            TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
  constexpr int STAGE_BYTES = stage_bytes<BN, SPLIT3>();
  constexpr uint32_t TMEM_COLS = BN;  // a power of two >= 32
  const int S = p.stages;
  // the epilogue boxes (NCONV warps x 2) reuse the ring: every MMA has completed
  // (and so every copy has landed) before the first box is written
  unsigned char *boxes = sm;
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + (size_t)S * STAGE_BYTES);
  uint64_t *conv = full + MAX_STAGES;
  uint64_t *empty = conv + MAX_STAGES;
  uint64_t *done = empty + MAX_STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  uint32_t *err = tmem_slot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM, bz = blockIdx.z;
  // with split-K, z = batch * ksplit + split: the split selects the K range,
  // the output slice is z itself (workspace [batch][ksplit][M][N])
  const int zab = p.ksplit > 1 ? bz / p.ksplit : bz;
  const int kb0 = p.ksplit > 1 ? (bz % p.ksplit) * p.kchunk : 0;
  const int ktot = (p.K + BK - 1) / BK;
  const int kblocks = p.ksplit > 1 ? min(p.kchunk, ktot - kb0) : ktot;
#ifdef AIDEEN_TC_PROF
  const long long t_start = clock64();
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  unsigned long long *prof_row = cta < 4096 ? g_tc_prof + 8 * cta : nullptr;
#endif

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], NCONV);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *err = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
#ifdef AIDEEN_TC_PROF
  if (tid == 0) TCP(0, clock64() - t_start);
  long long w_acc = 0;
#endif

  // 0 A (hi), 1 A lo, 2 B (hi), 3 B lo; single mode holds only 0 and 2
  auto stage_ptr = [&](int s, int which) -> unsigned char * {
    unsigned char *base = sm + (size_t)s * STAGE_BYTES;
    if (!SPLIT3) return which == 0 ? base : base + A_BYTES;
    return which == 0 ? base : which == 1 ? base + A_BYTES : which == 2 ? base + 2 * A_BYTES
                                                                        : base + 2 * A_BYTES + B_BYTES;
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < kblocks && ok; ++kb) {
        const int s = kb % S;
#ifdef AIDEEN_TC_PROF
        const long long w0 = clock64();
#endif
        if (kb >= S && !mbar_wait(&empty[s], ((kb / S) - 1) & 1)) { ok = false; break; }
#ifdef AIDEEN_TC_PROF
        w_acc += clock64() - w0;
#endif
        if (*(volatile uint32_t *)err) { ok = false; break; }
        const int k0 = (kb0 + kb) * BK;
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        const int za = p.a_batched ? zab : 0, zb = p.b_batched ? zab : 0;
        if (p.a_kmajor) {
          tma_load_3d(stage_ptr(s, 0), &mapA, &full[s], k0, m0, za);
        } else {
#pragma unroll
          for (int c = 0; c < BM / 32; ++c)
            tma_load_3d(stage_ptr(s, 0) + c * (BK * 128), &mapA, &full[s], m0 + 32 * c, k0, za);
        }
        if (p.b_kmajor) {
          tma_load_3d(stage_ptr(s, 2), &mapB, &full[s], k0, n0, zb);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
            tma_load_3d(stage_ptr(s, 2) + c * (BK * 128), &mapB, &full[s], n0 + 32 * c, k0, zb);
        }
        issued = kb + 1;
      }
      if (!ok) atomicExch(err, 1u);
      TCP(7, w_acc);
      // every issued copy must land before the CTA can exit (bounded)
      for (int kb = issued - S < 0 ? 0 : issued - S; kb < issued; ++kb)
        mbar_wait(&full[kb % S], (kb / S) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((p.a_kmajor ? 0u : 1u) << 15) |
                             ((p.b_kmajor ? 0u : 1u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(BM >> 4) << 24);
      // K-major: LBO unused (16), 8-row atoms (SBO 1024).  MN-major: 32-wide MN
      // blocks BK*128 bytes apart (LBO), 4-row K atoms (SBO 512).
      const uint32_t lboA = p.a_kmajor ? 16u : BK * 128u, sboA = p.a_kmajor ? 1024u : 512u;
      const uint32_t lboB = p.b_kmajor ? 16u : BK * 128u, sboB = p.b_kmajor ? 1024u : 512u;
      const uint32_t layA = p.a_kmajor ? 2u : 1u, layB = p.b_kmajor ? 2u : 1u;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int s = kb % S;
#ifdef AIDEEN_TC_PROF
        const long long w0 = clock64();
#endif
        if (!mbar_wait(&conv[s], (kb / S) & 1) || *(volatile uint32_t *)err) { ok = false; break; }
#ifdef AIDEEN_TC_PROF
        w_acc += clock64() - w0;
#endif
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int k8 = 0; k8 < BK / 8; ++k8) {
          // K-major: +32 B along the swizzled row; MN-major: +1024 B (8 K rows)
          const uint32_t koffA = p.a_kmajor ? k8 * 32 : k8 * 1024;
          const uint32_t koffB = p.b_kmajor ? k8 * 32 : k8 * 1024;
          const uint64_t ahi = sdesc(stage_ptr(s, 0) + koffA, lboA, sboA, layA);
          const uint64_t bhi = sdesc(stage_ptr(s, 2) + koffB, lboB, sboB, layB);
          umma_tf32(tmem, ahi, bhi, idesc, (kb > 0 || k8 > 0) ? 1u : 0u);
          if (SPLIT3) {
            const uint64_t alo = sdesc(stage_ptr(s, 1) + koffA, lboA, sboA, layA);
            const uint64_t blo = sdesc(stage_ptr(s, 3) + koffB, lboB, sboB, layB);
            umma_tf32(tmem, ahi, blo, idesc, 1u);
            umma_tf32(tmem, alo, bhi, idesc, 1u);
          }
        }
        umma_commit(&empty[s]);
      }
      if (!ok) atomicExch(err, 1u);
      TCP(6, w_acc);
      umma_commit(done);  // arrives once every MMA issued so far has completed
    }
  } else {  // ---------------- converters (32 * NCONV threads) + epilogue
    constexpr int NCT = 32 * NCONV;
    const int ct = tid - 64;
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % S;
#ifdef AIDEEN_TC_PROF
      const long long w0 = clock64();
#endif
      if (!mbar_wait(&full[s], (kb / S) & 1)) { atomicExch(err, 1u); break; }
      if (*(volatile uint32_t *)err) break;
#ifdef AIDEEN_TC_PROF
      w_acc += clock64() - w0;
#endif
      float4 *ra = reinterpret_cast<float4 *>(stage_ptr(s, 0));
      float4 *rb = reinterpret_cast<float4 *>(stage_ptr(s, 2));
      if (!SPLIT3) {
#pragma unroll 4
        for (int i = ct; i < A_BYTES / 16; i += NCT) round1(ra + i);
#pragma unroll 4
        for (int i = ct; i < B_BYTES / 16; i += NCT) round1(rb + i);
      } else {
        float4 *la = reinterpret_cast<float4 *>(stage_ptr(s, 1));
        float4 *lb = reinterpret_cast<float4 *>(stage_ptr(s, 3));
#pragma unroll 4
        for (int i = ct; i < A_BYTES / 16; i += NCT) split1(ra + i, la + i);
#pragma unroll 4
        for (int i = ct; i < B_BYTES / 16; i += NCT) split1(rb + i, lb + i);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
#ifdef AIDEEN_TC_PROF
      if (tid == 64 && kb == 0) TCP(1, clock64() - t_start);
      if (tid == 64 && kb == kblocks - 1) TCP(2, clock64() - t_start);
#endif
    }
    const bool ok = mbar_wait(done, 0) && !*(volatile uint32_t *)err;
#ifdef AIDEEN_TC_PROF
    if (tid == 64) { TCP(3, clock64() - t_start); TCP(5, w_acc); }
#endif
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && p.tma_epi) {
      const int q = warp & 3;  // TMEM lane quadrant this warp may access
      const int half = (warp - 2) >> 2;  // which alternate 32-column chunks
      const int rowbase = m0 + q * 32;
      unsigned char *mybox = boxes + (warp - 2) * 2 * BOX_BYTES;
      int nst = 0;
#pragma unroll 1
      for (int c0 = 32 * half; c0 < BN; c0 += 32 * (NCONV / 4)) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
            "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
            "%28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
              "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
              "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
              "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int col = n0 + c0;
        if (col >= p.N || rowbase >= p.M) continue;  // box entirely outside C
        unsigned char *box = mybox + (nst & 1) * BOX_BYTES;
        if (lane == 0) bulk_wait_read<1>();  // the store issued from this box two boxes ago is done reading
        __syncwarp();
        float4 *row = reinterpret_cast<float4 *>(box + lane * 128);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          row[k ^ (lane & 7)] = make_float4(p.alpha * __uint_as_float(r[4 * k]), p.alpha * __uint_as_float(r[4 * k + 1]),
                                            p.alpha * __uint_as_float(r[4 * k + 2]),
                                            p.alpha * __uint_as_float(r[4 * k + 3]));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (p.beta != 0.f) tma_reduce_add_3d(&mapC, box, col, rowbase, bz);
          else tma_store_3d(&mapC, box, col, rowbase, bz);
          bulk_commit();
        }
        ++nst;
      }
      if (lane == 0) bulk_wait<0>();  // stores complete before the CTA's shared memory goes away
    } else if (ok) {
      const int q = warp & 3;  // TMEM lane quadrant this warp may access
      const int half = (warp - 2) >> 2;
      const int row = m0 + q * 32 + lane;
      float *crow = p.C + (long)bz * p.strideC + (long)row * p.ldc;
#pragma unroll 1
      for (int c0 = 32 * half; c0 < BN; c0 += 32 * (NCONV / 4)) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
            "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
            "%28, %29, %30, %31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
              "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
              "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
              "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < p.M) {
          if (p.beta == 0.f && n0 + c0 + 32 <= p.N && ((p.ldc | (long)(n0 + c0)) & 3) == 0 &&
              ((reinterpret_cast<uintptr_t>(crow) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4 *>(crow + n0 + c0 + j) =
                  make_float4(p.alpha * __uint_as_float(r[j]), p.alpha * __uint_as_float(r[j + 1]),
                              p.alpha * __uint_as_float(r[j + 2]), p.alpha * __uint_as_float(r[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int col = n0 + c0 + j;
              if (col < p.N) {
                float v = p.alpha * __uint_as_float(r[j]);
                if (p.beta != 0.f) v += p.beta * crow[col];
                crow[col] = v;
              }
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && *(volatile uint32_t *)err) atomicCAS(&g_tc_error, 0u, 1u);
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
#ifdef AIDEEN_TC_PROF
  if (tid == 0) TCP(4, clock64() - t_start);
#endif
}

// ---------------------------------------------------------------- host side
// 3-D fp32 map: dim0 contiguous (extent e0), dim1 stride s1 elements, dim2 stride s2.
bool make_map(CUtensorMap *m, const float *base, uint64_t e0, uint64_t e1, uint64_t e2, uint64_t s1,
              uint64_t s2, uint32_t box0, uint32_t box1, bool kmajor) {
  return make_map_sw(m, base, e0, e1, e2, s1, s2, box0, box1,
                     kmajor ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

// Tuning knobs read once from the environment (0 = the built-in choice):
// AIDEEN_TC_BN (32, 64, 128, 256), AIDEEN_TC_STAGES (2..8), AIDEEN_TC_CPS
// (CTAs per SM the ring is sized for, 1 or 2).
int env_int(const char *name) {
  const char *v = getenv(name);
  return v ? atoi(v) : 0;
}
struct TcTuning {
  int bn = env_int("AIDEEN_TC_BN"), stages = env_int("AIDEEN_TC_STAGES"), cps = env_int("AIDEEN_TC_CPS");
  int slots = env_int("AIDEEN_TC_SLOTS");
};
const TcTuning &tuning() {
  static TcTuning t;
  return t;
}

// Ring depth: as many stages as fit the shared memory of `cps` CTAs per SM,
// no more than the K blocks one CTA walks (a short-K GEMM then holds a small
// ring and more CTAs share an SM), and at least the bytes of the epilogue
// boxes that reuse it (2 per epilogue warp: 4 warps when BN = 32, else 8).
int ring_stages(int stage_b, int cps, int kblocks = MAX_STAGES, int bn = 128) {
  const TcTuning &t = tuning();
  const long budget = SMEM_LIMIT / cps - 1024 * (cps - 1) - (long)ring_offset_bytes - (long)bar_bytes;
  int st = (int)(budget / stage_b);
  if (st > MAX_STAGES) st = MAX_STAGES;
  if (t.stages >= 2 && t.stages < st) st = t.stages;
  if (kblocks < st) st = kblocks;
  const int box_bytes = 2 * (bn == 32 ? 4 : NCONV) * BOX_BYTES;
  if (st < 1) st = 1;
  while (st * stage_b < box_bytes) ++st;
  return st;
}

template <int BN, bool SPLIT3>
cudaError_t launch_tc(dim3 grid, const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mc, TcParams p,
                      int cps, cudaStream_t st) {
  static bool attr_set = false;
  const int kb_cta = p.ksplit > 1 ? p.kchunk : (p.K + BK - 1) / BK;
  p.stages = ring_stages(stage_bytes<BN, SPLIT3>(), cps, kb_cta, BN);
  if (tc_smem(stage_bytes<BN, SPLIT3>(), p.stages) > (size_t)SMEM_LIMIT) return cudaErrorInvalidValue;
  if (!attr_set) {
    const cudaError_t e = cudaFuncSetAttribute(tcgemm_kernel<BN, SPLIT3>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  tcgemm_kernel<BN, SPLIT3><<<grid, TC_THREADS, tc_smem(stage_bytes<BN, SPLIT3>(), p.stages), st>>>(ma, mb, mc, p);
  return cudaGetLastError();
}

// C = alpha * sum_s ws[b][s] + beta * C over one split-K product of R x Cc
// outputs per batch entry, summed in split order (deterministic).  trans:
// workspace (r, c) is C's (c, r) (the product was formed with A and B
// swapped); col_group: C's column n sits at (n / col_group) * group_stride +
// n % col_group of its row.  Each thread sums 4 adjacent workspace columns.
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, int splits, int batch, int R, int Cc,
                                     float *C, long ldc, long strideC, float alpha, float beta, int trans,
                                     int col_group, long group_stride) {
  const int c4n = (Cc + 3) >> 2;
  const long per_b = (long)R * c4n, total = per_b * batch;
  const long rc = (long)R * Cc;
  const bool vec = (Cc & 3) == 0;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int bb = (int)(i / per_b);
    const int rem = (int)(i - (long)bb * per_b);
    const int r = rem / c4n, c = (rem - r * c4n) * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const float *src = ws + (long)bb * splits * rc + (long)r * Cc + c;
    for (int s = 0; s < splits; ++s, src += rc) {
      if (vec) {
        const float4 v = *reinterpret_cast<const float4 *>(src);
        acc[0] += v.x; acc[1] += v.y; acc[2] += v.z; acc[3] += v.w;
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (c + q < Cc) acc[q] += src[q];
      }
    }
    float *cb = C + (long)bb * strideC;
    if (!trans) {
      const long colbase = col_group > 0 ? (long)(c / col_group) * group_stride + c % col_group : c;
      float *dst = cb + (long)r * ldc + colbase;
      if (vec && (col_group == 0 || (col_group & 3) == 0) && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
        float4 o = make_float4(alpha * acc[0], alpha * acc[1], alpha * acc[2], alpha * acc[3]);
        if (beta != 0.f) {
          const float4 old = *reinterpret_cast<const float4 *>(dst);
          o.x += beta * old.x; o.y += beta * old.y; o.z += beta * old.z; o.w += beta * old.w;
        }
        *reinterpret_cast<float4 *>(dst) = o;
        continue;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (c + q >= Cc) break;
      const int row = trans ? c + q : r, col = trans ? r : c + q;
      float *dst = cb + (long)row * ldc +
                   (col_group > 0 ? (long)(col / col_group) * group_stride + col % col_group : col);
      *dst = beta != 0.f ? alpha * acc[q] + beta * *dst : alpha * acc[q];
    }
  }
}

}  // namespace

bool tc_gemm_supported(const GemmArgs &g) {
  if (g.abias) return false;
  if (g.K <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.B)) & 15) return false;
  if ((g.lda | g.ldb | g.strideA | g.strideB) & 3) return false;
  return encode_fn() != nullptr;
}

cudaError_t tc_gemm(const GemmArgs &g0, cudaStream_t st, float *ws, size_t ws_floats) {
  if (g0.M <= 0 || g0.N <= 0 || g0.batch <= 0) return cudaSuccess;
  GemmArgs g = g0;
  // A short output (M <= 64 rows, e.g. a 32-row head gradient) wastes most of
  // the 128-row MMA: form C^T = opB^T opA^T instead and let the split-K
  // reduction write it back transposed.
  bool trans = false;
  const size_t out_floats = (size_t)g0.batch * g0.M * g0.N;
  if (g.M <= 64 && g.N >= 128 && ws && out_floats <= ws_floats) {
    trans = true;
    g.M = g0.N; g.N = g0.M;
    g.A = g0.B; g.lda = g0.ldb; g.strideA = g0.strideB; g.transA = !g0.transB;
    g.B = g0.A; g.ldb = g0.lda; g.strideB = g0.strideA; g.transB = !g0.transA;
  }
  // the column-group and transposed outputs exist only in the split-K reduction
  const bool need_ws = trans || g.col_group > 0;
  if (need_ws && (!ws || out_floats > ws_floats)) return cudaErrorInvalidValue;
  // A: K-major when not transposed (row m contiguous along k).
  const bool a_k = !g.transA, b_k = g.transB;
  const bool split3 = !g.tf32;
  const TcTuning &t = tuning();
  int BN = g.N <= 32 ? 32 : g.N <= 64 ? 64 : (split3 || g.N < 256) ? 128 : 256;
  // narrower tiles while twice as many still fit one wave and K is too short
  // to split (measured: 2048 x 512 x 1024 single TF32, 32 tiles
  // of 256 columns 36.8 us, 128 tiles of 64 columns 24.9 us)
  {
    const int kbl = (g.K + BK - 1) / BK, tm = (g.M + BM - 1) / BM;
    while (BN > 32 && 2L * ((g.N + BN - 1) / BN) * tm * g.batch <= 148 && !(ws && kbl >= 64)) BN /= 2;
  }
  if (t.bn == 32 || t.bn == 64 || t.bn == 128 || (t.bn == 256 && !split3)) BN = t.bn;
  CUtensorMap ma, mb;
  const bool a_batched = g.strideA != 0 && g.batch > 1;
  bool ok;
  if (a_k)  // dims: k (contiguous), m, batch
    ok = make_map(&ma, g.A, g.K, g.M, a_batched ? g.batch : 1, g.lda, g.strideA, BK, BM, true);
  else      // dims: m (contiguous), k, batch
    ok = make_map(&ma, g.A, g.M, g.K, a_batched ? g.batch : 1, g.lda, g.strideA, 32, BK, false);
  if (!ok) return cudaErrorInvalidValue;
  const bool b_batched = g.strideB != 0 && g.batch > 1;
  if (b_k)  // B stored [n][k]
    ok = make_map(&mb, g.B, g.K, g.N, b_batched ? g.batch : 1, g.ldb, g.strideB, BK, BN, true);
  else      // B stored [k][n]
    ok = make_map(&mb, g.B, g.N, g.K, b_batched ? g.batch : 1, g.ldb, g.strideB, 32, BK, false);
  if (!ok) return cudaErrorInvalidValue;
  TcParams p{g.M, g.N, g.K, a_k, b_k, g.C, g.ldc, g.strideC, g.alpha, g.beta, a_batched ? 1 : 0,
             b_batched ? 1 : 0, 1, 0, 0, 0};
  const int tiles_n = (g.N + BN - 1) / BN, tiles_m = (g.M + BM - 1) / BM;
  const int tiles = tiles_n * tiles_m * g.batch;
  const int kblocks = (g.K + BK - 1) / BK;
  int zdim = g.batch;
  // Split K when the output (all batches) has too few tiles to fill the GPU
  // and K is long enough: as many splits as fit whole in one wave of the
  // resident CTA slots (two per SM when half the shared memory still holds a
  // 2-stage ring, else one); a second, partial wave would run alone.
  const int sb = split3 ? 2 * (BM + BN) * BK * 4 : (BM + BN) * BK * 4;
  int splits = 1, chunk = kblocks;
  if (ws && tiles < 148 && kblocks >= 64) {
    const int slots = t.slots > 0 ? t.slots : 148 * (ring_stages(sb, 2, MAX_STAGES, BN) >= 2 ? 2 : 1);
    splits = slots / tiles;
    if (splits < 1) splits = 1;
    if (splits > 16) splits = 16;
    if (splits > kblocks / 4) splits = kblocks / 4;
    chunk = (kblocks + splits - 1) / splits;
    splits = (kblocks + chunk - 1) / chunk;
  }
  if (ws && splits > 1 && (size_t)splits * out_floats > ws_floats) {  // as many splits as the workspace holds
    splits = (int)(ws_floats / out_floats);
    if (splits < 1) splits = 1;
    chunk = (kblocks + splits - 1) / splits;
    splits = (kblocks + chunk - 1) / chunk;
  }
  const bool use_ws = need_ws || splits > 1;
  if (use_ws) {
    {
      p.ksplit = splits;
      p.kchunk = chunk;
      p.C = ws;
      p.ldc = g.N;
      p.strideC = (long)g.M * g.N;
      p.alpha = 1.f;
      p.beta = 0.f;
      zdim = splits * g.batch;
    }
  }
  const bool to_ws = p.C == ws && ws != nullptr && use_ws;
  // Coalesced epilogue through bulk tensor stores when C allows a tensor map
  // (16-byte aligned rows) and beta is 0 or 1 (reduce-add in L2).
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  if ((p.beta == 0.f || p.beta == 1.f) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
      ((p.ldc | p.strideC) & 3) == 0 &&
      make_map_sw(&mc, p.C, g.N, g.M, zdim, p.ldc, p.strideC, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
    p.tma_epi = 1;
  dim3 grid(tiles_n, tiles_m, zdim);
  // two CTAs per SM whenever the grid covers the GPU more than once: one
  // CTA's prologue, first-load latency and epilogue then overlap the other's
  // main loop, which pays more than a deeper ring (measured: 3xTF32 at
  // 16384 x 512 x 512 x 8, 557 -> 480 us with a 1-stage ring per CTA)
  int cps = (long)tiles_n * tiles_m * zdim > 148 ? 2 : 1;
  if (t.cps == 1 || t.cps == 2) cps = t.cps;
  cudaError_t e;
  if (split3) {
    e = BN == 32 ? launch_tc<32, true>(grid, ma, mb, mc, p, cps, st)
        : BN == 64 ? launch_tc<64, true>(grid, ma, mb, mc, p, cps, st)
                   : launch_tc<128, true>(grid, ma, mb, mc, p, cps, st);
  } else {
    e = BN == 32 ? launch_tc<32, false>(grid, ma, mb, mc, p, cps, st)
        : BN == 64 ? launch_tc<64, false>(grid, ma, mb, mc, p, cps, st)
        : BN == 128 ? launch_tc<128, false>(grid, ma, mb, mc, p, cps, st)
                    : launch_tc<256, false>(grid, ma, mb, mc, p, cps, st);
  }
  if (e != cudaSuccess || !to_ws) return e;
  tc_extra_launches++;
  splitk_reduce_kernel<<<148 * 4, 256, 0, st>>>(ws, p.ksplit, g.batch, g.M, g.N, g0.C, g0.ldc,
                                                g.batch > 1 ? g0.strideC : 0, g0.alpha, g0.beta, trans ? 1 : 0,
                                                g0.col_group, g0.group_stride);
  return cudaGetLastError();
}

thread_local unsigned tc_extra_launches = 0;

unsigned tc_take_extra_launches() {
  const unsigned v = tc_extra_launches;
  tc_extra_launches = 0;
  return v;
}

unsigned int tc_gemm_error(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(v));
  if (reset) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_tc_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace aideen

#ifdef AIDEEN_TC_PROF
extern "C" int aideen_debug_tc_prof(unsigned long long *out, int n, int reset) {
  if (out && cudaMemcpyFromSymbol(out, aideen::g_tc_prof, n * sizeof(unsigned long long)) != cudaSuccess) return 2;
  if (reset) {
    static unsigned long long zeros[4096 * 8];
    cudaMemcpyToSymbol(aideen::g_tc_prof, zeros, sizeof(zeros));
  }
  return 0;
}
#endif
