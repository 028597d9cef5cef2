// fp32-accurate GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[b] = alpha * opA(A[b]) * opB(B[b]) + beta * C[b], row-major, the same
// contract as gemm_f32 (kernels.cuh).  One CTA computes a 128 x BN tile:
//
//   * TMA (cp.async.bulk.tensor, no multicast) brings fp32 tiles of A and B
//     into 128-byte-swizzled shared memory, BK = 32 along K per stage;
//   * all threads split each staged value x into x_hi = x with the low 13
//     mantissa bits cleared (exactly representable in tf32) and
//     x_lo = x - x_hi, in the same swizzled layout;
//   * one thread issues, per K=8 step, three tcgen05.mma kind::tf32
//     (hi*hi + hi*lo + lo*hi) accumulating in TMEM (fp32), then
//     tcgen05.commit releases the stage to the TMA producer;
//   * the epilogue reads the accumulator with tcgen05.ld (warp w owns TMEM
//     lanes 32w..32w+31 = tile rows) and applies alpha/beta.
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

constexpr int BM = 128, BK = 32, STAGES = 3, TC_THREADS = 192;

__device__ unsigned int g_tc_error;  // first error code seen by any tcgemm CTA

// x -> tf32 in place, rounded to nearest (ties to even) instead of the
// truncation the tensor core applies to fp32 bit patterns.
__device__ __forceinline__ uint32_t tf32_rn(uint32_t u) {
  return (u + 0x0FFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
}
__device__ __forceinline__ void round1(float4 *raw) {
  float4 v = *raw;
  v.x = __uint_as_float(tf32_rn(__float_as_uint(v.x)));
  v.y = __uint_as_float(tf32_rn(__float_as_uint(v.y)));
  v.z = __uint_as_float(tf32_rn(__float_as_uint(v.z)));
  v.w = __uint_as_float(tf32_rn(__float_as_uint(v.w)));
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
  int single;                // 1: one TF32 product per term (operands rounded to tf32)
};

// Warp roles (192 threads): warp 0 lane 0 = TMA producer, warp 1 = TMEM
// owner + MMA issuer (lane 0), warps 2..5 = hi/lo splitters and epilogue
// (warp w reads TMEM lanes 32*(w%4)..+31, so the four cover all 128 rows).
// Per stage s: full[s] (TMA landed) -> conv[s] (split done, 4 warp arrivals)
// -> empty[s] (MMAs done, tcgen05.commit) -> producer refills.
constexpr int BOX_BYTES = 32 * 32 * 4;  // one 32x32 fp32 epilogue box

template <int BN>
__global__ void __launch_bounds__(TC_THREADS) tcgemm_kernel(const __grid_constant__ CUtensorMap mapA,
                                                            const __grid_constant__ CUtensorMap mapB,
                                                            const __grid_constant__ CUtensorMap mapC,
                                                            TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
  constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  unsigned char *boxes = sm + STAGES * STAGE_BYTES;  // 4 epilogue warps x 2 boxes
  uint64_t *full = reinterpret_cast<uint64_t *>(boxes + 8 * BOX_BYTES);
  uint64_t *conv = full + STAGES;
  uint64_t *empty = conv + STAGES;
  uint64_t *done = empty + STAGES;
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

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *err = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  auto stage_ptr = [&](int s, int which) -> unsigned char * {
    unsigned char *base = sm + s * STAGE_BYTES;  // 0 A hi, 1 A lo, 2 B hi, 3 B lo
    return which == 0 ? base : which == 1 ? base + A_BYTES : which == 2 ? base + 2 * A_BYTES
                                                                        : base + 2 * A_BYTES + B_BYTES;
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < kblocks && ok; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1)) { ok = false; break; }
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
      // every issued copy must land before the CTA can exit (bounded)
      for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; ++kb)
        mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1);
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
        const int s = kb % STAGES;
        if (!mbar_wait(&conv[s], (kb / STAGES) & 1) || *(volatile uint32_t *)err) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int k8 = 0; k8 < BK / 8; ++k8) {
          // K-major: +32 B along the swizzled row; MN-major: +1024 B (8 K rows)
          const uint32_t koffA = p.a_kmajor ? k8 * 32 : k8 * 1024;
          const uint32_t koffB = p.b_kmajor ? k8 * 32 : k8 * 1024;
          const uint64_t ahi = sdesc(stage_ptr(s, 0) + koffA, lboA, sboA, layA);
          const uint64_t alo = sdesc(stage_ptr(s, 1) + koffA, lboA, sboA, layA);
          const uint64_t bhi = sdesc(stage_ptr(s, 2) + koffB, lboB, sboB, layB);
          const uint64_t blo = sdesc(stage_ptr(s, 3) + koffB, lboB, sboB, layB);
          umma_tf32(tmem, ahi, bhi, idesc, (kb > 0 || k8 > 0) ? 1u : 0u);
          if (!p.single) {
            umma_tf32(tmem, ahi, blo, idesc, 1u);
            umma_tf32(tmem, alo, bhi, idesc, 1u);
          }
        }
        umma_commit(&empty[s]);
      }
      if (!ok) atomicExch(err, 1u);
      umma_commit(done);  // arrives once every MMA issued so far has completed
    }
  } else {  // ---------------- splitters (128 threads) + epilogue
    const int ct = tid - 64;
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&full[s], (kb / STAGES) & 1)) { atomicExch(err, 1u); break; }
      if (*(volatile uint32_t *)err) break;
      float4 *ra = reinterpret_cast<float4 *>(stage_ptr(s, 0));
      float4 *la = reinterpret_cast<float4 *>(stage_ptr(s, 1));
      float4 *rb = reinterpret_cast<float4 *>(stage_ptr(s, 2));
      float4 *lb = reinterpret_cast<float4 *>(stage_ptr(s, 3));
      if (p.single) {
#pragma unroll 4
        for (int i = ct; i < A_BYTES / 16; i += 128) round1(ra + i);
#pragma unroll 4
        for (int i = ct; i < B_BYTES / 16; i += 128) round1(rb + i);
      } else {
#pragma unroll 4
        for (int i = ct; i < A_BYTES / 16; i += 128) split1(ra + i, la + i);
#pragma unroll 4
        for (int i = ct; i < B_BYTES / 16; i += 128) split1(rb + i, lb + i);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
    const bool ok = mbar_wait(done, 0) && !*(volatile uint32_t *)err;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && p.tma_epi) {
      const int q = warp & 3;  // TMEM lane quadrant this warp may access
      const int rowbase = m0 + q * 32;
      unsigned char *mybox = boxes + (warp - 2) * 2 * BOX_BYTES;
      int nst = 0;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
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
      const int row = m0 + q * 32 + lane;
      float *crow = p.C + (long)bz * p.strideC + (long)row * p.ldc;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN));
}

// ---------------------------------------------------------------- host side
// 3-D fp32 map: dim0 contiguous (extent e0), dim1 stride s1 elements, dim2 stride s2.
bool make_map(CUtensorMap *m, const float *base, uint64_t e0, uint64_t e1, uint64_t e2, uint64_t s1,
              uint64_t s2, uint32_t box0, uint32_t box1, bool kmajor) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {e0, e1, e2 ? e2 : 1};
  const cuuint64_t strides[2] = {s1 * 4, (s2 ? s2 : s1 * e1) * 4};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE,
            kmajor ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
size_t tc_smem() {
  return 1024 + STAGES * (size_t)(2 * BM * BK * 4 + 2 * BN * BK * 4) + 8 * BOX_BYTES + 8 * (3 * STAGES + 1) +
         16;
}

}  // namespace

bool tc_gemm_supported(const GemmArgs &g) {
  if (g.abias) return false;
  if (g.K <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.B)) & 15) return false;
  if ((g.lda | g.ldb | g.strideA | g.strideB) & 3) return false;
  return encode_fn() != nullptr;
}

namespace {
// C[b] = alpha * sum_s ws[b][s] + beta * C[b], summed in split order (deterministic).
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, int splits, int batch, int M, int N,
                                     float *C, long ldc, long strideC, float alpha, float beta) {
  const size_t mn = (size_t)M * N, total = mn * batch;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t bb = i / mn, r = i % mn;
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[(bb * splits + s) * mn + r];
    const size_t m = r / N, n = r % N;
    float *c = C + bb * strideC + m * ldc + n;
    *c = beta != 0.f ? alpha * acc + beta * *c : alpha * acc;
  }
}
}  // namespace

cudaError_t tc_gemm(const GemmArgs &g, cudaStream_t st, float *ws, size_t ws_floats) {
  // A: K-major when not transposed (row m contiguous along k).
  const bool a_k = !g.transA, b_k = g.transB;
  CUtensorMap ma, mb;
  const bool a_batched = g.strideA != 0 && g.batch > 1;
  bool ok;
  if (a_k)  // dims: k (contiguous), m, batch
    ok = make_map(&ma, g.A, g.K, g.M, a_batched ? g.batch : 1, g.lda, g.strideA, BK, BM, true);
  else      // dims: m (contiguous), k, batch
    ok = make_map(&ma, g.A, g.M, g.K, a_batched ? g.batch : 1, g.lda, g.strideA, 32, BK, false);
  if (!ok) return cudaErrorInvalidValue;
  const int BN = g.N >= 128 ? 128 : 32;
  const bool b_batched = g.strideB != 0 && g.batch > 1;
  if (b_k)  // B stored [n][k]
    ok = make_map(&mb, g.B, g.K, g.N, b_batched ? g.batch : 1, g.ldb, g.strideB, BK, BN, true);
  else      // B stored [k][n]
    ok = make_map(&mb, g.B, g.N, g.K, b_batched ? g.batch : 1, g.ldb, g.strideB, 32, BK, false);
  if (!ok) return cudaErrorInvalidValue;
  TcParams p{g.M, g.N, g.K, a_k, b_k, g.C, g.ldc, g.strideC, g.alpha, g.beta, a_batched ? 1 : 0,
             b_batched ? 1 : 0, 1, 0, 0, g.tf32 ? 1 : 0};
  const int tiles_n = (g.N + BN - 1) / BN, tiles_m = (g.M + BM - 1) / BM;
  const int tiles = tiles_n * tiles_m * g.batch;
  const int kblocks = (g.K + BK - 1) / BK;
  int zdim = g.batch;
  // Split K when the output (all batches) has too few tiles to fill the GPU
  // and K is long enough; the partial sums go to the workspace.
  if (ws && tiles < 148 && kblocks >= 64) {
    int splits = (2 * 148 + tiles - 1) / tiles;
    if (splits > 16) splits = 16;
    if (splits > kblocks / 4) splits = kblocks / 4;
    const int chunk = (kblocks + splits - 1) / splits;
    splits = (kblocks + chunk - 1) / chunk;
    if ((size_t)splits * g.batch * g.M * g.N <= ws_floats && splits > 1) {
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
  // Coalesced epilogue through bulk tensor stores when C allows a tensor map
  // (16-byte aligned rows) and beta is 0 or 1 (reduce-add in L2).
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  if ((p.beta == 0.f || p.beta == 1.f) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
      ((p.ldc | p.strideC) & 3) == 0 &&
      make_map_sw(&mc, p.C, g.N, g.M, zdim, p.ldc, p.strideC, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
    p.tma_epi = 1;
  dim3 grid(tiles_n, tiles_m, zdim);
  if (BN == 128) {
    const size_t smem = tc_smem<128>();
    cudaFuncSetAttribute(tcgemm_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tcgemm_kernel<128><<<grid, TC_THREADS, smem, st>>>(ma, mb, mc, p);
  } else {
    const size_t smem = tc_smem<32>();
    cudaFuncSetAttribute(tcgemm_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    tcgemm_kernel<32><<<grid, TC_THREADS, smem, st>>>(ma, mb, mc, p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.ksplit <= 1) return e;
  tc_extra_launches++;
  splitk_reduce_kernel<<<148 * 4, 256, 0, st>>>(ws, p.ksplit, g.batch, g.M, g.N, g.C, g.ldc,
                                                g.batch > 1 ? g.strideC : 0, g.alpha, g.beta);
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
