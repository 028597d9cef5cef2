// Persistent fp32-accurate GEMM on pre-split operands (tcgen05, sm_100a).
//
// Same contract as tc_gemm (kernels.cuh) for beta in {0, 1}, but every
// operand arrives as two arrays with identical strides: x_hi (x with the low
// 13 mantissa bits cleared, exact in tf32) and x_lo = x - x_hi, written by the
// kernel that produced x.  With no split work left in the GEMM, shared-memory
// bandwidth goes to the tensor cores:
//
//   * one CTA per SM loops over 128 x 256 output tiles (m fastest, so the CTAs
//     running together share the B tile in L2), with split-K units when the
//     output has too few tiles to fill the GPU;
//   * wide mode (no row statistics): 256 x 256 tiles as two M = 128 MMAs that
//     share each B stage (3 stages of 64 KB, both accumulators in the 512 TMEM
//     columns, epilogue not overlapped), which cuts the L2 -> SM traffic of
//     the re-read B slices by half for the long-K and tall-M LM-head GEMMs;
//   * warp 0 / lane 0 streams A_hi, A_lo, B_hi, B_lo K-slices (BK = 16) by TMA
//     into a 4-stage ring (64-byte swizzle for K-major operands, 128-byte
//     swizzle on 32-byte atoms for MN-major ones);
//   * warp 1 / lane 0 issues, per K = 8, three tcgen05.mma kind::tf32
//     (hi*hi + hi*lo + lo*hi) into one of two TMEM accumulators (2 x 256
//     columns), so the epilogue of tile j overlaps the MMAs of tile j+1;
//   * warps 2..5 drain the accumulator (tcgen05.ld, warp w owns TMEM lanes
//     32*(w%4)..+31), scale by alpha, stage 32x32 boxes in 128-byte-swizzled
//     shared memory and write them with bulk tensor stores (beta = 0) or bulk
//     tensor reduce-adds (beta = 1, the add happens in L2).
//
// Every mbarrier wait is bounded; on a timeout the kernel records an error,
// stops issuing, waits for its own copies and MMAs, frees TMEM and returns.
#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.cuh"
#include "tc_common.cuh"

namespace aideen {
namespace {

constexpr int PM = 128, PN = 256, PK = 16, PSTAGES = 4, P_THREADS = 192;
constexpr int PA_BYTES = PM * PK * 4;                     // one A tile (hi or lo): 8 KB
constexpr int PB_BYTES = PN * PK * 4;                     // one B tile: 16 KB
constexpr int PSTAGE_BYTES = 2 * PA_BYTES + 2 * PB_BYTES;  // 48 KB
constexpr int PWSTAGES = 3;                                  // wide mode: 3 stages of
constexpr int PWSTAGE_BYTES = 4 * PA_BYTES + 2 * PB_BYTES;  // 64 KB (2 A sub-tiles)
static_assert(PWSTAGES * PWSTAGE_BYTES == PSTAGES * PSTAGE_BYTES, "ring size shared by both modes");
constexpr int PBOX_BYTES = 32 * 32 * 4;                   // one 32x32 epilogue box
constexpr size_t P_SMEM = 1024 + (size_t)PSTAGES * PSTAGE_BYTES + 8 * PBOX_BYTES + 16 * 8 + 16;

__device__ unsigned int g_split_error;

struct SplitParams {
  int M, N, K;
  int a_kmajor, b_kmajor, a_batched, b_batched;
  int tiles_m, tiles_n, zdim;  // work units = tiles_m * tiles_n * zdim
  int ksplit, kchunk;          // split-K when ksplit > 1 (z = split index, operands unbatched)
  float alpha;
  int reduce_add;
  int wide;  // 256-row tiles (two 128-row sub-tiles sharing the B stage)
  // optional per-(row, 256-column tile) softmax statistics of (C + bias) in
  // base 2: row_stats[row * tiles_n + tile] = (max z, sum exp2(z - max)),
  // z = (alpha * acc + bias[col]) * log2(e)
  const float *row_bias;
  float2 *row_stats;
};

__global__ void __launch_bounds__(P_THREADS, 1)
    tc_split_kernel(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                    const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl,
                    const __grid_constant__ CUtensorMap mC, SplitParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *sm = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *boxes = sm + PSTAGES * PSTAGE_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(boxes + 8 * PBOX_BYTES);
  uint64_t *empty = full + PSTAGES;
  uint64_t *tfull = empty + PSTAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  uint32_t *err = tmem_slot + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int per_z = p.tiles_m * p.tiles_n;
  const int units = per_z * p.zdim;
  const int ktot = (p.K + PK - 1) / PK;
  const int nsub = p.wide ? 2 : 1;                   // 128-row sub-tiles per tile
  const int TM = PM * nsub;                          // tile rows
  const int nstage = p.wide ? PWSTAGES : PSTAGES;
  const int stage_bytes = p.wide ? PWSTAGE_BYTES : PSTAGE_BYTES;
  const int nacc = p.wide ? 1 : 2;                   // TMEM accumulator sets (nsub x 256 columns each)

  if (tid == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(done, 1);
    *err = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2u * PN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // unit -> output tile and K range
  auto coords = [&](int u, int &m0, int &n0, int &z, int &kb0, int &nkb) {
    z = u / per_z;
    const int rem = u - z * per_z;
    n0 = (rem / p.tiles_m) * PN;
    m0 = (rem % p.tiles_m) * TM;
    if (p.ksplit > 1) {
      kb0 = z * p.kchunk;
      nkb = min(p.kchunk, ktot - kb0);
    } else {
      kb0 = 0;
      nkb = ktot;
    }
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int m0, n0, z, kb0, nkb;
        coords(u, m0, n0, z, kb0, nkb);
        const int zo = p.ksplit > 1 ? 0 : z;
        const int za = p.a_batched ? zo : 0, zb = p.b_batched ? zo : 0;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % nstage;
          if (it >= (uint32_t)nstage && !mbar_wait(&empty[s], ((it / nstage) - 1) & 1)) { ok = false; break; }
          if (*(volatile uint32_t *)err) { ok = false; break; }
          const int k0 = (kb0 + kb) * PK;
          unsigned char *st = sm + s * stage_bytes;
          mbar_expect_tx(&full[s], stage_bytes);
          for (int sub = 0; sub < nsub; ++sub) {  // A sub-tile: hi then lo
            unsigned char *sa = st + sub * 2 * PA_BYTES;
            const int ms = m0 + sub * PM;
            if (p.a_kmajor) {
              tma_load_3d(sa, &mAh, &full[s], k0, ms, za);
              tma_load_3d(sa + PA_BYTES, &mAl, &full[s], k0, ms, za);
            } else {
#pragma unroll
              for (int c = 0; c < PM / 32; ++c) {
                tma_load_3d(sa + c * (PK * 128), &mAh, &full[s], ms + 32 * c, k0, za);
                tma_load_3d(sa + PA_BYTES + c * (PK * 128), &mAl, &full[s], ms + 32 * c, k0, za);
              }
            }
          }
          unsigned char *sb = st + nsub * 2 * PA_BYTES;
          if (p.b_kmajor) {
            tma_load_3d(sb, &mBh, &full[s], k0, n0, zb);
            tma_load_3d(sb + PB_BYTES, &mBl, &full[s], k0, n0, zb);
          } else {
#pragma unroll
            for (int c = 0; c < PN / 32; ++c) {
              tma_load_3d(sb + c * (PK * 128), &mBh, &full[s], n0 + 32 * c, k0, zb);
              tma_load_3d(sb + PB_BYTES + c * (PK * 128), &mBl, &full[s], n0 + 32 * c, k0, zb);
            }
          }
        }
      }
      if (!ok) atomicExch(err, 1u);
      // every issued copy must land before the CTA can exit (bounded)
      const uint32_t first = it > (uint32_t)nstage ? it - nstage : 0;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % nstage], (j / nstage) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((p.a_kmajor ? 0u : 1u) << 15) |
                             ((p.b_kmajor ? 0u : 1u) << 16) | ((uint32_t)(PN >> 3) << 17) |
                             ((uint32_t)(PM >> 4) << 24);
      // K-major: 64-byte rows, 8-row atoms (SBO 512), layout 4 (64B swizzle).
      // MN-major: 32-wide MN blocks PK*128 bytes apart (LBO), SBO 512, layout 1.
      const uint32_t lboA = p.a_kmajor ? 16u : PK * 128u, lboB = p.b_kmajor ? 16u : PK * 128u;
      const uint32_t layA = p.a_kmajor ? 4u : 1u, layB = p.b_kmajor ? 4u : 1u;
      uint32_t it = 0;
      int j = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++j) {
        int m0, n0, z, kb0, nkb;
        coords(u, m0, n0, z, kb0, nkb);
        const int a = j % nacc;
        if (j >= nacc && !mbar_wait(&tempty[a], ((j / nacc) - 1) & 1)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % nstage;
          if (!mbar_wait(&full[s], (it / nstage) & 1) || *(volatile uint32_t *)err) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          unsigned char *st = sm + s * stage_bytes;
          unsigned char *sb = st + nsub * 2 * PA_BYTES;
#pragma unroll
          for (int k8 = 0; k8 < PK / 8; ++k8) {
            const uint32_t koffA = p.a_kmajor ? k8 * 32 : k8 * 1024;
            const uint32_t koffB = p.b_kmajor ? k8 * 32 : k8 * 1024;
            const uint64_t bhi = sdesc(sb + koffB, lboB, 512u, layB);
            const uint64_t blo = sdesc(sb + PB_BYTES + koffB, lboB, 512u, layB);
            for (int sub = 0; sub < nsub; ++sub) {
              const uint32_t tacc = tmem + (uint32_t)((a + sub) * PN);
              const uint64_t ahi = sdesc(st + sub * 2 * PA_BYTES + koffA, lboA, 512u, layA);
              const uint64_t alo = sdesc(st + sub * 2 * PA_BYTES + PA_BYTES + koffA, lboA, 512u, layA);
              umma_tf32(tacc, ahi, bhi, idesc, (kb > 0 || k8 > 0) ? 1u : 0u);
              umma_tf32(tacc, ahi, blo, idesc, 1u);
              umma_tf32(tacc, alo, bhi, idesc, 1u);
            }
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[a]);
      }
      if (!ok) atomicExch(err, 1u);
      umma_commit(done);
      mbar_wait(done, 0);  // every MMA issued by this CTA has completed
    }
  } else {  // ---------------- epilogue (128 threads)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    unsigned char *mybox = boxes + (warp - 2) * 2 * PBOX_BYTES;
    int j = 0, nst = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      int m0, n0, z, kb0, nkb;
      coords(u, m0, n0, z, kb0, nkb);
      const int a = j % nacc;
      if (!mbar_wait(&tfull[a], (j / nacc) & 1) || *(volatile uint32_t *)err) {
        atomicExch(err, 1u);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int sub = 0; sub < nsub; ++sub) {
      const int rowbase = m0 + sub * PM + q * 32;
      float st_m = -INFINITY, st_s = 0.f;  // this lane's row: running softmax statistics
#pragma unroll 1
      for (int c = 0; c < PN / 32; ++c) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((a + sub) * PN + c * 32);
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
        if (sub == nsub - 1 && c == PN / 32 - 1) {  // accumulators fully read: hand them back
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[a]);
        }
        const int col = n0 + c * 32;
        if (p.row_stats) {
          constexpr float kLog2e = 1.4426950408889634f;
          float zc[32];
          float mc = -INFINITY;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            zc[k] = col + k < p.N ? (p.alpha * __uint_as_float(r[k]) + __ldg(p.row_bias + col + k)) * kLog2e
                                  : -INFINITY;
            mc = fmaxf(mc, zc[k]);
          }
          if (mc > -INFINITY) {
            float sc = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) sc += exp2f(zc[k] - mc);
            if (mc > st_m) { st_s = st_s * exp2f(st_m - mc) + sc; st_m = mc; }
            else st_s += sc * exp2f(mc - st_m);
          }
        }
        if (col >= p.N || rowbase >= p.M) continue;  // box entirely outside C
        unsigned char *box = mybox + (nst & 1) * PBOX_BYTES;
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
          if (p.reduce_add) tma_reduce_add_3d(&mC, box, col, rowbase, z);
          else tma_store_3d(&mC, box, col, rowbase, z);
          bulk_commit();
        }
        ++nst;
      }
      if (p.row_stats && rowbase + lane < p.M)
        p.row_stats[(size_t)(rowbase + lane) * p.tiles_n + n0 / PN] = make_float2(st_m, st_s);
      }
    }
    if (lane == 0) bulk_wait<0>();  // stores complete before the CTA's shared memory goes away
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && *(volatile uint32_t *)err) atomicCAS(&g_split_error, 0u, 1u);
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2u * PN));
}

// C = alpha * sum_s ws[s] + beta * C in split order (deterministic).
__global__ void split_reduce_kernel(const float *__restrict__ ws, int splits, int M, int N, float *C,
                                    long ldc, float alpha, float beta) {
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[(size_t)s * total + i];
    const size_t m = i / N, n = i % N;
    float *c = C + m * ldc + n;
    *c = beta != 0.f ? alpha * acc + beta * *c : alpha * acc;
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool tc_split_supported(const GemmArgs &g, const float *A_lo, const float *B_lo) {
  if (g.abias || g.K <= 0 || g.M <= 0 || g.N <= 0) return false;
  if (!(g.beta == 0.f || g.beta == 1.f)) return false;
  if (!aligned16(g.A) || !aligned16(g.B) || !aligned16(A_lo) || !aligned16(B_lo) || !aligned16(g.C))
    return false;
  if ((g.lda | g.ldb | g.ldc | g.strideA | g.strideB | g.strideC) & 3) return false;
  return encode_fn() != nullptr;
}

cudaError_t tc_gemm_split(const GemmArgs &g, const float *A_lo, const float *B_lo, cudaStream_t st,
                          float *ws, size_t ws_floats, int max_ctas, const float *row_bias,
                          float2 *row_stats) {
  if (!tc_split_supported(g, A_lo, B_lo)) return cudaErrorInvalidValue;
  if (row_stats && (g.batch != 1 || !row_bias)) return cudaErrorInvalidValue;
  const bool a_k = !g.transA, b_k = g.transB;
  const bool a_b = g.strideA != 0 && g.batch > 1, b_b = g.strideB != 0 && g.batch > 1;
  CUtensorMap mah, mal, mbh, mbl, mc;
  bool ok = true;
  if (a_k) {  // dims: k (contiguous), m, batch
    ok = ok && make_map_sw(&mah, g.A, g.K, g.M, a_b ? g.batch : 1, g.lda, g.strideA, PK, PM, CU_TENSOR_MAP_SWIZZLE_64B);
    ok = ok && make_map_sw(&mal, A_lo, g.K, g.M, a_b ? g.batch : 1, g.lda, g.strideA, PK, PM, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {    // dims: m (contiguous), k, batch
    ok = ok && make_map_sw(&mah, g.A, g.M, g.K, a_b ? g.batch : 1, g.lda, g.strideA, 32, PK,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    ok = ok && make_map_sw(&mal, A_lo, g.M, g.K, a_b ? g.batch : 1, g.lda, g.strideA, 32, PK,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  }
  if (b_k) {  // B stored [n][k]
    ok = ok && make_map_sw(&mbh, g.B, g.K, g.N, b_b ? g.batch : 1, g.ldb, g.strideB, PK, PN, CU_TENSOR_MAP_SWIZZLE_64B);
    ok = ok && make_map_sw(&mbl, B_lo, g.K, g.N, b_b ? g.batch : 1, g.ldb, g.strideB, PK, PN, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {    // B stored [k][n]
    ok = ok && make_map_sw(&mbh, g.B, g.N, g.K, b_b ? g.batch : 1, g.ldb, g.strideB, 32, PK,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    ok = ok && make_map_sw(&mbl, B_lo, g.N, g.K, b_b ? g.batch : 1, g.ldb, g.strideB, 32, PK,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  }
  if (!ok) return cudaErrorInvalidValue;
  SplitParams p{};
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.a_kmajor = a_k; p.b_kmajor = b_k; p.a_batched = a_b; p.b_batched = b_b;
  // wide tiles for the GEMMs without row statistics (AIDEEN_SPLIT_NARROW forces 128-row tiles)
  // (the logits GEMM with row statistics keeps 128-row tiles: its short K makes
  // the overlapped epilogue worth more than the saved B traffic, measured)
  p.wide = (!row_stats && g.M > PM && !getenv("AIDEEN_SPLIT_NARROW")) ? 1 : 0;
  p.tiles_m = (g.M + PM * (1 + p.wide) - 1) / (PM * (1 + p.wide));
  p.tiles_n = (g.N + PN - 1) / PN;
  p.zdim = g.batch;
  p.ksplit = 1; p.kchunk = 0;
  p.alpha = g.alpha;
  p.reduce_add = g.beta == 1.f ? 1 : 0;
  p.row_bias = row_bias;
  p.row_stats = row_stats;
  const int nsm = max_ctas > 0 && max_ctas < sm_count() ? max_ctas : sm_count();
  const int tiles = p.tiles_m * p.tiles_n;
  const int kblocks = (g.K + PK - 1) / PK;
  float *Cmap = g.C;
  long cld = g.ldc, cstride = g.strideC;
  int cz = g.batch;
  // Split K when the output has too few tiles to keep every SM busy: pick the
  // split count (<= 64, within the workspace) that minimises the per-CTA share
  // of K blocks plus the partial sums' round trip (about 1.6e-6 K-block times
  // per output element and split: written once, read once by the reduction).
  if (ws && g.batch == 1 && tiles < nsm && kblocks >= 128 && !row_stats) {
    int best = 1;
    double best_cost = (double)kblocks;  // one unit of all K blocks per CTA
    const double per_split = 1.6e-6 * (double)g.M * g.N * (p.wide ? 0.5 : 1.0);
    for (int s = 2; s <= 64; ++s) {
      const int chunk = (kblocks + s - 1) / s;
      const int splits = (kblocks + chunk - 1) / chunk;
      const int rounds = (tiles * splits + nsm - 1) / nsm;
      const double cost = (double)rounds * chunk + per_split * splits;
      if ((size_t)splits * g.M * g.N <= ws_floats && cost < best_cost) { best_cost = cost; best = s; }
    }
    if (best > 1) {
      const int chunk = (kblocks + best - 1) / best;
      p.ksplit = (kblocks + chunk - 1) / chunk;
      p.kchunk = chunk;
      p.zdim = p.ksplit;
      p.alpha = 1.f;
      p.reduce_add = 0;
      Cmap = ws; cld = g.N; cstride = (long)g.M * g.N; cz = p.ksplit;
    }
  }
  if (!make_map_sw(&mc, Cmap, g.N, g.M, cz, cld, cstride, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const int units = tiles * p.zdim;
  const int grid = units < nsm ? units : nsm;
  cudaError_t e = cudaFuncSetAttribute(tc_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P_SMEM);
  if (e != cudaSuccess) return e;
  tc_split_kernel<<<grid, P_THREADS, P_SMEM, st>>>(mah, mal, mbh, mbl, mc, p);
  e = cudaGetLastError();
  if (e != cudaSuccess || p.ksplit <= 1) return e;
  tc_extra_launches++;
  split_reduce_kernel<<<nsm * 4, 256, 0, st>>>(ws, p.ksplit, g.M, g.N, g.C, g.ldc, g.alpha, g.beta);
  return cudaGetLastError();
}

unsigned int tc_split_error(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_split_error, sizeof(v));
  if (reset) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_split_error, &z, sizeof(z));
  }
  return v;
}

// x -> (hi, lo): hi = x with the low 13 mantissa bits cleared, lo = x - hi.
__global__ void split_hilo_kernel(const float4 *__restrict__ x, float4 *__restrict__ hi,
                                  float4 *__restrict__ lo, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    float4 h;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
    hi[i] = h;
    lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
  }
}

cudaError_t launch_split_hilo(const float *x, float *hi, float *lo, size_t n, cudaStream_t st) {
  if (n % 4) return cudaErrorInvalidValue;
  const size_t n4 = n / 4;
  if (!n4) return cudaSuccess;
  size_t blocks = (n4 + 255) / 256;
  if (blocks > (size_t)sm_count() * 16) blocks = (size_t)sm_count() * 16;
  split_hilo_kernel<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(x),
                                                       reinterpret_cast<float4 *>(hi),
                                                       reinterpret_cast<float4 *>(lo), n4);
  return cudaGetLastError();
}

// out[c][r] = split(x[r][c]) for an R x C row-major x (row stride ldx), into
// hiT / loT with row stride ldt; 32 x 32 tiles through shared memory.
__global__ void transpose_split_kernel(const float *__restrict__ x, int R, int C, long ldx,
                                       float *__restrict__ hiT, float *__restrict__ loT, long ldt) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < R && c < C) ? x[(size_t)r * ldx + c] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + tx;
    if (c < C && r < R) {
      const float v = tile[tx][i];
      const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
      hiT[(size_t)c * ldt + r] = h;
      loT[(size_t)c * ldt + r] = v - h;
    }
  }
}

cudaError_t launch_transpose_split(const float *x, int R, int C, long ldx, float *hiT, float *loT, long ldt,
                                   cudaStream_t st) {
  if (R <= 0 || C <= 0) return cudaSuccess;
  transpose_split_kernel<<<dim3((C + 31) / 32, (R + 31) / 32), 256, 0, st>>>(x, R, C, ldx, hiT, loT, ldt);
  return cudaGetLastError();
}

}  // namespace aideen
