// Strided-batched fp32 GEMM on CUDA cores (exact fp32 FMA accumulation).
//
// The fallback for operand shapes the tcgen05 kernels cannot describe with
// TMA (strides or extents that are not 16-byte multiples); the hot path's
// shapes never take it.  Also the comparator of the tensor-core GEMM
// self-test (aideen_gemm_selftest).
#include "kernels.cuh"

namespace aideen {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;  // 256 threads, 4x4 per thread

__global__ void __launch_bounds__(256) gemm_kernel(GemmArgs g) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int b = blockIdx.z;
  const float *A = g.A + (long)b * g.strideA;
  const float *B = g.B + (long)b * g.strideB;
  float *C = g.C + (long)b * g.strideC;
  const float *ab = g.abias ? g.abias + (long)b * g.strideAbias : nullptr;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  float acc[TM][TN] = {};
  for (int k0 = 0; k0 < g.K; k0 += BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      int mm, kk;
      if (g.transA) { kk = e / BM; mm = e % BM; }   // coalesced along m
      else { mm = e / BK; kk = e % BK; }            // coalesced along k
      const int m = m0 + mm, k = k0 + kk;
      float val = 0.f;
      if (m < g.M && k < g.K) {
        val = g.transA ? A[(long)k * g.lda + m] : A[(long)m * g.lda + k];
        if (ab) val += ab[g.transA ? m : k];
      }
      As[kk][mm] = val;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256;
      int nn, kk;
      if (g.transB) { nn = e / BK; kk = e % BK; }
      else { kk = e / BN; nn = e % BN; }
      const int n = n0 + nn, k = k0 + kk;
      float val = 0.f;
      if (n < g.N && k < g.K) val = g.transB ? B[(long)n * g.ldb + k] : B[(long)k * g.ldb + n];
      Bs[kk][nn] = val;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], bb[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < TN; ++j) bb[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n >= g.N) continue;
      float *c = C + (long)m * g.ldc +
                 (g.col_group > 0 ? (long)(n / g.col_group) * g.group_stride + n % g.col_group : n);
      float r = g.alpha * acc[i][j];
      if (g.beta != 0.f) r += g.beta * *c;
      *c = r;
    }
  }
}

}  // namespace

cudaError_t gemm_f32(const GemmArgs &g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
  dim3 grid((g.N + BN - 1) / BN, (g.M + BM - 1) / BM, g.batch);
  gemm_kernel<<<grid, 256, 0, s>>>(g);
  return cudaGetLastError();
}

}  // namespace aideen
