// Shared device helpers: warp/block reductions and small vector ops.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace aideen {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Type-II Anderson mixing weights from the Gram of n_res (2 or 3) pseudo-
// residuals, g6 = <d0,d0>, <d0,d1>, <d0,d2>, <d1,d1>, <d1,d2>, <d2,d2>:
// Tikhonov term 1e-4*trace, Cramer solve with a floored determinant, clamp to
// [-2, 3] and renormalisation to sum 1 with a most-recent fallback
// (staged_adjoint_picard_clean.wgsl:1075-1124).
__device__ __forceinline__ void anderson_solve(const float (&g6)[6], int n_res, float &b0, float &b1,
                                               float &b2) {
  b2 = 0.f;
  if (n_res == 2) {
    float g00 = g6[0], g01 = g6[1], g10 = g6[1], g11 = g6[3];
    const float reg = fmaxf(1e-8f, 1e-4f * (fabsf(g00) + fabsf(g11)));
    g00 += reg;
    g11 += reg;
    const float det = g00 * g11 - g01 * g10;
    const float sdet = det < 0.f ? fminf(det, -1e-10f) : fmaxf(det, 1e-10f);
    b0 = (g11 - g01) / sdet;
    b1 = (g00 - g10) / sdet;
  } else {
    float g00 = g6[0], g01 = g6[1], g02 = g6[2];
    float g10 = g6[1], g11 = g6[3], g12 = g6[4];
    float g20 = g6[2], g21 = g6[4], g22 = g6[5];
    const float reg = fmaxf(1e-8f, 1e-4f * (fabsf(g00) + fabsf(g11) + fabsf(g22)));
    g00 += reg;
    g11 += reg;
    g22 += reg;
    const float det = g00 * (g11 * g22 - g12 * g21) - g01 * (g10 * g22 - g12 * g20) +
                      g02 * (g10 * g21 - g11 * g20);
    const float sdet = det < 0.f ? fminf(det, -1e-8f) : fmaxf(det, 1e-8f);
    b0 = ((g11 * g22 - g12 * g21) - g01 * (g22 - g12) + g02 * (g21 - g11)) / sdet;
    b1 = (g00 * (g22 - g12) - (g10 * g22 - g12 * g20) + g02 * (g10 - g20)) / sdet;
    b2 = (g00 * (g11 - g21) - g01 * (g10 - g20) + (g10 * g21 - g11 * g20)) / sdet;
  }
  b0 = fminf(fmaxf(b0, -2.f), 3.f);
  b1 = fminf(fmaxf(b1, -2.f), 3.f);
  if (n_res == 3) b2 = fminf(fmaxf(b2, -2.f), 3.f);
  const float ssum = b0 + b1 + (n_res == 3 ? b2 : 0.f);
  if (fabsf(ssum) < 1e-6f) {
    b0 = 1.f; b1 = 0.f; b2 = 0.f;
  } else {
    b0 /= ssum; b1 /= ssum; b2 = n_res == 3 ? b2 / ssum : 0.f;
  }
}

// Block-wide sums of K (<= 8) values per thread; every thread receives the
// totals.  `red` is shared scratch of 2 * 8 * 32 floats.  Consecutive calls
// alternate halves of `red`, so one __syncthreads per call suffices: a thread
// reaches call i+2 (same half as call i) only after passing call i+1's
// barrier, which every thread reaches only after reading call i's result.
struct BlockReducer {
  float *red;
  int parity;
  __device__ __forceinline__ explicit BlockReducer(float *r) : red(r), parity(0) {}
  template <int K>
  __device__ __forceinline__ void sum(float (&v)[K]) {
    static_assert(K <= 8, "at most 8 values per reduction");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    float *buf = red + parity * 8 * 32;
    parity ^= 1;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float x = warp_sum(v[k]);
      if (lane == 0) buf[k * 32 + warp] = x;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float s = 0.f;
      for (int w = 0; w < nw; ++w) s += buf[k * 32 + w];
      v[k] = s;
    }
  }
};

// Same protocol for doubles; `red` holds 2 * 8 * 32 doubles.
// Block sum with the warp count known at compile time (blockDim = 32 * NW,
// NW a multiple of 4): the warp partials come back as NW/4 float4 loads.
template <int NW, int K>
__device__ __forceinline__ void block_sum_static(float *red, int &parity, float (&v)[K]) {
  static_assert(NW % 4 == 0 && NW <= 32 && K <= 8, "static block sum shape");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *buf = red + parity * 8 * 32;
  parity ^= 1;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float x = warp_sum(v[k]);
    if (lane == 0) buf[k * 32 + warp] = x;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) {
    float4 acc = reinterpret_cast<const float4 *>(buf + k * 32)[0];
#pragma unroll
    for (int w = 4; w < NW; w += 4) {
      const float4 q = reinterpret_cast<const float4 *>(buf + k * 32 + w)[0];
      acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
    }
    v[k] = (acc.x + acc.y) + (acc.z + acc.w);
  }
}

struct BlockReducerD {
  double *red;
  int parity;
  __device__ __forceinline__ explicit BlockReducerD(double *r) : red(r), parity(0) {}
  template <int K>
  __device__ __forceinline__ void sum(double (&v)[K]) {
    static_assert(K <= 8, "at most 8 values per reduction");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    double *buf = red + parity * 8 * 32;
    parity ^= 1;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      double x = v[k];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) buf[k * 32 + warp] = x;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < K; ++k) {
      double s = 0.0;
      for (int w = 0; w < nw; ++w) s += buf[k * 32 + w];
      v[k] = s;
    }
  }
};

// Reduce 32 per-lane partial vectors p[0..31] across a warp so that lane r
// ends up holding the sum over lanes of p[r] (31 shuffles in total).  At each
// step a lane keeps one half of its window and ships the other half to its
// partner (lane ^ off), which keeps the mirror half.
__device__ __forceinline__ float warp_transpose_reduce32(float (&p)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? p[i] : p[i + off];
      const float keep = upper ? p[i + off] : p[i];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return p[0];
}

__device__ __forceinline__ float4 f4(float a) { return make_float4(a, a, a, a); }
__device__ __forceinline__ float4 operator+(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 operator-(float4 a, float4 b) {
  return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w);
}
__device__ __forceinline__ float4 operator*(float4 a, float4 b) {
  return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}
__device__ __forceinline__ float4 operator*(float s, float4 a) {
  return make_float4(s * a.x, s * a.y, s * a.z, s * a.w);
}
__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}
__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
__device__ __forceinline__ float4 tanh4(float4 a) {
  return make_float4(tanhf(a.x), tanhf(a.y), tanhf(a.z), tanhf(a.w));
}
__device__ __forceinline__ bool finite4(float4 a) {
  return isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w);
}

// Packed fp32 FMA (sm_100 FFMA2: two lanes of fp32 per instruction issue),
// each component rounded like fmaf.  AIDEEN_NO_FFMA2 builds the scalar form.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
#ifdef AIDEEN_NO_FFMA2
  return make_float2(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
#else
  return __ffma2_rn(a, b, c);
#endif
}
__device__ __forceinline__ float4 fma4(float4 a, float4 b, float4 c) {
  const float2 lo = fma2(make_float2(a.x, a.y), make_float2(b.x, b.y), make_float2(c.x, c.y));
  const float2 hi = fma2(make_float2(a.z, a.w), make_float2(b.z, b.w), make_float2(c.z, c.w));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
// acc + a * b accumulated per component (a float4 dot product's partial sums)
__device__ __forceinline__ float4 dot4_acc(float4 acc, float4 a, float4 b) { return fma4(a, b, acc); }
__device__ __forceinline__ float hsum4(float4 a) { return (a.x + a.y) + (a.z + a.w); }

// float2 counterparts (the Picard kernel's per-thread vectors)
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 operator+(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 operator-(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 operator*(float2 a, float2 b) { return make_float2(a.x * b.x, a.y * b.y); }
__device__ __forceinline__ float2 operator*(float s, float2 a) { return make_float2(s * a.x, s * a.y); }
__device__ __forceinline__ float dot2(float2 a, float2 b) { return a.x * b.x + a.y * b.y; }
__device__ __forceinline__ float2 ld2(const float *p) { return *reinterpret_cast<const float2 *>(p); }
__device__ __forceinline__ void st2(float *p, float2 v) { *reinterpret_cast<float2 *>(p) = v; }
__device__ __forceinline__ float2 tanh2(float2 a) { return make_float2(tanhf(a.x), tanhf(a.y)); }

}  // namespace aideen
