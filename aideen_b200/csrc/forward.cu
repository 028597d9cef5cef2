// Forward DEQ solve of the AIDEEN slot block on sm_100a.
//
//   embed_gather       tokens -> S_in          (embedding_train.wgsl:35, gather only)
//   attn_softmax       iter-0 slot attention softmax / mix / RMS-normalise
//                      (deq_slot_attn_unified_clean.wgsl:395-450)
//   attn_scale         attention RMS scale + injection A = attn*scale (:452-495)
//   picard             persistent token-serial Picard solve, one CTA per
//                      (sequence, slot); with FPM memory the h CTAs of one
//                      sequence form a thread-block cluster and exchange the
//                      per-slot memory and its read keys through distributed
//                      shared memory (:700-2300)
//   pool_rmsnorm       H_pooled = mean over slots (deq_forward_pool.wgsl:32-65)
//                      + the LM-head RMSNorm input (lm_train.wgsl:100-125)
//   solve_stats        iteration / non-finite counters
#include <cooperative_groups.h>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace aideen {

#ifdef AIDEEN_PICARD_PROF
// Phase timer of the Picard kernel (profiling builds only): cycles per CTA in
// [0] token sync, [1] Picard iterations, [2] FPM read, [3] h* stores, [4] FPM write.
__device__ unsigned long long g_picard_prof[1024 * 8];
#define PT(i)                                               \
  {                                                         \
    const long long _n = clock64();                         \
    _pacc[i] += _n - _pt;                                   \
    _pt = _n;                                               \
  }
#else
#define PT(i)
#endif

__global__ void embed_gather_kernel(const int32_t *__restrict__ tok, const float *__restrict__ emb,
                                    float *__restrict__ S, int N, int d, int vocab) {
  const int n = blockIdx.x;
  if (n >= N) return;
  int t = tok[n];
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  for (int j = threadIdx.x * 4; j < d; j += blockDim.x * 4)
    st4(S + (size_t)n * d + j, ld4(emb + (size_t)t * d + j));
}

// One block per token, one warp per slot, lane = head dimension (32).
__global__ void attn_softmax_kernel(AttnArgs a) {
  __shared__ float Ks[16][33], Vs[16][33];
  const int n = blockIdx.x;
  const int s = threadIdx.x >> 5, c = threadIdx.x & 31;
  const int h = a.h, d = a.d;
  const size_t row = ((size_t)n * h + s) * kHeadDim + c;
  const size_t qrow = ((size_t)n * h + s) * a.qkv_ld + c;
  Ks[s][c] = a.Kh[qrow] + a.W[a.off_kb + (size_t)s * d + c];
  Vs[s][c] = a.Vh[qrow];
  const float q = a.Qh[qrow] + a.W[a.off_qb + (size_t)s * d + c];
  __syncthreads();
  const float gain = 2.0f * rsqrtf((float)kHeadDim);
  float logit[16];
  float mx = -1e30f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (k < h) {
      float l = warp_sum(q * Ks[k][c]) * gain;
      if (h > 1 && k == s) l = -1e30f;
      logit[k] = l;
      mx = fmaxf(mx, l);
    }
  }
  float se = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < h) { logit[k] = expf(logit[k] - mx); se += logit[k]; }
  se = fmaxf(se, 1e-12f);
  float mix = 0.f, vmean = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < h) {
      logit[k] = logit[k] / se;
      mix += logit[k] * Vs[k][c];
      vmean += Vs[k][c];
    }
  mix -= vmean / (float)h;
  const float r = sqrtf(warp_sum(mix * mix) / (float)kHeadDim + 1e-6f);
  a.nmix[row] = mix / r;
  if (c == 0) {
    a.rmix[(size_t)n * h + s] = r;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k < h) a.alpha[((size_t)n * h + s) * h + k] = logit[k];
  }
}

// One warp per (token, slot): A = attn * max(R,1e-3)/max(rho,1e-6).
__global__ void attn_scale_kernel(AttnArgs a, int rows) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const int d = a.d, s = w % a.h;
  const float *sig = a.signal + (size_t)w * d;
  const float *am = a.amat + (size_t)w * d;
  const float *anc = a.W + a.off_anchor + (size_t)s * d;
  float ss = 0.f, aa = 0.f;
  for (int j = lane * 4; j < d; j += 128) {
    const float4 src = ld4(sig + j) + ld4(anc + j);
    const float4 x = ld4(am + j);
    ss += dot4(src, src);
    aa += dot4(x, x);
  }
  ss = warp_sum(ss);
  aa = warp_sum(aa);
  const float R = sqrtf(ss / d + 1e-6f), rho = sqrtf(aa / d + 1e-6f);
  const float sc = fmaxf(R, 1e-3f) / fmaxf(rho, 1e-6f);
  for (int j = lane * 4; j < d; j += 128) st4(a.A + (size_t)w * d + j, sc * ld4(am + j));
  if (lane == 0) { a.scale[w] = sc; a.rho[w] = rho; a.Rsrc[w] = R; }
}

// ---- Picard element ownership ---------------------------------------------
// The block has d/2 threads; thread t = hf * (d/4) + l (hf = 0, 1) owns the
// float2 at j0 = 4 l + 2 hf.  With d = 512 this pairs warps w and w + 4 on the
// same TMEM lane quadrant (lane l), each using half of the lane's columns.
__device__ __forceinline__ int picard_j0() {
  const int th = blockDim.x >> 1;
  return 4 * (threadIdx.x % th) + 2 * (threadIdx.x / th);
}

// y_q[r] = sum_j Mq[j*32 + r] x[j], r < 32, for Q (1 or 2) matrices sharing x.
// Each thread stages its float2 of x in xs; then lane l of warp w reads rows
// j = 64 w + 4 i + (l >> 3), columns 4 (l & 7)..+3, so one warp load covers
// four whole 128-byte rows (coalesced, conflict-free in shared memory); every
// warp covers 64 rows.  Results land in out[q*32 + r].  Three block barriers.
// SYNC_OUT = false skips the last barrier: for results that only the writing
// warp (warp 0) reads, or that peers read after a cluster barrier.
template <int Q, bool SYNC_OUT = true>
__device__ __forceinline__ void mv_d_to_32(const float *M0, const float *M1, float2 x, int j0, float *xs,
                                           float *out, float *part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  st2(xs + j0, x);
  __syncthreads();
  const int g = lane >> 3, rq = (lane & 7) * 4;
  float4 acc[Q];
#pragma unroll
  for (int q = 0; q < Q; ++q) acc[q] = f4(0.f);
  const int jb = warp * 64 + g;
  if (Q == 1) {  // two accumulator chains for latency
    float4 acc1 = f4(0.f);
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const int j = jb + 4 * i;
      acc[0] = acc[0] + xs[j] * ld4(M0 + (size_t)j * kRank + rq);
      acc1 = acc1 + xs[j + 4] * ld4(M0 + (size_t)(j + 4) * kRank + rq);
    }
    acc[0] = acc[0] + acc1;
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = jb + 4 * i;
      const float xj = xs[j];
      acc[0] = acc[0] + xj * ld4(M0 + (size_t)j * kRank + rq);
      acc[Q - 1] = acc[Q - 1] + xj * ld4(M1 + (size_t)j * kRank + rq);
    }
  }
#pragma unroll
  for (int q = 0; q < Q; ++q) {
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
      acc[q].x += __shfl_xor_sync(0xffffffffu, acc[q].x, o);
      acc[q].y += __shfl_xor_sync(0xffffffffu, acc[q].y, o);
      acc[q].z += __shfl_xor_sync(0xffffffffu, acc[q].z, o);
      acc[q].w += __shfl_xor_sync(0xffffffffu, acc[q].w, o);
    }
    if (g == 0) st4(part + warp * 64 + q * 32 + rq, acc[q]);
  }
  __syncthreads();
  if (threadIdx.x < 32 * Q) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += part[w * 64 + threadIdx.x];
    out[threadIdx.x] = t;
  }
  if (SYNC_OUT) __syncthreads();
}

// Warp partials of out = M . x for x already staged in xs (all of it visible to
// every thread): each warp's 64 rows, reduced over the warp, into part[warp *
// 64 + 0..31].  No block barrier: the caller's next one publishes part.
__device__ __forceinline__ void mv_d_to_32_partials(const float *M0, const float *xs, float *part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, rq = (lane & 7) * 4;
  const int jb = warp * 64 + g;
  float4 acc = f4(0.f), acc1 = f4(0.f);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const int j = jb + 4 * i;
    acc = acc + xs[j] * ld4(M0 + (size_t)j * kRank + rq);
    acc1 = acc1 + xs[j + 4] * ld4(M0 + (size_t)(j + 4) * kRank + rq);
  }
  acc = acc + acc1;
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
  }
  if (g == 0) st4(part + warp * 64 + rq, acc);
}

// Lane l of the calling warp: sum over the NW warps of part[w * 64 + l].
template <int NW>
__device__ __forceinline__ float sum_partials32(const float *part) {
  const int lane = threadIdx.x & 31;
  const int nw = NW > 0 ? NW : (int)(blockDim.x >> 5);
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < (NW > 0 ? NW : 32); ++w) {
    if (NW == 0 && w >= nw) break;
    t += part[w * 64 + lane];
  }
  return t;
}

// Two 32->d products in one pass: ya = Ma . ina, yb = Mb . inb (thread's 2 outputs).
__device__ __forceinline__ void mv2_32_to_d(const float *Ma, const float *ina, const float *Mb,
                                            const float *inb, int d, int j0, float2 &ya, float2 &yb) {
  float2 a = f2(0.f), b = f2(0.f);
#pragma unroll
  for (int r = 0; r < kRank; ++r) {
    a = a + ina[r] * ld2(Ma + (size_t)r * d + j0);
    b = b + inb[r] * ld2(Mb + (size_t)r * d + j0);
  }
  ya = a;
  yb = b;
}

// ---- tensor-memory staging of rank-32 FPM matrices (d = 512) ---------------
// TMEM lane l holds the rows / outputs of both threads owning l; the thread
// with half hf uses the lane's columns [64 hf, 64 hf + 64) of every matrix
// (128 columns per matrix).  A d->32 matrix M[j][r]: column 64 hf + 32 k + r
// holds M[j0 + k][r].  A 32->d matrix M[r][o]: column 64 hf + 32 c + 2 rr + k
// holds M[16 c + rr][j0 + k].  Loads complete at tmem_wait (which also orders
// the destination registers after the wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Copy this thread's part of a rank-32 matrix from global memory into TMEM
// (layouts above; tcol already includes the 64 hf column offset).
__device__ __forceinline__ void tmem_stage(uint32_t tcol, const float *M, int d, int j0, bool rows_d) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t v[32];
    if (rows_d) {
      const float *row = M + (size_t)(j0 + c) * kRank;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 x = ld4(row + 4 * i);
        v[4 * i] = __float_as_uint(x.x); v[4 * i + 1] = __float_as_uint(x.y);
        v[4 * i + 2] = __float_as_uint(x.z); v[4 * i + 3] = __float_as_uint(x.w);
      }
    } else {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) {
        const float2 x = ld2(M + (size_t)(16 * c + rr) * d + j0);
        v[2 * rr] = __float_as_uint(x.x);
        v[2 * rr + 1] = __float_as_uint(x.y);
      }
    }
    tmem_st32(tcol + 32 * c, v);
  }
}

// out[0..32) = Ms . x with Ms in shared memory (mv_d_to_32 layout) and
// out[32..64) = Mt . x with Mt (d->32) in TMEM at lane-relative column tcol.
__device__ __forceinline__ void mv_d_to_32_smem_tmem(const float *Ms, uint32_t tcol, float2 x, int j0,
                                                     float *xs, float *out, float *part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  st2(xs + j0, x);
  __syncthreads();
  const int g = lane >> 3, rq = (lane & 7) * 4;
  float4 acc = f4(0.f), acc1 = f4(0.f);  // two chains for latency
  const int jb = warp * 64 + g;
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    const int j = jb + 4 * i;
    acc = acc + xs[j] * ld4(Ms + (size_t)j * kRank + rq);
    acc1 = acc1 + xs[j + 4] * ld4(Ms + (size_t)(j + 4) * kRank + rq);
  }
  acc = acc + acc1;
#pragma unroll
  for (int o = 8; o <= 16; o <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
  }
  if (g == 0) st4(part + warp * 64 + rq, acc);
  float p[32];
  {
    uint32_t w0[32];
    tmem_ld32(tcol, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) p[r] = x.x * __uint_as_float(w0[r]);
    tmem_ld32(tcol + 32, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) p[r] += x.y * __uint_as_float(w0[r]);
  }
  part[warp * 64 + 32 + lane] = warp_transpose_reduce32(p);
  __syncthreads();
  if (threadIdx.x < 64) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += part[w * 64 + threadIdx.x];
    out[threadIdx.x] = t;
  }
  __syncthreads();
}

// ya = Ma . ina, yb = Mb . inb for two 32->d matrices in TMEM (thread's 2 outputs).
__device__ __forceinline__ void mv2_32_to_d_tmem(uint32_t ta, const float *ina, uint32_t tb, const float *inb,
                                                 float2 &ya, float2 &yb) {
  float2 a = f2(0.f), b = f2(0.f);
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    uint32_t wa[32], wb[32];
    tmem_ld32(ta + 32 * c, wa);
    tmem_ld32(tb + 32 * c, wb);
    tmem_wait(wa);
    tmem_wait(wb);
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) {
      const float xa = ina[16 * c + rr], xb = inb[16 * c + rr];
      a.x += xa * __uint_as_float(wa[2 * rr]); a.y += xa * __uint_as_float(wa[2 * rr + 1]);
      b.x += xb * __uint_as_float(wb[2 * rr]); b.y += xb * __uint_as_float(wb[2 * rr + 1]);
    }
  }
  ya = a;
  yb = b;
}

// Forward Anderson step (type-II Anderson acceleration in the difference
// form of Walker & Ni, SIAM J. Numer. Anal. 49(4), 2011): with residuals f_i
// of the last n + 1 iterations and D_i = f_i - f_{i+1}, gamma minimises
// |f_0 - sum_i gamma_i D_i|.  q = <D0,D0>, <D0,D1>, <D1,D1>, <D0,f0>, <D1,f0>
// (n = 1 or 2), ridge 1e-3 * trace on the diagonal.  False (plain Picard
// step) for a zero trace or any |gamma_i| > 20.
__device__ __forceinline__ bool anderson_fwd_gamma(const float (&q)[5], int n, float &g0, float &g1) {
  if (n == 1) {
    const float tr = q[0];
    if (!(tr > 0.f)) return false;
    g0 = q[3] / (q[0] + 1e-3f * tr);
    g1 = 0.f;
  } else {
    const float tr = q[0] + q[2];
    if (!(tr > 0.f)) return false;
    const float lam = 1e-3f * tr;
    const float a = q[0] + lam, b = q[1], c = q[2] + lam;
    const float det = a * c - b * b;
    if (!(det > 0.f)) return false;
    const float idet = 1.f / det;
    g0 = (c * q[3] - b * q[4]) * idet;
    g1 = (a * q[4] - b * q[3]) * idet;
  }
  return fmaxf(fabsf(g0), fabsf(g1)) <= 20.f;
}

// out[0..32) = Ma . x, out[32..64) = Mb . x for two d->32 matrices in TMEM.
__device__ __forceinline__ void mv2_d_to_32_tmem(uint32_t ta, uint32_t tb, float2 x, float *out, float *part) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float pa[32], pb[32];
  {
    uint32_t w0[32];
    tmem_ld32(ta, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) pa[r] = x.x * __uint_as_float(w0[r]);
    tmem_ld32(ta + 32, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) pa[r] += x.y * __uint_as_float(w0[r]);
  }
  part[warp * 64 + lane] = warp_transpose_reduce32(pa);
  {
    uint32_t w0[32];
    tmem_ld32(tb, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) pb[r] = x.x * __uint_as_float(w0[r]);
    tmem_ld32(tb + 32, w0);
    tmem_wait(w0);
#pragma unroll
    for (int r = 0; r < 32; ++r) pb[r] += x.y * __uint_as_float(w0[r]);
  }
  part[warp * 64 + 32 + lane] = warp_transpose_reduce32(pb);
  __syncthreads();
  if (threadIdx.x < 64) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += part[w * 64 + threadIdx.x];
    out[threadIdx.x] = t;
  }
  __syncthreads();
}

// ---- inbox exchange of the FPM memory rows and read keys -------------------
__device__ unsigned int g_picard_error;  // a bounded inbox wait gave up (data of that token invalid)

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void inbox_arm(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// Bounded wait for phase `parity`; false if it gave up.
__device__ __forceinline__ bool inbox_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  for (uint32_t i = 0; i < (1u << 24); ++i) {
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
// Copy `bytes` of this CTA's shared memory to the same-layout slot in CTA
// `rank`, completing on that CTA's mbarrier.
__device__ __forceinline__ void push_to(const void *src, const void *dst_local, uint64_t *bar_local,
                                        uint32_t rank, uint32_t bytes) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          cluster_addr(smem_addr(dst_local), rank)),
      "r"(smem_addr(src)), "r"(bytes), "r"(cluster_addr(smem_addr(bar_local), rank))
      : "memory");
}

// (fast reciprocal: ~2 ulp, on the Picard write's dependency chain)
__device__ __forceinline__ float2 sigmoid2(float2 x) {
  return make_float2(__fdividef(1.f, 1.f + __expf(-x.x)), __fdividef(1.f, 1.f + __expf(-x.y)));
}

// Persistent token-serial solve.  blockDim = d/2 (one float2 per thread, see
// picard_j0), grid = B*h, block = b*h + s.  FPM=true requires a cluster of h CTAs.
template <int NW, int K>
__device__ __forceinline__ void bsum(BlockReducer &R, float (&v)[K]) {
  if constexpr (NW > 0) block_sum_static<NW>(R.red, R.parity, v);
  else R.sum(v);
}

// NW > 0: blockDim = 32 * NW fixed at compile time (static block reductions).
// ASSOC (with FPM): the upper h/2 slots run the reference's default associative
// branch (deq_slot_attn_unified_clean.wgsl:554-556) in place of the FPM write:
//   read   the one bank's value V, hard-read whatever its address score
//          (:1376-1385), added to the memory context scaled to
//          sigmoid(alpha_assoc) * |signal| * alpha_m / max(|V|, 1e-3) (:1505-1563);
//   write  (:2293-2948) value = x / rms(x) renormalised (x: the token's S_in row),
//          payload = value + P / rms(P) (P: the previous token's value), written
//          into V when the bank is empty (usage < 1e-4), t > 0 and
//          cos(V, P / rms(P)) <= 0.85; usage <- max(0.999 usage, mass); the
//          memory takes in 0.019 * mass of h* / rms(h*) (the FPM write is skipped
//          on these slots, :1971, so its gate factor stays 1.0 capped at 0.95);
//          the stored signal, which the adjoint's branch and the FPM backward
//          read, becomes the unnormalised payload (:2497).
// V and P live in this CTA's shared memory (each thread its own two elements),
// the usage in a register; all three are loaded and stored per launch.
template <bool FPM, int MAXT, int NW, bool ASSOC = false>
__global__ void __launch_bounds__(MAXT) picard_kernel(PicardArgs a) {
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  float *red = sm;               // 512
  float *vec = red + 512;        // 64   (q / bottleneck | retain-up)
  float *part = vec + 64;        // 1024 (up to 16 warps x 64)
  float *wsm = part + 1024;      // 64   ([0,16) read weights, [16] gate, [17,33) b_read_mem)
  float *keybuf = wsm + 64;      // 2 x 32
  float *mbuf = keybuf + 64;     // 2 x d
  float *xs = mbuf + 2 * a.d;    // d    (matvec input staging)
  float *wres = xs + a.d;        // n_resident x (d x 32) staged FPM matrices
  const int d = a.d, h = a.h, T = a.T;
  const int b = blockIdx.x / h, s = blockIdx.x % h;
  const int j0 = picard_j0();
  const int warp = threadIdx.x >> 5;
  const bool upper = ASSOC && s >= h / 2;  // an associative slot
  const float inv_d = 1.f / (float)d;
  const float *W = a.W;
  const float2 NS = ld2(W + a.off_ns + j0);
  const float2 anc = ld2(W + a.off_anchor + (size_t)s * d + j0);
  BlockReducer R(red);
  float2 hcur = f2(0.f), m = f2(0.f), hsv = f2(0.f), hbv = f2(0.f), wxv = f2(0.f), adv = f2(0.f);
  int cur = 0;
  // Per-slot rank-32 FPM matrices, staged in shared memory as far as they fit:
  // 0 W_k_mem, 1 W_q_mem, 2 W_k_write, 3 W_retain_up ([d][32]); 4 W_v_write,
  // 5 W_retain_down ([32][d]).  The rest stay in global memory (L2-resident),
  // or, at d = 512, in tensor memory.
  const float *mat[6];
  uint32_t tmem = 0;
  __shared__ uint32_t tmem_slot;
  if constexpr (FPM) {
    if (a.use_tmem) {  // matrices 3..5 in tensor memory, 128 columns each
      if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(&tmem_slot)),
                     "r"(512u));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncthreads();
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      // this warp's lane quadrant, this thread's half of the lane's columns
      tmem = tmem_slot + ((uint32_t)(32 * (warp & 3)) << 16) +
             64u * (uint32_t)(threadIdx.x / (blockDim.x >> 1));
    }
    const size_t ms = (size_t)s * d * kRank;
    const float *src[6] = {W + a.off_wkm + ms, W + a.off_wqm + ms, W + a.off_wkw + ms,
                           W + a.off_wup + ms, W + a.off_wvw + ms, W + a.off_wdown + ms};
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      float *dst = wres + (size_t)i * d * kRank;
      const bool res = i < a.n_resident;
      if (res)
        for (int q = threadIdx.x * 4; q < d * kRank; q += blockDim.x * 4) st4(dst + q, ld4(src[i] + q));
      mat[i] = res ? dst : src[i];
    }
    if (a.use_tmem && a.push) {
      tmem_stage(tmem + 0, mat[2], d, j0, true);     // W_k_write     [d][32]
      tmem_stage(tmem + 128, mat[3], d, j0, true);   // W_retain_up   [d][32]
      tmem_stage(tmem + 256, mat[4], d, j0, false);  // W_v_write     [32][d]
      tmem_stage(tmem + 384, mat[5], d, j0, false);  // W_retain_down [32][d]
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    } else if (a.use_tmem) {
      tmem_stage(tmem + 0, mat[3], d, j0, true);     // W_retain_up   [d][32]
      tmem_stage(tmem + 128, mat[4], d, j0, false);  // W_v_write     [32][d]
      tmem_stage(tmem + 256, mat[5], d, j0, false);  // W_retain_down [32][d]
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    m = ld2(a.mstate + ((size_t)b * h + s) * d + j0);
    st2(mbuf + j0, m);
    if (threadIdx.x < h) wsm[17 + threadIdx.x] = W[a.off_bread + threadIdx.x];  // b_read_mem
    hsv = ld2(W + a.off_hscale + (size_t)s * d + j0);
    hbv = ld2(W + a.off_hbias + (size_t)s * d + j0);
    wxv = make_float2(0.5f * tanhf(W[a.off_wx + (size_t)(j0 + 0) * d + j0 + 0]),
                      0.5f * tanhf(W[a.off_wx + (size_t)(j0 + 1) * d + j0 + 1]));
    const float2 al = ld2(W + a.off_alog + (size_t)s * d + j0);
    adv = make_float2(1.f / (1.f + expf(al.x)), 1.f / (1.f + expf(al.y)));
    __syncthreads();
    // read key of the carried memory for the first token (:855-883)
    mv_d_to_32<1, false>(mat[0], nullptr, m + hsv * tanh2(m) + hbv, j0, xs, keybuf, part);
  }
  const float band = fmaxf(a.eps, 0.15f * 0.2f);
  // loop-invariant factors of the memory read: score scale 1 / (sqrt(32) tau),
  // the uniform weight 1 / h and 1 / max(1 - 1/h, 1e-6) of the confidence gate
  const float score_scale = rsqrtf((float)kRank) / fmaxf(a.tau, 1e-3f);
  const float uni = 1.f / (float)(h > 1 ? h : 1);
  const float inv_conf = 1.f / fmaxf(1e-6f, 1.f - uni);
  // loop-invariant write parameters of this slot, staged in shared memory so
  // the token loop issues no global parameter loads: [0,d) b_delta,
  // [d,2d) W_write_gate, [2d,3d) b_retain (b_write_mem sits in wsm[40])
  float *wprm = wres + (size_t)a.n_resident * d * kRank;
  if constexpr (FPM) {
    st2(wprm + j0, ld2(W + a.off_bdelta + (size_t)s * d + j0));
    st2(wprm + d + j0, ld2(W + a.off_wgate + (size_t)s * d + j0));
    st2(wprm + 2 * d + j0, ld2(W + a.off_bret + (size_t)s * d + j0));
    if (threadIdx.x == 0) wsm[40] = W[a.off_bwrite + s];
    __syncthreads();
  }
  // push mode inbox: [2][h][d] memory rows and [2][h][32] read keys of every
  // slot, double-buffered by token parity, one mbarrier per buffer
  // ASSOC: bank value V and previous source P of this CTA's slot
  float *asv = wprm + 3 * d;
  float *asp = asv + d;
  float *inbox_m = wprm + 3 * d + (ASSOC ? 2 * d : 0);
  float *inbox_k = inbox_m + 2 * (size_t)h * d;
  uint64_t *inbar = reinterpret_cast<uint64_t *>(inbox_k + 2 * (size_t)h * kRank);
  const uint32_t inbox_bytes = (uint32_t)h * (uint32_t)(d + kRank) * 4u;
  if constexpr (FPM) {
    if (a.push) {
      if (threadIdx.x == 0) {
        for (int q = 0; q < 2; ++q)
          asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&inbar[q])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      }
      // every CTA's inbox barriers exist before anyone pushes
      asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
      asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
      __syncthreads();  // keybuf[0] / mbuf[0] of the prologue are complete
      if (threadIdx.x == 0) {
        inbox_arm(&inbar[0], inbox_bytes);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int q = 0; q < h; ++q) {
          push_to(mbuf, inbox_m + (size_t)s * d, &inbar[0], q, (uint32_t)d * 4u);
          push_to(keybuf, inbox_k + (size_t)s * kRank, &inbar[0], q, kRank * 4u);
        }
      }
    } else {
      // the prologue's memory and read key are published: split cluster barrier,
      // waited on before the first remote read
      asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    }
  }
#ifdef AIDEEN_PICARD_PROF
  long long _pt = clock64();
  long long _pacc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#endif
  // ASSOC: the carried bank state of this slot (V and P into this thread's own
  // shared-memory slots, so no barrier orders them); the usage in a register
  // (every thread updates it identically); sigmoid(alpha_assoc[s]) in wsm[54]
  // and the token's five sums in wsm[48..52], so nothing else of the branch
  // stays live in registers across the Picard iterations
  float au = 0.f;
  const size_t aso = ((size_t)b * h + s) * d + j0;
  if constexpr (ASSOC) {
    if (upper) {
      st2(asv + j0, ld2(a.assoc_v + aso));
      st2(asp + j0, ld2(a.assoc_p + aso));
      au = a.assoc_u[b * h + s];
      if (threadIdx.x == 0) wsm[54] = 1.f / (1.f + expf(-W[a.off_alpha_assoc + s]));
    }
  }
  // rows of the next token, loaded one token ahead
  // rows are token-major: row (t, b) = t * B + b
  const size_t e0 = (((size_t)a.t0 * a.B + b) * h + s) * d + j0;
  const size_t tstride = (size_t)a.B * h * d;  // one token step in a row-major [N][h][d] buffer
  float2 sig_nx = ld2(a.signal + e0);
  float2 Av_nx = a.slot_coord ? ld2(a.A + e0) : f2(0.f);

  // sum of squares of the next token's iteration-0 `dep` and `signal`,
  // reduced together with the previous token's last block reduction
  float dep0_sq = 0.f, sig_sq = 0.f;
  for (int t = a.t0; t < a.t1; ++t) {
    const size_t n = (size_t)t * a.B + b;
    const size_t e = (n * h + s) * d + j0;
    const float2 sig = sig_nx;
    const float2 Av = Av_nx;
    if (t + 1 < a.t1) {
      sig_nx = ld2(a.signal + e + tstride);
      if (a.slot_coord) Av_nx = ld2(a.A + e + tstride);
    }
    // ASSOC: this token's S_in row ([N][d], token-major)
    const float *xrow = a.s_in + ((size_t)t * a.B + b) * d + j0;
    if (t == 0) {
      float v[1] = {dot2(sig, sig)};
      bsum<NW>(R, v);
      const float den = fmaxf(sqrtf(v[0] * inv_d + 1e-6f), 1e-6f);
      hcur = make_float2(sig.x / den, sig.y / den);
      sig_sq = v[0];
    }
    if (t > 0 && t == a.t0) {  // a later token range: continue from the stored fixed point
      hcur = ld2(a.hstar + e - tstride);
    }
    if (t == a.t0 || !FPM) {
      const float2 dep0 = sig + hcur + anc + Av;
      float v[2] = {dot2(dep0, dep0), dot2(sig, sig)};
      bsum<NW>(R, v);
      dep0_sq = v[0];
      if (t > 0) sig_sq = v[1];  // (t == 0 computed it above; only the FPM read uses it)
    }
    float2 ctx = f2(0.f);
    bool waited = false;  // this token's cluster-barrier wait
    PT(0);
    float prev = 1.f;
    int it = 0;
    bool conv = false;
    // 1 / rms(dep) of the current iteration (one reciprocal instead of per-element divisions)
    float irr = rsqrtf(dep0_sq * inv_d + 1e-6f);
    float hq_sq = 0.f;
    // forward Anderson ring: Picard outputs g and residuals f = g - x of the
    // last two iterations of this token
    float2 ag1 = f2(0.f), ag2 = f2(0.f), af1 = f2(0.f), af2 = f2(0.f);
    while (it < a.max_iters && !conv) {
      if constexpr (FPM) {
        if (it == 1) {
          // every slot's key + memory for this token is visible past this wait
          if (a.push) {
            if (threadIdx.x == 0) {
              const int tl = t - a.t0;
              if (!inbox_wait(&inbar[tl & 1], (tl >> 1) & 1)) atomicExch(&g_picard_error, 1u);
              if (t + 1 < a.t1) inbox_arm(&inbar[(tl + 1) & 1], inbox_bytes);
            }
            // the next block barrier (inside the query product) orders the inbox reads
          } else {
            asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
          }
          waited = true;
          PT(0);
          // Model-A memory read from the first structured state (:1031-1200)
          const float ihq = rsqrtf(fmaxf(hq_sq, 1e-6f));
          const float sig_c = fmaxf(sig_sq, 1e-6f);
          const float sig_norm = sig_c * rsqrtf(sig_c);
          // the query lands in vec[0..32), written and read by warp 0 only
          // (q = W_q_mem . h / |h|: the staged h is unscaled, the sum is scaled)
          mv_d_to_32_partials(mat[1], xs, part);
          __syncthreads();
          if (threadIdx.x < 32) vec[threadIdx.x] = ihq * sum_partials32<NW>(part);
          PT(6);
          cg::cluster_group cl = cg::this_cluster();
          if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            __syncwarp();
            float kr[16];
            if (a.push) {
              const float *kb = inbox_k + (size_t)((t - a.t0) & 1) * h * kRank;
#pragma unroll
              for (int ms = 0; ms < 16; ++ms) kr[ms] = ms < h ? kb[ms * kRank + lane] : 0.f;
            } else {
#pragma unroll
              for (int ms = 0; ms < 16; ++ms)
                kr[ms] = ms < h ? cl.map_shared_rank(keybuf + cur * 32, ms)[lane] : 0.f;
            }
#ifdef AIDEEN_PICARD_PROF
            {
              float chk = 0.f;
#pragma unroll
              for (int ms = 0; ms < 16; ++ms) chk += kr[ms];
              if (chk == 12345.678f) wsm[41] = chk;
              PT(5);
            }
#endif
            const float qv = vec[lane];
            // 16 dot products over the warp in 16 shuffles: halving exchanges
            // (xor 16, 8, 4, 2) leave lane l with slot (l >> 1)'s partial, one
            // more xor-1 sum completes it
            float p[16];
#pragma unroll
            for (int ms = 0; ms < 16; ++ms) p[ms] = qv * kr[ms];
#pragma unroll
            for (int off = 16, nv = 8; off >= 2; off >>= 1, nv >>= 1) {
              const bool upper = (lane & off) != 0;
#pragma unroll
              for (int i = 0; i < nv; ++i) {
                const float send = upper ? p[i] : p[i + nv];
                const float keep = upper ? p[i + nv] : p[i];
                p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
              }
            }
            const float part_dot = p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
            float sc = __shfl_sync(0xffffffffu, part_dot, (lane & 15) << 1);
            if (lane >= h) sc = -1e30f;
            if (lane < h) sc = (sc + wsm[17 + lane]) * score_scale;
            const float mx = warp_max(sc);
            const float ex = lane < h ? __expf(sc - mx) : 0.f;
            const float se = fmaxf(warp_sum(ex), 1e-12f);
            const float w = __fdividef(ex, se);
            const float peak = warp_max(lane < h ? w : 0.f);
            if (lane < h) wsm[lane] = w;
            if (lane == 0) {
              const float conf = fminf(fmaxf((peak - uni) * inv_conf, 0.f), 1.f);
              wsm[16] = fmaxf(conf * rsqrtf(fmaxf(conf, 1e-30f)), a.gate_min);
            }
          }
          __syncthreads();
          PT(7);
          float2 mr = f2(0.f);
          if (a.push) {
            const float *mb = inbox_m + (size_t)((t - a.t0) & 1) * h * d + j0;
            for (int q = 0; q < h; ++q) mr = mr + wsm[q] * ld2(mb + (size_t)q * d);
          } else {
            for (int base = 0; base < h; base += 8) {   // 8 remote loads in flight at a time
              float2 mm[8];
#pragma unroll
              for (int q = 0; q < 8; ++q)
                if (base + q < h) mm[q] = ld2(cl.map_shared_rank(mbuf + cur * d, base + q) + j0);
#pragma unroll
              for (int q = 0; q < 8; ++q)
                if (base + q < h) mr = mr + wsm[base + q] * mm[q];
            }
          }
          const float2 mu = tanh2(mr);
          float v1[1] = {dot2(mu, mu)};
          bsum<NW>(R, v1);
          // |mu| >= 1e-3 (the 1e-6 floor on |mu|^2), so 1 / max(|mu|, 1e-6) = rsqrt(|mu|^2)
          const float coef = sig_norm * fmaxf(a.alpha_m, 0.001f) * rsqrtf(fmaxf(v1[0], 1e-6f)) * wsm[16];
          ctx = coef * mu;
          if (upper) {  // the bank's value, hard-read (:1505-1563)
            const float sc = wsm[54] * sig_norm * fmaxf(a.alpha_m, 0.001f) / fmaxf(sqrtf(fmaxf(wsm[52], 1e-6f)), 1e-6f);
            ctx = ctx + sc * ld2(asv + j0);
          }
          PT(2);
        }
      }
      float2 pre = sig + hcur + anc;
      if (it == 0) pre = pre + Av;
      if (FPM && it >= 1) pre = pre + ctx;
      const float2 f = NS * (irr * pre);
      const float2 hn = a.blend * f + (1.f - a.blend) * hcur;
      const float2 dh = hn - hcur;
      // one reduction per iteration: |dh|^2 of this iteration, |dep|^2 of the
      // next one (dep has no attention term after iteration 0) and, after
      // iteration 0 with FPM, |h|^2 for the memory read's query
      const float2 dep_nx = sig + hn + anc;
      // the memory read's query input (h after iteration 0), published by this
      // iteration's reduction barrier
      if (FPM && it == 0) st2(xs + j0, hn);
      float v2[3] = {dot2(dh, dh), dot2(dep_nx, dep_nx), dot2(hn, hn)};
      // Anderson mixing from the third iteration on, over the residuals of
      // iterations >= 1 (the map is fixed within the token from there); the
      // slot's normal equations ride along in this iteration's reduction
      const bool mix = a.anderson_m >= 2 && it >= 2;
      const int n_res = it < a.anderson_m ? it : a.anderson_m;
      float q5[5];
      if (mix) {
        const float2 D0 = dh - af1;
        const float2 D1 = n_res == 3 ? af1 - af2 : f2(0.f);
        float v7[7] = {v2[0], v2[1], dot2(D0, D0), dot2(D0, D1), dot2(D1, D1), dot2(D0, dh), dot2(D1, dh)};
        bsum<NW>(R, v7);
        v2[0] = v7[0];
        v2[1] = v7[1];
#pragma unroll
        for (int q = 0; q < 5; ++q) q5[q] = v7[2 + q];
      } else if (FPM && it == 0) {
        if (upper) {
          // this token's sums |x|^2, |P|^2, x.P, V.P, |V|^2 ride along, parked
          // in wsm[48..52] (read after later barriers)
          const float2 Vv = ld2(asv + j0), Pv = ld2(asp + j0), xin = ld2(xrow);
          float v8[8] = {v2[0], v2[1], v2[2], dot2(xin, xin), dot2(Pv, Pv), dot2(xin, Pv), dot2(Vv, Pv),
                         dot2(Vv, Vv)};
          bsum<NW>(R, v8);
          v2[0] = v8[0];
          v2[1] = v8[1];
          v2[2] = v8[2];
          if (threadIdx.x == 0) {
#pragma unroll
            for (int q = 0; q < 5; ++q) wsm[48 + q] = v8[3 + q];
          }
        } else {
          bsum<NW>(R, v2);
        }
      } else {
        float v2b[2] = {v2[0], v2[1]};
        bsum<NW>(R, v2b);
        v2[0] = v2b[0];
        v2[1] = v2b[1];
      }
      // rms(dep) >= 1e-3 always (the 1e-6 floor), so max(rms, 1e-6) = rms
      const float ex = v2[0] * inv_d + 1e-12f;  // > 0
      const float err = ex * rsqrtf(ex) * irr;  // sqrt(ex) off the IEEE square-root path
      irr = rsqrtf(v2[1] * inv_d + 1e-6f);
      hq_sq = v2[2];
      hcur = hn;
      const bool strict = err < a.eps;
      // plateau = |err - prev| / max(prev, eps) <= 0.10, without the division
      const bool homeo = (it + 1 >= 4) && (err <= band) && (fabsf(err - prev) <= 0.10f * fmaxf(prev, a.eps));
      conv = strict || homeo;
      if (mix && !conv) {
        float g0, g1;
        if (anderson_fwd_gamma(q5, n_res - 1, g0, g1)) {
          // next iterate g_0 - sum gamma_i (g_i - g_{i+1}); its |dep|^2 needs
          // one more reduction
          hcur = hn - g0 * (hn - ag1) - g1 * (ag1 - ag2);
          const float2 depm = sig + hcur + anc;
          float v1[1] = {dot2(depm, depm)};
          bsum<NW>(R, v1);
          irr = rsqrtf(v1[0] * inv_d + 1e-6f);
        }
      }
      af2 = af1;
      af1 = dh;
      ag2 = ag1;
      ag1 = hn;
      prev = err;
      ++it;
      PT(1);
    }
    float2 pre_adj = sig + hcur;
    if (a.slot_coord) pre_adj = pre_adj + Av + anc;
    if (!FPM) {
      st2(a.hstar + e, hcur);
      st2(a.pre + e, pre_adj);
      if (threadIdx.x == 0) a.iters[n * h + s] = it;
    }
    PT(3);
    if constexpr (FPM) {
      if (!waited) {  // solve stopped before the memory read: still consume this token's phase
        if (a.push) {
          if (threadIdx.x == 0) {
            const int tl = t - a.t0;
            if (!inbox_wait(&inbar[tl & 1], (tl >> 1) & 1)) atomicExch(&g_picard_error, 1u);
            if (t + 1 < a.t1) inbox_arm(&inbar[(tl + 1) & 1], inbox_bytes);
          }
        } else {
          asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        }
        PT(0);
      }
      float2 mn;
      if (upper) {
        // associative write in place of the FPM write (:2293-2948); one
        // reduction: |h*|^2 and the next token's |dep0|^2, |signal|^2
        const float2 dep0n = sig_nx + hcur + anc + Av_nx;
        float v3[3] = {dot2(hcur, hcur), dot2(dep0n, dep0n), dot2(sig_nx, sig_nx)};
        bsum<NW>(R, v3);
        dep0_sq = v3[1];
        sig_sq = v3[2];
        const float a_xx = wsm[48], a_pp = wsm[49], a_xp = wsm[50], a_vp = wsm[51], a_vv = wsm[52];
        const float2 xin = ld2(xrow);
        const float irc = 1.f / fmaxf(sqrtf(a_xx * inv_d + 1e-6f), 1e-6f);
        const float irv = 1.f / fmaxf(sqrtf(a_xx * irc * irc * inv_d + 1e-6f), 1e-6f);
        const float kv = irc * irv;  // value = kv * x
        const float irp = 1.f / fmaxf(sqrtf(a_pp * inv_d + 1e-6f), 1e-6f);
        const float2 Pv = ld2(asp + j0), Vv = ld2(asv + j0);
        st2(a.assoc_read + e, Vv);  // the value this token read (the alpha_assoc gradient's input)
        const float2 val = kv * xin;
        const float2 pay_raw = val + irp * Pv;
        const float qq = a_xx * kv * kv + 2.f * a_xp * kv * irp + a_pp * irp * irp;  // |payload|^2
        const float irq = 1.f / fmaxf(sqrtf(qq * inv_d + 1e-6f), 1e-6f);
        const float uc = fminf(fmaxf(isfinite(au) ? au : 0.f, 0.f), 1.f);
        float cosv = a_vp * irp / sqrtf(fmaxf(a_vv * a_pp * irp * irp, 1e-12f));
        if (!isfinite(cosv)) cosv = -1.f;
        const float mass = (t > 0 && uc < 1e-4f && !(cosv > 0.85f)) ? 1.f : 0.f;
        st2(asv + j0, (1.f - mass) * Vv + (mass * irq) * pay_raw);
        st2(asp + j0, val);
        au = fminf(fmaxf(fmaxf(0.999f * uc, mass), 0.f), 1.f);
        const float cc = 0.02f * 0.95f * mass;
        const float irh = 1.f / fmaxf(sqrtf(v3[0] * inv_d + 1e-6f), 1e-6f);
        mn = (1.f - cc) * m + (cc * irh) * hcur;
        // the stored signal is the payload from here on: the adjoint's branch and
        // the FPM backward read it
        pre_adj = pay_raw + hcur;
        if (a.slot_coord) pre_adj = pre_adj + Av + anc;
        st2(a.sig_store + e, pay_raw);
      } else {
        // post-solve memory write (:1965-2140)
        const float2 c = 0.5f * (hcur + sig);
        PT(4);
        float2 pv, dv;
        if (a.use_tmem && a.push) {
          mv2_d_to_32_tmem(tmem + 0, tmem + 128, c, vec, part);   // bottleneck | retain-up
          PT(5);
          mv2_32_to_d_tmem(tmem + 256, vec, tmem + 384, vec + 32, pv, dv);
        } else if (a.use_tmem) {
          mv_d_to_32_smem_tmem(mat[2], tmem + 0, c, j0, xs, vec, part);   // bottleneck | retain-up
          PT(5);
          mv2_32_to_d_tmem(tmem + 128, vec, tmem + 256, vec + 32, pv, dv);
        } else {
          mv_d_to_32<2>(mat[2], mat[3], c, j0, xs, vec, part);   // bottleneck | retain-up
          PT(5);
          mv2_32_to_d(mat[4], vec, mat[5], vec + 32, d, j0, pv, dv);
        }
        PT(6);
        const float2 prop = tanh2(ld2(wprm + j0) + pv);
        const float2 df = prop - m;
        // the next token's iteration-0 |dep|^2 and |signal|^2 ride along
        const float2 dep0n = sig_nx + hcur + anc + Av_nx;
        float v3[6] = {dot2(m, m), dot2(df, df), dot2(hcur, hcur), dot2(ld2(wprm + d + j0), c), dot2(dep0n, dep0n),
                       dot2(sig_nx, sig_nx)};
        bsum<NW>(R, v3);
        dep0_sq = v3[4];
        sig_sq = v3[5];
        const float2 hu = rsqrtf(fmaxf(v3[2] * inv_d, 1e-6f)) * hcur;
        const float raw_z = __fdividef(1.f, 1.f + __expf(-(v3[3] * rsqrtf((float)d) + wsm[40] - 1.5f)));
        const float z = fminf(fmaxf(raw_z, 0.f), 1.f);
        const float pq = fmaxf(v3[0], 1e-6f), dq = fmaxf(v3[1], 1e-6f);
        const float prev_norm = pq * rsqrtf(pq);
        const float diff_norm = dq * rsqrtf(dq);
        const float novelty = __fdividef(diff_norm, diff_norm + prev_norm + 1e-6f);
        const float2 rrv = sigmoid2(ld2(wprm + 2 * d + j0) + dv);
        const float2 retain = f2(1.f) - novelty * (f2(1.f) - rrv);
        const float2 write = (z * 0.1f) * prop;
        const float zq = fmaxf(z, 1e-6f);
        const float2 x = (zq * rsqrtf(zq)) * hu + wxv * hu + write;
        const float2 base = adv * m + (f2(1.f) - adv) * x;
        mn = retain * m + (f2(1.f) - retain) * base;
      }
      if constexpr (ASSOC) {
        if (!upper) st2(a.sig_store + e, sig);
      }
      st2(mbuf + (cur ^ 1) * d + j0, mn);
      m = mn;
      PT(4);
      // read key of the new memory, used by every slot at the next token
      // peers read the key after the cluster barrier below; no block barrier needed
      if (a.push) {
        // push this token's memory row and key into every slot's inbox for the
        // next token (none, and no key, after the last token of the launch)
        if (t + 1 < a.t1) {
          st2(xs + j0, m + hsv * tanh2(m) + hbv);
          __syncthreads();
          mv_d_to_32_partials(mat[0], xs, part);
          PT(7);
          __syncthreads();  // key partials and the mbuf row complete
          if (warp == 0) {
            const int lane = threadIdx.x & 31;
            keybuf[(cur ^ 1) * 32 + lane] = sum_partials32<NW>(part);
            __syncwarp();
            if (lane == 0) {
              const int nb = (t - a.t0 + 1) & 1;
              asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
              for (int q = 0; q < h; ++q) {
                push_to(mbuf + (cur ^ 1) * d, inbox_m + ((size_t)nb * h + s) * d, &inbar[nb], q, (uint32_t)d * 4u);
                push_to(keybuf + (cur ^ 1) * 32, inbox_k + ((size_t)nb * h + s) * kRank, &inbar[nb], q,
                        kRank * 4u);
              }
            }
          }
        }
        cur ^= 1;
      } else {
        mv_d_to_32<1, false>(mat[0], nullptr, m + hsv * tanh2(m) + hbv, j0, xs, keybuf + (cur ^ 1) * 32, part);
        PT(7);
        cur ^= 1;
        // publish this token's memory and key to the cluster; the global stores
        // (no reader inside this kernel) come after the arrive, so its release
        // orders only the shared-memory writes
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
      }
      st2(a.hist + e, mn);
      st2(a.hstar + e, hcur);
      st2(a.pre + e, pre_adj);
      st2(a.fpmctx + e, ctx);
      if (threadIdx.x == 0) a.iters[n * h + s] = it;
      PT(4);
    }
  }
#ifdef AIDEEN_PICARD_PROF
  if (threadIdx.x == 0)
    for (int i = 0; i < 8; ++i) g_picard_prof[blockIdx.x * 8 + i] += _pacc[i];
#endif
  if constexpr (ASSOC) {
    if (upper) {
      st2(a.assoc_v + aso, ld2(asv + j0));
      st2(a.assoc_p + aso, ld2(asp + j0));
      if (threadIdx.x == 0) a.assoc_u[b * h + s] = au;
    }
  }
  if constexpr (FPM) {
    st2(a.mstate + ((size_t)b * h + s) * d + j0, m);
    if (a.push) {  // no CTA leaves while a peer may still push into it
      asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
      asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    } else {
      // match the last arrive: peers may read this block's memory until they pass it
      asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
    if (a.use_tmem) {
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncthreads();
      if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_slot), "r"(512u));
    }
  }
}

__global__ void pool_rmsnorm_kernel(const float *__restrict__ hstar, const float *__restrict__ g,
                                    float *__restrict__ pooled, float *__restrict__ y,
                                    float *__restrict__ lrms, int h, int d) {
  __shared__ __align__(16) float red[512];
  const int n = blockIdx.x, j0 = threadIdx.x * 4;
  float4 p = f4(0.f);
  for (int s = 0; s < h; ++s) p = p + ld4(hstar + ((size_t)n * h + s) * d + j0);
  p = (1.f / (float)h) * p;
  st4(pooled + (size_t)n * d + j0, p);
  if (!y) return;
  BlockReducer R(red);
  float v[1] = {dot4(p, p)};
  R.sum(v);
  const float r = sqrtf(v[0] / d + 1e-5f);
  const float4 gg = ld4(g + j0);
  st4(y + (size_t)n * d + j0,
      make_float4(p.x / r * gg.x, p.y / r * gg.y, p.z / r * gg.z, p.w / r * gg.w));
  if (threadIdx.x == 0) lrms[n] = r;
}

__global__ void solve_stats_kernel(const int32_t *__restrict__ iters, const float *__restrict__ hstar,
                                   int rows, int d, int max_iters,
                                   unsigned long long *__restrict__ st) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  bool bad = false;
  for (int j = lane * 4; j < d; j += 128) bad |= !finite4(ld4(hstar + (size_t)w * d + j));
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    const int it = iters[w];
    atomicAdd(&st[0], (unsigned long long)it);
    atomicMax(&st[1], (unsigned long long)it);
    if (it >= max_iters) atomicAdd(&st[2], 1ull);
    if (bad) atomicAdd(&st[3], 1ull);
  }
}

// ---------------------------------------------------------------------------
cudaError_t launch_embed(const int32_t *tok, const float *emb, float *S, int N, int d, int vocab,
                         cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  embed_gather_kernel<<<N, 128, 0, st>>>(tok, emb, S, N, d, vocab);
  return cudaGetLastError();
}

cudaError_t launch_attn_softmax(const AttnArgs &a, int N, cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  attn_softmax_kernel<<<N, 32 * a.h, 0, st>>>(a);
  return cudaGetLastError();
}

__global__ void pack_qkv_kernel(const float *__restrict__ W, size_t oq, size_t ok, size_t ov, int h, int d,
                                float *__restrict__ Wcat) {
  const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;  // over h*d*96
  if (i >= (size_t)h * d * 96) return;
  const int c = (int)(i % 96);
  const size_t sj = i / 96;  // s*d + j
  const size_t src = (c < 32 ? oq : c < 64 ? ok : ov) + (sj / d) * (size_t)d * d + (sj % d) * d + (c % 32);
  Wcat[i] = W[src];
}

cudaError_t launch_pack_qkv(const float *W, size_t oq, size_t ok, size_t ov, int h, int d, float *Wcat,
                            cudaStream_t st) {
  const size_t n = (size_t)h * d * 96;
  pack_qkv_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(W, oq, ok, ov, h, d, Wcat);
  return cudaGetLastError();
}

cudaError_t launch_attn_scale(const AttnArgs &a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  attn_scale_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, rows);
  return cudaGetLastError();
}

// Reads (and clears) the flag a Picard launch sets when a bounded inbox wait
// gave up; ordered on `st` after the solve.
unsigned int *picard_error_dev() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g_picard_error) == cudaSuccess ? static_cast<unsigned int *>(p) : nullptr;
}

cudaError_t picard_error_async(unsigned int *host_flag, cudaStream_t st) {
  static const unsigned int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(host_flag, g_picard_error, sizeof(unsigned int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbolAsync(g_picard_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
}

static size_t picard_smem_base(int d) {
  // red, vec, part, wsm, keybuf, mbuf (2d), xs (d), write parameters (3d)
  return (size_t)(512 + 64 + 1024 + 64 + 64 + 6 * d) * sizeof(float);
}

template <bool FPM, int MAXT, int NW = 0, bool ASSOC = false>
static cudaError_t picard_launch(const PicardArgs &a, cudaStream_t st) {
  const int threads = a.d / 2;
  // ASSOC: the bank value and previous source of the CTA's slot (2 d floats)
  size_t smem = picard_smem_base(a.d) + (ASSOC ? 2 * (size_t)a.d * sizeof(float) : 0);
  if (!FPM) {
    cudaError_t e = cudaFuncSetAttribute(picard_kernel<false, MAXT, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    picard_kernel<false, MAXT, NW><<<a.B * a.h, threads, smem, st>>>(a);
    return cudaGetLastError();
  }
  cudaError_t e = cudaFuncSetAttribute(picard_kernel<true, MAXT, NW, ASSOC>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t mat_bytes = (size_t)a.d * kRank * sizeof(float);
  PicardArgs p = a;
  p.n_resident = 0;
  while (p.n_resident < 6 && smem + mat_bytes <= (size_t)optin) {
    smem += mat_bytes;
    ++p.n_resident;
  }
  // d = 512: the three matrices that do not fit in shared memory go to tensor
  // memory (one 256-thread block per SM owns all 512 columns); with h <= 8 a
  // fourth one moves there too, and the freed shared memory holds the inbox of
  // the pushed memory rows / read keys
  static const bool no_tmem = getenv("AIDEEN_PICARD_NO_TMEM") != nullptr;
  static const bool no_push = getenv("AIDEEN_PICARD_NO_PUSH") != nullptr;
  p.use_tmem = (a.d == 512 && p.n_resident == 3 && !no_tmem) ? 1 : 0;
  p.push = (p.use_tmem && a.h <= 8 && !no_push) ? 1 : 0;
  if (p.push) {
    p.n_resident = 2;
    smem -= mat_bytes;
    smem += (2 * (size_t)a.h * (a.d + kRank) + 4) * sizeof(float);
  }
  e = cudaFuncSetAttribute(picard_kernel<true, MAXT, NW, ASSOC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.B * a.h);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.h;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, picard_kernel<true, MAXT, NW, ASSOC>, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_picard(const PicardArgs &a, bool fpm, cudaStream_t st) {
  if (a.B <= 0 || a.T <= 0 || a.t1 <= a.t0) return cudaSuccess;
  if (fpm && a.assoc) {  // the associative branch on the upper slots
    if (a.d > 512) return picard_launch<true, 512, 0, true>(a, st);
    if (a.d == 512) return picard_launch<true, 256, 8, true>(a, st);
    return picard_launch<true, 256, 0, true>(a, st);
  }
  if (a.d > 512) return fpm ? picard_launch<true, 512>(a, st) : picard_launch<false, 512>(a, st);
  if (a.d == 512)  // 256 threads: eight warps, static reductions
    return fpm ? picard_launch<true, 256, 8>(a, st) : picard_launch<false, 256, 8>(a, st);
  return fpm ? picard_launch<true, 256>(a, st) : picard_launch<false, 256>(a, st);
}

cudaError_t launch_pool_rmsnorm(const float *hstar, const float *g, float *pooled, float *y,
                                float *lrms, int N, int h, int d, cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  pool_rmsnorm_kernel<<<N, d / 4, 0, st>>>(hstar, g, pooled, y, lrms, h, d);
  return cudaGetLastError();
}

cudaError_t launch_solve_stats(const int32_t *iters, const float *hstar, int rows, int d,
                               int max_iters, unsigned long long *st4p, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  solve_stats_kernel<<<(rows + 7) / 8, 256, 0, st>>>(iters, hstar, rows, d, max_iters, st4p);
  return cudaGetLastError();
}

}  // namespace aideen

#ifdef AIDEEN_PICARD_PROF
extern "C" int aideen_debug_picard_prof(unsigned long long *out, int n, int reset) {
  if (out && cudaMemcpyFromSymbol(out, aideen::g_picard_prof, n * sizeof(unsigned long long)) != cudaSuccess) return 2;
  if (reset) {
    static unsigned long long zeros[1024 * 8];
    cudaMemcpyToSymbol(aideen::g_picard_prof, zeros, sizeof(zeros));
  }
  return 0;
}
#endif
