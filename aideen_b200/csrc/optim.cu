#include <cooperative_groups.h>
// Fused optimizer sweeps, spectral renormalisation and LM-head helpers.
//
//   adam        bias-corrected Adam, one float4 pass over w, g, m, v
//               (aideen-training-lab/src/optimizer.rs:105-183)
//   clipped_sgd w <- w*(1 - lr*wd [main weights]) - clamp(lr*g*scale, +-0.5)
//               (fused_deq_update.wgsl:402-410, 809-823)
//   spectral    power iteration + rescale, a cluster of 8 CTAs per matrix
//               (aideen-block/src/shaders/spectral_renorm.wgsl:83-196)
//   softmax_ce / rmsnorm_bwd: dense LM-head loss and dL/dH_pooled
//               (lm_train.wgsl:79-130, 327-395)
#include "common.cuh"
#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace aideen {

// Two float4 groups per thread and iteration (8 independent 16-byte loads in
// flight); the gradient and moments stream through with evict-first hints,
// the weights (read again by the next forward) with default caching.
__device__ __forceinline__ void adam4(float *__restrict__ w, const float *__restrict__ g, float *__restrict__ m1,
                                      float *__restrict__ m2, size_t i, float4 gg, float4 m, float4 v, float4 ww,
                                      float lr, float b1, float b2, float eps, float bc1, float bc2) {
  m = b1 * m + (1.f - b1) * gg;
  v = b2 * v + (1.f - b2) * (gg * gg);
  __stcs(reinterpret_cast<float4 *>(m1) + i, m);
  __stcs(reinterpret_cast<float4 *>(m2) + i, v);
  ww.x -= lr * (m.x / bc1) / (sqrtf(v.x / bc2) + eps);
  ww.y -= lr * (m.y / bc1) / (sqrtf(v.y / bc2) + eps);
  ww.z -= lr * (m.z / bc1) / (sqrtf(v.z / bc2) + eps);
  ww.w -= lr * (m.w / bc1) / (sqrtf(v.w / bc2) + eps);
  reinterpret_cast<float4 *>(w)[i] = ww;
}

__global__ void adam_kernel(float *__restrict__ w, const float *__restrict__ g, float *__restrict__ m1,
                            float *__restrict__ m2, size_t n, float lr, float b1, float b2,
                            float eps, float bc1, float bc2, float gs) {
  const size_t n4 = n / 4;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  const float4 *a4 = reinterpret_cast<const float4 *>(m1);
  const float4 *b4 = reinterpret_cast<const float4 *>(m2);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += 2 * stride) {
    const size_t j = i + stride;
    const bool two = j < n4;
    const float4 ga = __ldcs(g4 + i), ma = __ldcs(a4 + i), va = __ldcs(b4 + i), wa = w4[i];
    float4 gb = f4(0.f), mb = f4(0.f), vb = f4(0.f), wb = f4(0.f);
    if (two) {
      gb = __ldcs(g4 + j);
      mb = __ldcs(a4 + j);
      vb = __ldcs(b4 + j);
      wb = w4[j];
    }
    adam4(w, g, m1, m2, i, gs * ga, ma, va, wa, lr, b1, b2, eps, bc1, bc2);
    if (two) adam4(w, g, m1, m2, j, gs * gb, mb, vb, wb, lr, b1, b2, eps, bc1, bc2);
  }
  if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {  // tail
    const size_t i = n4 * 4 + threadIdx.x;
    const float gg = gs * g[i];
    const float m = b1 * m1[i] + (1.f - b1) * gg;
    const float v = b2 * m2[i] + (1.f - b2) * gg * gg;
    m1[i] = m;
    m2[i] = v;
    w[i] -= lr * (m / bc1) / (sqrtf(v / bc2) + eps);
  }
}

static int sweep_blocks(size_t n4) {
  size_t b = (n4 + 255) / 256;
  if (b > 148 * 8) b = 148 * 8;
  return b < 1 ? 1 : (int)b;
}

// Adam over a list of strided segments (rows of row4 float4s, `stride` floats
// apart): the same arithmetic as adam_kernel on exactly the listed entries.
__global__ void adam_segs_kernel(float *__restrict__ w, const float *__restrict__ g, float *__restrict__ m1,
                                 float *__restrict__ m2, AdamSegs sg, float lr, float b1, float b2, float eps,
                                 float bc1, float bc2, float gs) {
  const unsigned long long total = sg.start4[sg.n];
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  const float4 *g4 = reinterpret_cast<const float4 *>(g);
  const float4 *a4 = reinterpret_cast<const float4 *>(m1);
  const float4 *b4 = reinterpret_cast<const float4 *>(m2);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < total; i += stride) {
    int k = 0;
    while (k + 1 < sg.n && i >= sg.start4[k + 1]) ++k;
    const unsigned long long li = i - sg.start4[k];
    const unsigned long long r = li / (unsigned)sg.row4[k], c = li - r * (unsigned)sg.row4[k];
    const size_t q = (sg.off[k] + r * (unsigned long long)sg.stride[k]) / 4 + c;  // float4 index
    adam4(w, g, m1, m2, q, gs * __ldcs(g4 + q), __ldcs(a4 + q), __ldcs(b4 + q), w4[q], lr, b1, b2, eps, bc1, bc2);
  }
}

cudaError_t launch_adam_segs(float *w, const float *g, float *m1, float *m2, const AdamSegs &sg, float lr,
                             float b1, float b2, float eps, float bc1, float bc2, float gs, cudaStream_t st) {
  if (sg.n <= 0 || sg.start4[sg.n] == 0) return cudaSuccess;
  adam_segs_kernel<<<sweep_blocks(sg.start4[sg.n]), 256, 0, st>>>(w, g, m1, m2, sg, lr, b1, b2, eps, bc1, bc2,
                                                                   gs);
  return cudaGetLastError();
}

__global__ void clipped_sgd_kernel(float *__restrict__ w, const float *__restrict__ g, size_t n,
                                   size_t main_len, float lr, float wd, float gs) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float mult = i < main_len ? 1.f - lr * wd : 1.f;
    const float step = fminf(fmaxf(lr * g[i] * gs, -0.5f), 0.5f);
    w[i] = w[i] * mult - step;
  }
}


cudaError_t launch_adam(float *w, const float *g, float *m1, float *m2, size_t n, float lr, float b1,
                        float b2, float eps, float bc1, float bc2, float gs, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  adam_kernel<<<sweep_blocks(n / 4), 256, 0, st>>>(w, g, m1, m2, n, lr, b1, b2, eps, bc1, bc2, gs);
  return cudaGetLastError();
}

cudaError_t launch_clipped_sgd(float *w, const float *g, size_t n, size_t main_len, float lr,
                               float wd, float gs, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  clipped_sgd_kernel<<<sweep_blocks(n), 256, 0, st>>>(w, g, n, main_len, lr, wd, gs);
  return cudaGetLastError();
}

struct SpecArgs {
  float *W;
  int d, h, n_iters;
  size_t wq, wk, wv, wo, win, wx, wout;
  float attn, winth, fpm, wvth, woth;
  float *sigmas;
};

// Power iteration (d a multiple of 128, d <= 1024): a cluster of 8 CTAs per
// matrix, CTA q owning rows [q*R, (q+1)*R), R = d/8, streamed from L2 on every
// sweep (all 5h+2 matrices stay L2-resident and every CTA of the launch is
// resident at once).  One sweep over the local rows forms both u_r = A_r . v
// (a warp per row) and this CTA's share of A^T u, kept per lane (lane owns
// the float4 columns lane + 32 i); the shares are summed over warps and then
// over the cluster in rank order.  Sweep 0 uses the reference's start vector
// u = 1/sqrt(d); sweep k >= 1 gives sigma_k = |A v_k| and v_{k+1} = A^T u_k /
// |A^T u_k|, the same vectors as the reference's v = A^T u / |A^T u|,
// u = A v, sigma = |u|, u /= sigma (the scale of u cancels in the next
// normalisation).
constexpr int kSpecCluster = 8;

template <int NV>
__global__ void __launch_bounds__(256, NV <= 4 ? 3 : 1) spectral_sweep_kernel(SpecArgs a) {
  extern __shared__ __align__(16) float smc[];
  cg::cluster_group cl = cg::this_cluster();
  const int d = a.d, h = a.h, R = d / kSpecCluster;
  const int q = (int)cl.block_rank();
  const int mi = blockIdx.x / kSpecCluster;
  float *vfull = smc;                 // d   normalised v
  float *vpart = vfull + d;           // d   this CTA's share of A^T u
  float *wpart = vpart + d;           // 8 x d per-warp shares
  float *vslice = wpart + 8 * d;      // R   cluster sum of the column slice [q*R, (q+1)*R)
  float *nrm = vslice + R;            // [0] slice |v|^2, [1] local |u|^2 (published between the syncs)
  float *red = nrm + 4;               // 8 per-warp |u|^2
  size_t off;
  float thr;
  if (mi < h) { off = a.wq + (size_t)mi * d * d; thr = a.attn; }
  else if (mi < 2 * h) { off = a.wk + (size_t)(mi - h) * d * d; thr = a.attn; }
  else if (mi < 3 * h) { off = a.wv + (size_t)(mi - 2 * h) * d * d; thr = a.wvth; }
  else if (mi < 4 * h) { off = a.wo + (size_t)(mi - 3 * h) * d * d; thr = a.woth; }
  else if (mi < 5 * h) { off = a.win + (size_t)(mi - 4 * h) * d * d; thr = a.winth; }
  else if (mi == 5 * h) { off = a.wx; thr = a.fpm; }
  else { off = a.wout; thr = a.fpm; }
  float *M = a.W + off + (size_t)q * R * d;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float u0 = 1.f / sqrtf((float)d);
  float sigma = 1.f;
  for (int it = 0; it <= a.n_iters; ++it) {
    float4 vr[NV], acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      vr[i] = it > 0 ? ld4(vfull + 4 * (lane + 32 * i)) : f4(0.f);
      acc[i] = f4(0.f);
    }
    float uu = 0.f;
#pragma unroll 1
    for (int r = warp; r < R; r += 8) {
      float4 av[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) av[i] = ld4(M + (size_t)r * d + 4 * (lane + 32 * i));
      float ur = u0;
      if (it > 0) {
        float p = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) p += dot4(av[i], vr[i]);
        ur = warp_sum(p);
        uu += ur * ur;
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) acc[i] = fma4(av[i], f4(ur), acc[i]);
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) st4(wpart + (size_t)warp * d + 4 * (lane + 32 * i), acc[i]);
    if (lane == 0) red[warp] = uu;
    __syncthreads();
    for (int c = tid; c < d; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += wpart[(size_t)w * d + c];
      vpart[c] = t;
    }
    float uu_cta = 0.f;
    if (tid == 0)
      for (int w = 0; w < 8; ++w) uu_cta += red[w];
    cl.sync();
    if (tid == 0) nrm[1] = uu_cta;
    // this CTA's column slice of A^T u, summed over the cluster in rank order
    float part = 0.f;
    for (int i = tid; i < R; i += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int p = 0; p < kSpecCluster; ++p) t += cl.map_shared_rank(vpart, p)[q * R + i];
      vslice[i] = t;
      part += t * t;
    }
    part = warp_sum(part);
    __syncthreads();  // red[] reads above are done
    if (lane == 0) red[warp] = part;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += red[w];
      nrm[0] = t;
    }
    cl.sync();
    float vn2 = 0.f, un2 = 0.f;
#pragma unroll
    for (int p = 0; p < kSpecCluster; ++p) {
      const float *pn = cl.map_shared_rank(nrm, p);
      vn2 += pn[0];
      un2 += pn[1];
    }
    if (it > 0) sigma = sqrtf(un2 + 1e-12f);
    const float vn = sqrtf(vn2 + 1e-12f);
    for (int c = tid; c < d; c += blockDim.x) vfull[c] = cl.map_shared_rank(vslice, c / R)[c % R] / vn;
    __syncthreads();
  }
  if (tid == 0 && q == 0 && a.sigmas) a.sigmas[mi] = sigma;
  if (sigma > thr) {
    const float sc = thr / sigma;
    for (int i = tid * 4; i < R * d; i += blockDim.x * 4) st4(M + i, sc * ld4(M + i));
  }
  cl.sync();  // peers' last remote reads of this CTA's vectors and norms are done
}

cudaError_t launch_spectral(float *W, int d, int h, const Layout &L, int n_iters, float attn,
                            float win, float fpm, float wv, float wo, float *sigmas,
                            cudaStream_t st) {
  SpecArgs a{W, d, h, n_iters, L.wq, L.wk, L.wv, L.wo, L.win, L.wx, L.wout,
             attn, win, fpm, wv, wo, sigmas};
  if (d % 128 == 0 && d <= 1024) {
    const int R = d / kSpecCluster;
    const size_t smem = (10 * (size_t)d + (size_t)R + 12) * sizeof(float);
    auto kern = d == 128 ? spectral_sweep_kernel<1> : d == 256 ? spectral_sweep_kernel<2>
              : d == 512 ? spectral_sweep_kernel<4> : spectral_sweep_kernel<8>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((5 * h + 2) * kSpecCluster);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSpecCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
  return cudaErrorInvalidValue;  // the library's d (128, 256, 512, 1024) always takes the cluster kernel
}

// ---------------------------------------------------------------- LM head
__global__ void count_active_kernel(const int32_t *__restrict__ tg, int N, float *out) {
  __shared__ int cnt;
  if (threadIdx.x == 0) cnt = 0;
  __syncthreads();
  int c = 0;
  for (int i = threadIdx.x; i < N; i += blockDim.x) c += tg[i] >= 0;
  atomicAdd(&cnt, c);
  __syncthreads();
  if (threadIdx.x == 0) *out = (float)(cnt > 0 ? cnt : 1);
}

cudaError_t launch_count_active(const int32_t *tg, int N, float *out, cudaStream_t st) {
  count_active_kernel<<<1, 1024, 0, st>>>(tg, N, out);
  return cudaGetLastError();
}

// One block per row, two read passes and one write: pass 1 keeps an online
// (max, sum) of logits + b_lm in base-2 units; pass 2 re-reads the row (an
// L2 hit: the rows of the resident blocks fit in L2) and overwrites it with
// dlogits = (softmax - onehot) / n_active.  Rows start 16-byte aligned
// (ld % 4 == 0); the bias is read with float4 where its address allows.
__global__ void __launch_bounds__(1024) softmax_ce_kernel(float *__restrict__ logits,
                                                          const float *__restrict__ bias,
                                                          const int32_t *__restrict__ tg,
                                                          const float *__restrict__ n_active, int V,
                                                          long ld, float *__restrict__ loss_rows,
                                                          float *__restrict__ lo_out) {
  __shared__ float rm[32], rs[32];
  constexpr float kLog2e = 1.4426950408889634f;
  const int n = blockIdx.x;
  float *row = logits + (size_t)n * ld;
  const int t = tg[n];
  const int V4 = V / 4;
  const bool bias_vec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
  auto load4 = [&](int i) -> float4 {
    const float4 x = *reinterpret_cast<const float4 *>(row + 4 * i);
    const float4 b = bias_vec ? *reinterpret_cast<const float4 *>(bias + 4 * i)
                              : make_float4(bias[4 * i], bias[4 * i + 1], bias[4 * i + 2], bias[4 * i + 3]);
    return make_float4((x.x + b.x) * kLog2e, (x.y + b.y) * kLog2e, (x.z + b.z) * kLog2e,
                       (x.w + b.w) * kLog2e);
  };
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    const float4 x = load4(i);
    const float mx = fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w));
    if (mx > m) { s *= exp2f(m - mx); m = mx; }
    s += exp2f(x.x - m) + exp2f(x.y - m) + exp2f(x.z - m) + exp2f(x.w - m);
  }
  for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) {
    const float x = (row[i] + bias[i]) * kLog2e;
    if (x > m) { s *= exp2f(m - x); m = x; }
    s += exp2f(x - m);
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * exp2f(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * exp2f(m2 - mm));
    m = mm;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { rm[warp] = m; rs[warp] = s; }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < nw; ++w) M = fmaxf(M, rm[w]);
  float S = 0.f;
  for (int w = 0; w < nw; ++w) S += (rm[w] == -INFINITY) ? 0.f : rs[w] * exp2f(rm[w] - M);
  const float inv_na = 1.f / *n_active;
  float *lrow = lo_out ? lo_out + (size_t)n * ld : nullptr;
  if (t < 0 || t >= V) {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      row[i] = 0.f;
      if (lrow) lrow[i] = 0.f;
    }
    if (threadIdx.x == 0) loss_rows[n] = 0.f;
    return;
  }
  const float lt = row[t] + bias[t];
  __syncthreads();  // every thread has read row[t] before it is overwritten
  // loss = -(x_t - ln sum exp x) with M, S in base 2: ln sum = (M + log2 S) ln 2
  if (threadIdx.x == 0) loss_rows[n] = -(lt - (M + log2f(S)) * 0.6931471805599453f) * inv_na;
  const float scale = inv_na / S;
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    const float4 x = load4(i);
    float4 p = make_float4(exp2f(x.x - M) * scale, exp2f(x.y - M) * scale, exp2f(x.z - M) * scale,
                           exp2f(x.w - M) * scale);
    if ((t >> 2) == i) {
      const int j = t & 3;
      if (j == 0) p.x -= inv_na; else if (j == 1) p.y -= inv_na; else if (j == 2) p.z -= inv_na; else p.w -= inv_na;
    }
    if (lrow) {
      float4 h;
      h.x = __uint_as_float(__float_as_uint(p.x) & 0xFFFFE000u);
      h.y = __uint_as_float(__float_as_uint(p.y) & 0xFFFFE000u);
      h.z = __uint_as_float(__float_as_uint(p.z) & 0xFFFFE000u);
      h.w = __uint_as_float(__float_as_uint(p.w) & 0xFFFFE000u);
      *reinterpret_cast<float4 *>(lrow + 4 * i) = make_float4(p.x - h.x, p.y - h.y, p.z - h.z, p.w - h.w);
      p = h;
    }
    *reinterpret_cast<float4 *>(row + 4 * i) = p;
  }
  for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) {
    float p = exp2f((row[i] + bias[i]) * kLog2e - M) * scale;
    if (i == t) p -= inv_na;
    if (lrow) {
      const float h = __uint_as_float(__float_as_uint(p) & 0xFFFFE000u);
      lrow[i] = p - h;
      p = h;
    }
    row[i] = p;
  }
}

cudaError_t launch_softmax_ce(float *logits, const float *bias, const int32_t *tg,
                              const float *n_active, int N, int V, long ld, float *loss_rows, float *lo,
                              cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  softmax_ce_kernel<<<N, 1024, 0, st>>>(logits, bias, tg, n_active, V, ld, loss_rows, lo);
  return cudaGetLastError();
}

// Pre-split variant that also emits column partial sums of dlogits: one
// block of 1024 threads walks `rows` consecutive rows (two read passes and
// one write per row, as softmax_ce_kernel), writes each row as tf32-exact
// high part (in place) + remainder (lo), and adds the row into a per-block
// column accumulator held in shared memory (ld floats, each column owned by
// one thread, so no atomics); the block's sums go to colpart[block][v].
__global__ void __launch_bounds__(1024) softmax_ce_rows_kernel(float *__restrict__ logits,
                                                               const float *__restrict__ bias,
                                                               const int32_t *__restrict__ tg,
                                                               const float *__restrict__ n_active, int N,
                                                               int V, long ld, int rows,
                                                               float *__restrict__ loss_rows,
                                                               float *__restrict__ lo_out,
                                                               float *__restrict__ colpart, int accumulate,
                                                               const float2 *__restrict__ stats) {
  extern __shared__ __align__(16) float colacc[];
  __shared__ float rm[32], rs[32];
  constexpr float kLog2e = 1.4426950408889634f;
  const int V4 = V / 4;
  const int tail = V - 4 * V4;
  const bool bias_vec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float inv_na = 1.f / *n_active;
  for (int i = threadIdx.x; i < V; i += blockDim.x) colacc[i] = 0.f;
  auto bias4 = [&](int i) -> float4 {
    return bias_vec ? *reinterpret_cast<const float4 *>(bias + 4 * i)
                    : make_float4(bias[4 * i], bias[4 * i + 1], bias[4 * i + 2], bias[4 * i + 3]);
  };
  for (int rr = 0; rr < rows; ++rr) {
    const int n = blockIdx.x * rows + rr;
    if (n >= N) break;
    float *row = logits + (size_t)n * ld;
    float *lrow = lo_out + (size_t)n * ld;
    const int t = tg[n];
    float m = -INFINITY, sacc = 0.f;
    if (stats) {  // combine the GEMM epilogue's per-tile statistics
      const int nt = (V + 255) / 256;
      for (int i = threadIdx.x; i < nt; i += blockDim.x) {
        const float2 tsm = stats[(size_t)n * nt + i];
        if (tsm.x == -INFINITY) continue;
        if (tsm.x > m) { sacc = sacc * exp2f(m - tsm.x) + tsm.y; m = tsm.x; }
        else sacc += tsm.y * exp2f(tsm.x - m);
      }
    } else {
      for (int i = threadIdx.x; i < V4; i += blockDim.x) {
        const float4 x4 = *reinterpret_cast<const float4 *>(row + 4 * i);
        const float4 b4 = bias4(i);
        const float4 x = make_float4((x4.x + b4.x) * kLog2e, (x4.y + b4.y) * kLog2e, (x4.z + b4.z) * kLog2e,
                                     (x4.w + b4.w) * kLog2e);
        const float mx = fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w));
        if (mx > m) { sacc *= exp2f(m - mx); m = mx; }
        sacc += exp2f(x.x - m) + exp2f(x.y - m) + exp2f(x.z - m) + exp2f(x.w - m);
      }
      if ((int)threadIdx.x < tail) {
        const int i = 4 * V4 + threadIdx.x;
        const float x = (row[i] + bias[i]) * kLog2e;
        if (x > m) { sacc *= exp2f(m - x); m = x; }
        sacc += exp2f(x - m);
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, sacc, o);
      const float mm = fmaxf(m, m2);
      sacc = (m == -INFINITY ? 0.f : sacc * exp2f(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * exp2f(m2 - mm));
      m = mm;
    }
    __syncthreads();  // the previous row's readers of rm / rs are done
    if (lane == 0) { rm[warp] = m; rs[warp] = sacc; }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, rm[w]);
    float S = 0.f;
    for (int w = 0; w < nw; ++w) S += (rm[w] == -INFINITY) ? 0.f : rs[w] * exp2f(rm[w] - M);
    const bool ignore = t < 0 || t >= V;
    const float lt = ignore ? 0.f : row[t] + bias[t];
    __syncthreads();  // every thread has read row[t] before it is overwritten
    if (threadIdx.x == 0)
      loss_rows[n] = ignore ? 0.f : -(lt - (M + log2f(S)) * 0.6931471805599453f) * inv_na;
    const float scale = ignore ? 0.f : inv_na / S;
    for (int i = threadIdx.x; i < V4; i += blockDim.x) {
      const float4 x4 = *reinterpret_cast<const float4 *>(row + 4 * i);
      const float4 b4 = bias4(i);
      float4 p = make_float4(exp2f((x4.x + b4.x) * kLog2e - M) * scale, exp2f((x4.y + b4.y) * kLog2e - M) * scale,
                             exp2f((x4.z + b4.z) * kLog2e - M) * scale, exp2f((x4.w + b4.w) * kLog2e - M) * scale);
      if (!ignore && (t >> 2) == i) {
        const int j = t & 3;
        if (j == 0) p.x -= inv_na; else if (j == 1) p.y -= inv_na; else if (j == 2) p.z -= inv_na; else p.w -= inv_na;
      }
      float4 *ca = reinterpret_cast<float4 *>(colacc + 4 * i);
      *ca = *ca + p;
      float4 h;
      h.x = __uint_as_float(__float_as_uint(p.x) & 0xFFFFE000u);
      h.y = __uint_as_float(__float_as_uint(p.y) & 0xFFFFE000u);
      h.z = __uint_as_float(__float_as_uint(p.z) & 0xFFFFE000u);
      h.w = __uint_as_float(__float_as_uint(p.w) & 0xFFFFE000u);
      *reinterpret_cast<float4 *>(lrow + 4 * i) = make_float4(p.x - h.x, p.y - h.y, p.z - h.z, p.w - h.w);
      *reinterpret_cast<float4 *>(row + 4 * i) = h;
    }
    if ((int)threadIdx.x < tail) {
      const int i = 4 * V4 + threadIdx.x;
      float p = exp2f((row[i] + bias[i]) * kLog2e - M) * scale;
      if (!ignore && i == t) p -= inv_na;
      colacc[i] += p;
      const float h = __uint_as_float(__float_as_uint(p) & 0xFFFFE000u);
      lrow[i] = p - h;
      row[i] = h;
    }
  }
  float *prow = colpart + (size_t)blockIdx.x * ld;
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    float4 v = *reinterpret_cast<const float4 *>(colacc + 4 * i);
    if (accumulate) v = v + *reinterpret_cast<const float4 *>(prow + 4 * i);
    *reinterpret_cast<float4 *>(prow + 4 * i) = v;
  }
  if ((int)threadIdx.x < tail)
    prow[4 * V4 + threadIdx.x] = colacc[4 * V4 + threadIdx.x] + (accumulate ? prow[4 * V4 + threadIdx.x] : 0.f);
}

namespace {
int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}
}  // namespace

// One wave: as many blocks as SMs (one block per SM: the accumulator takes
// V floats of shared memory), each with ceil(N / blocks) rows.
int softmax_rows_per_block(int N, int max_blocks) {
  const int nsm = max_blocks > 0 && max_blocks < num_sms() ? max_blocks : num_sms();
  return (N + nsm - 1) / nsm;
}
int softmax_rows_blocks(int N, int max_blocks) {
  const int r = softmax_rows_per_block(N, max_blocks);
  return (N + r - 1) / r;
}

cudaError_t launch_softmax_ce_split(float *logits, const float *bias, const int32_t *tg,
                                    const float *n_active, int N, int V, long ld, float *loss_rows,
                                    float *lo, float *colpart, cudaStream_t st, int max_blocks,
                                    bool accumulate, const float2 *stats) {
  if (N <= 0) return cudaSuccess;
  const size_t smem = (size_t)ld * sizeof(float);
  if (ld & 3 || smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(softmax_ce_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  softmax_ce_rows_kernel<<<softmax_rows_blocks(N, max_blocks), 1024, smem, st>>>(
      logits, bias, tg, n_active, N, V, ld, softmax_rows_per_block(N, max_blocks), loss_rows, lo, colpart,
      accumulate ? 1 : 0, stats);
  return cudaGetLastError();
}

// dl_dh = g/r * dy - P * (sum dy*g*P) / (d r^3); ggp = dy * P / r (per-token gain-gradient part)
__global__ void rmsnorm_bwd_kernel(const float *__restrict__ dy, const float *__restrict__ P,
                                   const float *__restrict__ lrms, const float *__restrict__ g,
                                   float *__restrict__ dl_dh, float *__restrict__ ggp, int d) {
  __shared__ __align__(16) float red[512];
  const int n = blockIdx.x, j0 = threadIdx.x * 4;
  const float4 dd = ld4(dy + (size_t)n * d + j0), p = ld4(P + (size_t)n * d + j0), gg = ld4(g + j0);
  const float r = lrms[n];
  const float4 dyg = dd * gg;
  BlockReducer R(red);
  float v[1] = {dot4(dyg, p)};
  R.sum(v);
  const float coef = v[0] / ((float)d * r * r * r);
  const float ir = 1.f / r;
  st4(dl_dh + (size_t)n * d + j0, ir * dyg - coef * p);
  st4(ggp + (size_t)n * d + j0, ir * (dd * p));
}

cudaError_t launch_rmsnorm_bwd(const float *dy, const float *P, const float *lrms, const float *g,
                               float *dl_dh, float *ggp, int N, int d, cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  rmsnorm_bwd_kernel<<<N, d / 4, 0, st>>>(dy, P, lrms, g, dl_dh, ggp, d);
  return cudaGetLastError();
}

__global__ void sum_kernel(const float *__restrict__ x, int n, float *out) {
  __shared__ __align__(16) float red[512];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  BlockReducer R(red);
  float v[1] = {s};
  R.sum(v);
  if (threadIdx.x == 0) *out = v[0];
}

cudaError_t launch_sum(const float *x, int n, float *out, cudaStream_t st) {
  sum_kernel<<<1, 1024, 0, st>>>(x, n, out);
  return cudaGetLastError();
}

}  // namespace aideen
