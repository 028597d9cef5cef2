// Sampled-softmax LM head with its fused Adam step, and the embedding-row Adam
// update: the reference's training step around the DEQ core.
//
//   sample_set      the step's sampled vocabulary S: the distinct valid targets
//                   plus deterministic candidates in draw order, sorted
//                   (gpu_lm_head.rs:213-281), built on the device in one CTA
//                   with a shared-memory bitmap of the vocabulary
//   gather_rows     W_S = W_lm[S] (K x d, zero rows past K)
//   softmax_sampled per token: softmax over the sampled logits (+ b_lm[S]),
//                   loss, and coef = (p - onehot) * valid / active in place
//                   (lm_train.wgsl:79-217)
//   lm_sampled_adam dW_S / db_S clamped to +-0.1, Adam on the sampled rows of
//                   W_lm and b_lm only; the updated rows also land in W_S for
//                   dL/dy (lm_train.wgsl:224-290, 327-395)
//   emb_csr         distinct tokens of the step and their positions, by a
//                   stable block radix sort of (token, position) keys
//                   (gpu_embedding.rs:47-70)
//   emb_adam        mean gradient row per distinct token, Adam on that
//                   embedding row (embedding_train.wgsl:100-147)
#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "kernels.cuh"

namespace aideen {

namespace {

__device__ __forceinline__ uint32_t sample_candidate(unsigned long long seed, uint32_t step,
                                                     unsigned long long draw, uint32_t V) {
  unsigned long long x = seed ^ ((unsigned long long)step * 0x9E3779B97F4A7C15ull) ^
                         (draw * 0xD1B54A32D192ED03ull);
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return (uint32_t)(x % (unsigned long long)V);
}

constexpr int kSetThreads = 1024;

// Block-wide exclusive scan of one int per thread (kSetThreads threads).
__device__ __forceinline__ int block_exclusive_scan(int v, int *sh, int &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;
  }
  __syncthreads();
  total = sh[31];
  const int before = warp ? sh[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

__global__ void __launch_bounds__(kSetThreads) sample_set_kernel(const int32_t *__restrict__ tg, int N, int V,
                                                                 int num_samples, int max_samples,
                                                                 unsigned long long seed, uint32_t step,
                                                                 int32_t *__restrict__ S, int *__restrict__ K_out,
                                                                 float *__restrict__ active_out, int cap,
                                                                 unsigned int *__restrict__ err) {
  extern __shared__ uint32_t bits[];
  __shared__ int sh[32];
  __shared__ int s_valid;
  const int nw = (V + 31) >> 5;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) bits[i] = 0u;
  if (threadIdx.x == 0) s_valid = 0;
  __syncthreads();
  int valid = 0;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int t = tg[i];
    if (t >= 0 && t < V) {
      atomicOr(&bits[t >> 5], 1u << (t & 31));
      ++valid;
    }
  }
  valid = __reduce_add_sync(0xffffffffu, valid);
  if ((threadIdx.x & 31) == 0) atomicAdd(&s_valid, valid);
  __syncthreads();
  int uniq = 0;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) uniq += __popc(bits[i]);
  int total = 0;
  block_exclusive_scan(uniq, sh, total);
  int desired = num_samples > N ? num_samples : N;
  desired = desired < V ? desired : V;
  desired = desired < max_samples ? desired : max_samples;
  if (threadIdx.x < 32) {
    // fill with candidates in draw order: one warp, 32 draws at a time; the
    // first of equal candidates in a round wins, present ids are skipped
    const int lane = threadIdx.x;
    int taken = 0;
    const int need = desired - total;
    unsigned long long base = 0;
    while (taken < need) {
      if (base >= (1ull << 26)) {  // far beyond any vocabulary's needs: give up
        if (lane == 0) atomicExch(err, 1u);
        break;
      }
      const uint32_t c = sample_candidate(seed, step, base + lane, (uint32_t)V);
      const bool present = (bits[c >> 5] >> (c & 31)) & 1u;
      const unsigned peers = __match_any_sync(0xffffffffu, c);
      const bool first = (__ffs(peers) - 1) == lane;
      unsigned mask = __ballot_sync(0xffffffffu, !present && first);
      int rem = need - taken;
      while (__popc(mask) > rem) mask &= ~(1u << (31 - __clz(mask)));
      if ((mask >> lane) & 1u) atomicOr(&bits[c >> 5], 1u << (c & 31));
      taken += __popc(mask);
      base += 32;
      __syncwarp();
    }
  }
  __syncthreads();
  // compaction in ascending id order: each thread owns a contiguous run of words
  const int per = (nw + blockDim.x - 1) / blockDim.x;
  const int w0 = threadIdx.x * per, w1 = min(nw, w0 + per);
  int cnt = 0;
  for (int i = w0; i < w1; ++i) cnt += __popc(bits[i]);
  int K = 0;
  int o = block_exclusive_scan(cnt, sh, K);
  for (int i = w0; i < w1; ++i) {
    uint32_t w = bits[i];
    while (w) {
      const int b = __ffs(w) - 1;
      w &= w - 1;
      if (o < cap) S[o] = i * 32 + b;
      ++o;
    }
  }
  if (threadIdx.x == 0) {
    if (K > cap) atomicExch(err, 2u);
    *K_out = K < cap ? K : cap;
    *active_out = (float)(s_valid > 0 ? s_valid : 1);
  }
}

__global__ void gather_rows_kernel(const float *__restrict__ W, const int32_t *__restrict__ S,
                                   const int *__restrict__ K, int d, float *__restrict__ WS) {
  const int k = blockIdx.x;
  const bool live = k < *K;
  const float *src = W + (size_t)(live ? S[k] : 0) * d;
  for (int j = threadIdx.x * 4; j < d; j += blockDim.x * 4)
    st4(WS + (size_t)k * d + j, live ? ld4(src + j) : f4(0.f));
}

// One CTA per token row of logits [N][ld] (ld = K cap): softmax over the
// first K sampled logits (+ b_lm[S]), loss row (already divided by the active
// count), coef = (p - onehot) * valid / active in place (zero past K).
__global__ void __launch_bounds__(256) softmax_sampled_kernel(float *__restrict__ logits, long ld,
                                                              const float *__restrict__ b_lm,
                                                              const int32_t *__restrict__ S,
                                                              const int *__restrict__ Kp,
                                                              const int32_t *__restrict__ tg, int V,
                                                              const float *__restrict__ active,
                                                              float *__restrict__ loss_rows) {
  __shared__ float red[2 * 8 * 32];
  __shared__ float wm[8];
  __shared__ int s_tk;
  __shared__ float s_et;
  const int n = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = *Kp;
  float *row = logits + (size_t)n * ld;
  const int t = tg[n];
  const bool valid = t >= 0 && t < V;
  if (threadIdx.x == 0) {
    s_tk = -1;
    s_et = 0.f;
  }
  __syncthreads();
  float mx = -3.4e38f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int v = S[k];
    const float z = row[k] + b_lm[v];
    row[k] = z;
    mx = fmaxf(mx, z);
    if (v == t) s_tk = k;  // S holds distinct ids: at most one writer
  }
  mx = warp_max(mx);
  if (lane == 0) wm[warp] = mx;
  __syncthreads();
  mx = wm[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, wm[w]);
  const int tk = s_tk;
  float se = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float e = __expf(row[k] - mx);
    row[k] = e;
    se += e;
    if (k == tk) s_et = e;
  }
  BlockReducer R(red);
  float v1[1] = {se};
  R.sum(v1);
  const float inv = 1.f / fmaxf(v1[0], 1e-10f);
  const float sc = valid ? 1.f / *active : 0.f;
  for (int k = threadIdx.x; k < (int)ld; k += blockDim.x) {
    float c = 0.f;
    if (k < K) c = (row[k] * inv - (k == tk ? 1.f : 0.f)) * sc;
    row[k] = c;
  }
  if (threadIdx.x == 0) loss_rows[n] = (valid && tk >= 0) ? -logf(fmaxf(s_et * inv, 1e-10f)) * sc : 0.f;
}

// Adam on the sampled rows: thread (k, j), j < d weight element, j == d bias.
__global__ void lm_sampled_adam_kernel(float *__restrict__ W, float *__restrict__ b, float *__restrict__ M1,
                                       float *__restrict__ M2, size_t off_b, const float *__restrict__ dW,
                                       const float *__restrict__ db, const int32_t *__restrict__ S,
                                       const int *__restrict__ Kp, int d, float *__restrict__ WS, float lr,
                                       float b1, float b2, float eps, float bc1, float bc2) {
  const int k = blockIdx.y;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= *Kp || j > d) return;
  const int v = S[k];
  float g;
  size_t idx;
  float *wp;
  if (j < d) {
    g = dW[(size_t)k * d + j];
    idx = (size_t)v * d + j;
    wp = W + idx;
  } else {
    g = db[k];
    idx = off_b + v;
    wp = b + v;
  }
  g = fminf(fmaxf(g, -0.1f), 0.1f);
  const float m = b1 * M1[idx] + (1.f - b1) * g;
  const float s = b2 * M2[idx] + (1.f - b2) * g * g;
  M1[idx] = m;
  M2[idx] = s;
  const float w = *wp - lr * (m / bc1) / (sqrtf(s / bc2) + eps);
  *wp = w;
  if (j < d) WS[(size_t)k * d + j] = w;
}

constexpr int kCsrThreads = 1024, kCsrItems = 16;

// Distinct tokens (ids clamped to V - 1) and their positions, sorted by
// (token, position): uniq[U], off[U + 1], pos[N]; U lands in *U_out.
__global__ void __launch_bounds__(kCsrThreads) emb_csr_kernel(const int32_t *__restrict__ tok, int N, int V,
                                                              int32_t *__restrict__ uniq, int32_t *__restrict__ off,
                                                              int32_t *__restrict__ pos, int *__restrict__ U_out) {
  using Sort = cub::BlockRadixSort<unsigned long long, kCsrThreads, kCsrItems>;
  using Scan = cub::BlockScan<int, kCsrThreads>;
  union Tmp {
    typename Sort::TempStorage sort;
    typename Scan::TempStorage scan;
  };
  // the sort's scratch exceeds the 48 KB of static shared memory: dynamic
  extern __shared__ __align__(16) unsigned char csr_smem[];
  Tmp &tmp = *reinterpret_cast<Tmp *>(csr_smem);
  unsigned long long *last_key =
      reinterpret_cast<unsigned long long *>(csr_smem + (sizeof(Tmp) + 15) / 16 * 16);
  unsigned long long key[kCsrItems];
#pragma unroll
  for (int i = 0; i < kCsrItems; ++i) {
    const int p = threadIdx.x * kCsrItems + i;
    if (p < N) {
      int t = tok[p];
      t = t < 0 ? 0 : (t > V - 1 ? V - 1 : t);
      key[i] = ((unsigned long long)(uint32_t)t << 32) | (uint32_t)p;
    } else {
      key[i] = ~0ull;  // sorts after every real key
    }
  }
  Sort(tmp.sort).Sort(key);  // blocked arrangement: thread x holds ranks x*ITEMS + i
  __syncthreads();
  last_key[threadIdx.x] = key[kCsrItems - 1];
  __syncthreads();
  int head[kCsrItems];
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < kCsrItems; ++i) {
    const int r = threadIdx.x * kCsrItems + i;
    const unsigned long long prev = i ? key[i - 1] : (threadIdx.x ? last_key[threadIdx.x - 1] : ~0ull);
    head[i] = r < N && (r == 0 || (prev >> 32) != (key[i] >> 32));
    cnt += head[i];
  }
  int base = 0, U = 0;
  Scan(tmp.scan).ExclusiveSum(cnt, base, U);
#pragma unroll
  for (int i = 0; i < kCsrItems; ++i) {
    const int r = threadIdx.x * kCsrItems + i;
    if (r >= N) continue;
    pos[r] = (int32_t)(key[i] & 0xffffffffu);
    if (head[i]) {
      uniq[base] = (int32_t)(key[i] >> 32);
      off[base] = r;
      ++base;
    }
  }
  if (threadIdx.x == 0) {
    off[U] = N;
    *U_out = U;
  }
}

// One CTA per distinct token: mean of its positions' gradient rows, Adam on
// the embedding row.
__global__ void emb_adam_kernel(float *__restrict__ emb, float *__restrict__ M1, float *__restrict__ M2,
                                const float *__restrict__ grad, const int32_t *__restrict__ uniq,
                                const int32_t *__restrict__ off, const int32_t *__restrict__ pos,
                                const int *__restrict__ Up, int d, float lr, float b1, float b2, float eps,
                                float bc1, float bc2) {
  const int u = blockIdx.x;
  if (u >= *Up) return;
  const int t = uniq[u], o0 = off[u], o1 = off[u + 1];
  const float ic = 1.f / (float)(o1 - o0 > 0 ? o1 - o0 : 1);
  for (int j = threadIdx.x * 4; j < d; j += blockDim.x * 4) {
    // eight independent partial sums (positions q = o0 + 8i + r), combined in
    // a fixed order: a frequent token's rows stream with 8 loads in flight
    float4 gp[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) gp[r] = f4(0.f);
    int q = o0;
    for (; q + 8 <= o1; q += 8) {
#pragma unroll
      for (int r = 0; r < 8; ++r) gp[r] = gp[r] + ld4(grad + (size_t)pos[q + r] * d + j);
    }
    for (int r = 0; q < o1; ++q, ++r) gp[r] = gp[r] + ld4(grad + (size_t)pos[q] * d + j);
    float4 g = ((gp[0] + gp[1]) + (gp[2] + gp[3])) + ((gp[4] + gp[5]) + (gp[6] + gp[7]));
    g = ic * g;
    const size_t idx = (size_t)t * d + j;
    float4 m = ld4(M1 + idx), s = ld4(M2 + idx), w = ld4(emb + idx);
    m = fma4(f4(1.f - b1), g, f4(b1) * m);
    s = fma4(f4(1.f - b2), g * g, f4(b2) * s);
    w.x -= lr * (m.x / bc1) / (sqrtf(s.x / bc2) + eps);
    w.y -= lr * (m.y / bc1) / (sqrtf(s.y / bc2) + eps);
    w.z -= lr * (m.z / bc1) / (sqrtf(s.z / bc2) + eps);
    w.w -= lr * (m.w / bc1) / (sqrtf(s.w / bc2) + eps);
    st4(M1 + idx, m);
    st4(M2 + idx, s);
    st4(emb + idx, w);
  }
}

}  // namespace

cudaError_t launch_sample_set(const int32_t *tg, int N, int V, int num_samples, int max_samples,
                              unsigned long long seed, uint32_t step, int32_t *S, int *K, float *active, int cap,
                              unsigned int *err, cudaStream_t st) {
  const size_t smem = (size_t)((V + 31) / 32) * 4;
  cudaError_t e = cudaFuncSetAttribute(sample_set_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  sample_set_kernel<<<1, kSetThreads, smem, st>>>(tg, N, V, num_samples, max_samples, seed, step, S, K, active,
                                                  cap, err);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float *W, const int32_t *S, const int *K, int cap, int d, float *WS,
                               cudaStream_t st) {
  if (cap <= 0) return cudaSuccess;
  gather_rows_kernel<<<cap, d / 4 < 256 ? d / 4 : 256, 0, st>>>(W, S, K, d, WS);
  return cudaGetLastError();
}

cudaError_t launch_softmax_sampled(float *logits, long ld, const float *b_lm, const int32_t *S, const int *K,
                                   const int32_t *tg, int V, const float *active, float *loss_rows, int N,
                                   cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  softmax_sampled_kernel<<<N, 256, 0, st>>>(logits, ld, b_lm, S, K, tg, V, active, loss_rows);
  return cudaGetLastError();
}

cudaError_t launch_lm_sampled_adam(float *W, float *b, float *M1, float *M2, size_t off_b, const float *dW,
                                   const float *db, const int32_t *S, const int *K, int cap, int d, float *WS,
                                   float lr, float b1, float b2, float eps, float bc1, float bc2, cudaStream_t st) {
  if (cap <= 0) return cudaSuccess;
  dim3 grid((d + 1 + 255) / 256, cap);
  lm_sampled_adam_kernel<<<grid, 256, 0, st>>>(W, b, M1, M2, off_b, dW, db, S, K, d, WS, lr, b1, b2, eps, bc1, bc2);
  return cudaGetLastError();
}

int emb_csr_max_tokens() { return kCsrThreads * kCsrItems; }

cudaError_t launch_emb_csr(const int32_t *tok, int N, int V, int32_t *uniq, int32_t *off, int32_t *pos, int *U,
                           cudaStream_t st) {
  if (N <= 0 || N > kCsrThreads * kCsrItems) return cudaErrorInvalidValue;
  using Sort = cub::BlockRadixSort<unsigned long long, kCsrThreads, kCsrItems>;
  using Scan = cub::BlockScan<int, kCsrThreads>;
  union Tmp {
    typename Sort::TempStorage sort;
    typename Scan::TempStorage scan;
  };
  const size_t smem = (sizeof(Tmp) + 15) / 16 * 16 + kCsrThreads * sizeof(unsigned long long);
  cudaError_t e = cudaFuncSetAttribute(emb_csr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  emb_csr_kernel<<<1, kCsrThreads, smem, st>>>(tok, N, V, uniq, off, pos, U);
  return cudaGetLastError();
}

cudaError_t launch_emb_adam(float *emb, float *M1, float *M2, const float *grad, const int32_t *uniq,
                            const int32_t *off, const int32_t *pos, const int *U, int ucap, int d, float lr,
                            float b1, float b2, float eps, float bc1, float bc2, cudaStream_t st) {
  if (ucap <= 0) return cudaSuccess;
  emb_adam_kernel<<<ucap, d / 4 < 256 ? d / 4 : 256, 0, st>>>(emb, M1, M2, grad, uniq, off, pos, U, d, lr, b1, b2,
                                                              eps, bc1, bc2);
  return cudaGetLastError();
}

}  // namespace aideen
