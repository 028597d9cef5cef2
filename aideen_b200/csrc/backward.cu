// Backward of the AIDEEN slot block on sm_100a.
//
//   adjoint          fused clean Picard adjoint: all `iters` iterations of
//                    v' = rhs + beta*J_norm^T v + (1-beta) v run on-chip, one
//                    warp per (token, slot) entry and one CTA per token so the
//                    optional Anderson mixing can form its per-token Gram
//                    (staged_adjoint_picard_clean.wgsl:143-248, 1011-1135).
//                    HBM traffic: pre + rhs in, v + g_pre out, once.
//   source_grad      sum_s beta*J_norm^T v (picard_source_grad_reduce_main, :250-327)
//   attn_bwd_scale   d(attn*scale)/d(attn, R) per entry
//   attn_bwd_softmax per-token softmax / mean-subtracted mix backward
//   dsig_init        dL/dsignal = g_pre + dL/dR * dR/dsrc
//   colsum           column sums (bias / anchor / NormScale gradients)
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace aideen {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

constexpr uint32_t kSpinLimit = 1u << 26;

// Set when a bounded wait of the adjoint ran out (the rows of that CTA's
// remaining tokens were not written); read and cleared by adjoint_error_async.
// Anderson iterates in registers instead of the shared-memory ring (a tuning
// switch read once per process).
static bool adj_reg_hist() {
  static const bool on = getenv("AIDEEN_ADJ_REG_HIST") != nullptr;
  return on;
}

__device__ unsigned int g_adjoint_error;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint32_t limit = kSpinLimit) {
  const uint32_t addr = smem_addr(bar);
  for (uint32_t i = 0; i < limit; ++i) {
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

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Persistent fused clean adjoint.  Each CTA walks tokens n = blockIdx.x,
// blockIdx.x + gridDim.x, ...; while a token's h warps (one per slot) run all
// `iters` iterations in registers, thread 0 has the next token's inputs
// (pre parts, per-slot RHS, pooled RHS row) streaming into the other half of a
// double-buffered shared-memory stage with cp.async.bulk, so HBM traffic
// overlaps the on-chip iterations.  Waits are bounded.
// Anderson weights of one token: block-reduce the Gram of the pseudo-residuals
// (g6 = this warp's partials <d0,d0>, <d0,d1>, <d0,d2>, <d1,d1>, <d1,d2>,
// <d2,d2>) over the token's h*d iterate, then anderson_solve
// (staged_adjoint_picard_clean.wgsl:1022-1135).  buf: 96 floats of shared memory.
template <int MA>
__device__ __forceinline__ void anderson_coefs(float (&g6)[6], int n_res, float *buf, int s, int lane, int h,
                                               float &b0, float &b1, float &b2) {
  b2 = 0.f;
#pragma unroll
  for (int q = 0; q < 6; ++q) {
    const float x = warp_sum(g6[q]);
    if (lane == 0) buf[q * 16 + s] = x;
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 6; ++q) {
    float t = 0.f;
    for (int w = 0; w < h; ++w) t += buf[q * 16 + w];
    g6[q] = t;
  }
  anderson_solve(g6, n_res, b0, b1, b2);
}

// HS: the Anderson iterates live in a shared-memory ring ([MA][h][d], each
// thread touching only its own elements) instead of registers, which leaves
// room for two CTAs (two tokens) per SM.
template <int F, int MA, int MAXT, int MINB, bool HS = false>
__global__ void __launch_bounds__(MAXT, MINB) adjoint_kernel(AdjointArgs a) {
  extern __shared__ __align__(128) unsigned char smraw[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smraw);  // [2]
  float *gram = reinterpret_cast<float *>(smraw + 128);  // [2][6][16]
  const int s = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.d, h = a.h;
  const size_t hd = (size_t)h * d;
  const int has_b = a.pre_b != nullptr, has_rs = a.rhs_slot != nullptr, has_tok = a.rhs_tok != nullptr;
  const size_t stage_f = hd * (1 + has_b + has_rs) + (has_tok ? d : 0);
  float *stage0 = gram + 192;
  // NormScale partials [h][d] reuse the current token's stage, consumed by then.
  const float beta = a.beta;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar[0])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar[1])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int n, int b) {
    float *st = stage0 + b * stage_f;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&bar[b])),
                 "r"((uint32_t)(stage_f * 4))
                 : "memory");
    size_t o = 0;
    bulk_g2s(st, a.pre_a + (size_t)n * hd, (uint32_t)(hd * 4), &bar[b]);
    o += hd;
    if (has_b) { bulk_g2s(st + o, a.pre_b + (size_t)n * hd, (uint32_t)(hd * 4), &bar[b]); o += hd; }
    if (has_rs) { bulk_g2s(st + o, a.rhs_slot + (size_t)n * hd, (uint32_t)(hd * 4), &bar[b]); o += hd; }
    if (has_tok) bulk_g2s(st + o, a.rhs_tok + (size_t)n * d, (uint32_t)(d * 4), &bar[b]);
  };
  if (threadIdx.x == 0 && (int)blockIdx.x < a.N) issue(blockIdx.x, 0);
  int it = 0;
  // per-CTA NormScale-gradient partial of this warp's slot, summed over the
  // CTA's tokens (nsg_cta mode)
  float4 nsv[F];
#pragma unroll
  for (int f = 0; f < F; ++f) nsv[f] = f4(0.f);
  for (int n = blockIdx.x; n < a.N; n += gridDim.x, ++it) {
    const int b = it & 1;
    const int nn = n + (int)gridDim.x;
    if (threadIdx.x == 0 && nn < a.N) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(nn, b ^ 1);
    }
    const bool ok = mbar_wait_bounded(&bar[b], (it >> 1) & 1, a.spin_limit);
    if (!__syncthreads_and(ok)) {
      // Give up on this CTA's remaining tokens: record the error, then let the
      // copies already issued into both stages land (bounded) before exiting.
      if (threadIdx.x == 0) {
        atomicExch(&g_adjoint_error, 1u);
        mbar_wait_bounded(&bar[b], (it >> 1) & 1);
        if (nn < a.N) mbar_wait_bounded(&bar[b ^ 1], ((it + 1) >> 1) & 1);
      }
      return;
    }
    const float *sa = stage0 + b * stage_f;
    float *nsacc = stage0 + b * stage_f;
    const float *sb = sa + hd;
    const float *srs = sa + hd * (1 + has_b);
    const float *st_tok = sa + hd * (1 + has_b + has_rs);
    const size_t e = ((size_t)n * h + s) * d;
    float4 pre[F], rhs[F], ns[F], v[F];
    float ss = 0.f;
    const float ih = 1.f / (float)h;
  #pragma unroll
    for (int f = 0; f < F; ++f) {
      const int j = (f * 32 + lane) * 4;
      pre[f] = ld4(sa + (size_t)s * d + j);
      if (a.pre_b) pre[f] = pre[f] + ld4(sb + (size_t)s * d + j);
      ns[f] = ld4(a.NS + j);
      float4 r = f4(0.f);
      if (a.rhs_tok) r = ih * ld4(st_tok + j);
      if (a.rhs_slot) r = r + ld4(srs + (size_t)s * d + j);
      rhs[f] = r;
      v[f] = r;
      ss += dot4(pre[f], pre[f]);
    }
    ss = warp_sum(ss);
    __syncthreads();  // this token's stage is consumed; it may be refilled
    const float rms = sqrtf(ss / (float)d + 1e-6f);
    const float inv = 1.f / fmaxf(rms, 1e-6f);
    const float den = fmaxf((float)d * rms * rms * rms, 1e-6f);
    const float inv_den = 1.f / den;
    // The step is diagonal + rank one: v' = rhs + a*v - ((w . v) / den) * pre with
    // a = beta*NS/rms + (1 - beta) and w = beta*NS*pre, so each iteration costs
    // three FMAs per element plus one warp reduction.
    float4 av[F], wv[F];
  #pragma unroll
    for (int f = 0; f < F; ++f) {
      av[f] = (beta * inv) * ns[f] + f4(1.f - beta);
      wv[f] = beta * (ns[f] * pre[f]);
    }
    float4 hist[(MA > 0 && !HS) ? MA : 1][F];
    float *ring = stage0 + 2 * stage_f + (size_t)s * d;  // HS: iterate slot q at ring + q * hd
    int k0 = 0;
    if constexpr (MA == 0) {
      // Two iterations per warp reduction.  With u = w (*) a,
      //   c_k     = w . v_k,
      //   c_{k+1} = w . v_{k+1} = w.rhs + u . v_k + ncs_k * w.pre,
      // so w . v_k and u . v_k, reduced together (one exchange splits the two
      // sums between the half-warps, four more finish them, one more shares
      // them back), give both steps' scalars: about half the reduction
      // instructions per iteration, which with the FMAs bounds this kernel at
      // 20 iterations (the FMA pipe and the issue slots, not HBM).
      float wr = 0.f, wp = 0.f;
#pragma unroll
      for (int f = 0; f < F; ++f) {
        wr += dot4(wv[f], rhs[f]);
        wp += dot4(wv[f], pre[f]);
      }
      wr = warp_sum(wr);
      wp = warp_sum(wp);
      float4 u[F];
#pragma unroll
      for (int f = 0; f < F; ++f) u[f] = wv[f] * av[f];
      const bool upper = (lane & 16) != 0;
      for (; k0 + 2 <= a.iters; k0 += 2) {
        float A0 = 0.f, A1 = 0.f, B0 = 0.f, B1 = 0.f;
#pragma unroll
        for (int f = 0; f < F; ++f) {
          A0 = fmaf(wv[f].x, v[f].x, A0); A1 = fmaf(wv[f].y, v[f].y, A1);
          A0 = fmaf(wv[f].z, v[f].z, A0); A1 = fmaf(wv[f].w, v[f].w, A1);
          B0 = fmaf(u[f].x, v[f].x, B0); B1 = fmaf(u[f].y, v[f].y, B1);
          B0 = fmaf(u[f].z, v[f].z, B0); B1 = fmaf(u[f].w, v[f].w, B1);
        }
        const float A = A0 + A1, Bq = B0 + B1;
        // lanes < 16 keep A, lanes >= 16 keep B; each sends the other half's value
        float x = (upper ? Bq : A) + __shfl_xor_sync(0xffffffffu, upper ? A : Bq, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        const float y = __shfl_xor_sync(0xffffffffu, x, 16);
        const float Asum = upper ? y : x, Bsum = upper ? x : y;
        const float ncs0 = -Asum * inv_den;
        const float ncs1 = -(wr + Bsum + ncs0 * wp) * inv_den;
        const float4 n0 = f4(ncs0), n1 = f4(ncs1);
#pragma unroll
        for (int f = 0; f < F; ++f) {
          const float4 v1 = fma4(n0, pre[f], fma4(av[f], v[f], rhs[f]));
          v[f] = fma4(n1, pre[f], fma4(av[f], v1, rhs[f]));
        }
      }
    }
    for (int k = k0; k < a.iters; ++k) {
      // w . v in two float4 partial sums (ILP), packed FMAs throughout
      float4 c0 = f4(0.f), c1 = f4(0.f);
#pragma unroll
      for (int f = 0; f < F; ++f) {
        if (f & 1) c1 = dot4_acc(c1, wv[f], v[f]);
        else c0 = dot4_acc(c0, wv[f], v[f]);
      }
      const float ncs = -warp_sum(hsum4(c0) + hsum4(c1)) * inv_den;
      const float4 nc4 = f4(ncs);
  #pragma unroll
      for (int f = 0; f < F; ++f) v[f] = fma4(nc4, pre[f], fma4(av[f], v[f], rhs[f]));
      if constexpr (MA > 0 && HS) {
        // hist i steps ago = ring slot (k - i) mod MA; this iterate goes to slot k mod MA
#pragma unroll
        for (int f = 0; f < F; ++f) st4(ring + (size_t)(k % MA) * hd + (f * 32 + lane) * 4, v[f]);
        const int n_res = k < MA - 1 ? k : MA - 1;
        if (k >= 2 && n_res >= 2) {
          const float *r1 = ring + (size_t)((k + MA - 1) % MA) * hd;
          const float *r2 = ring + (size_t)((k + MA - 2) % MA) * hd;
          const float *r3 = ring + (size_t)((k + MA - 3) % MA) * hd;
          float g6[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  #pragma unroll
          for (int f = 0; f < F; ++f) {
            const int j = (f * 32 + lane) * 4;
            const float4 h1 = ld4(r1 + j), h2 = ld4(r2 + j);
            const float4 d0 = v[f] - h1;
            const float4 d1 = h1 - h2;
            g6[0] += dot4(d0, d0);
            g6[1] += dot4(d0, d1);
            g6[3] += dot4(d1, d1);
            if (MA > 3 && n_res == 3) {
              const float4 d2 = h2 - ld4(r3 + j);
              g6[2] += dot4(d0, d2);
              g6[4] += dot4(d1, d2);
              g6[5] += dot4(d2, d2);
            }
          }
          float b0, b1, b2;
          anderson_coefs<MA>(g6, n_res, gram + (k & 1) * 96, s, lane, h, b0, b1, b2);
  #pragma unroll
          for (int f = 0; f < F; ++f) {
            const int j = (f * 32 + lane) * 4;
            float4 mixed = b0 * v[f] + b1 * ld4(r1 + j);
            if (MA > 3 && n_res == 3) mixed = mixed + b2 * ld4(r2 + j);
            v[f] = mixed;
          }
        }
      } else if constexpr (MA > 0) {
        // ring buffer as a shift register: hist[i] = iterate stored i steps ago
  #pragma unroll
        for (int i = MA - 1; i > 0; --i)
  #pragma unroll
          for (int f = 0; f < F; ++f) hist[i][f] = hist[i - 1][f];
  #pragma unroll
        for (int f = 0; f < F; ++f) hist[0][f] = v[f];
        const int n_res = k < MA - 1 ? k : MA - 1;
        if (k >= 2 && n_res >= 2) {
          // Gram of pseudo-residuals D_i = hist[i] - hist[i+1] over all h*d of the token
          float g6[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  #pragma unroll
          for (int f = 0; f < F; ++f) {
            const float4 d0 = hist[0][f] - hist[1][f];
            const float4 d1 = hist[1][f] - hist[MA > 2 ? 2 : 1][f];
            g6[0] += dot4(d0, d0);
            g6[1] += dot4(d0, d1);
            g6[3] += dot4(d1, d1);
            if (MA > 3 && n_res == 3) {
              const float4 d2 = hist[MA > 3 ? 2 : 1][f] - hist[MA > 3 ? 3 : 1][f];
              g6[2] += dot4(d0, d2);
              g6[4] += dot4(d1, d2);
              g6[5] += dot4(d2, d2);
            }
          }
          float b0, b1, b2;
          anderson_coefs<MA>(g6, n_res, gram + (k & 1) * 96, s, lane, h, b0, b1, b2);
  #pragma unroll
          for (int f = 0; f < F; ++f) {
            float4 mixed = b0 * hist[0][f] + b1 * hist[1][f];
            if (MA > 3 && n_res == 3) mixed = mixed + b2 * hist[MA > 3 ? 2 : 1][f];
            v[f] = mixed;
          }
        }
      }
    }
    float c = 0.f;
  #pragma unroll
    for (int f = 0; f < F; ++f) c += dot4(wv[f], v[f]);
    const float cs = warp_sum(c) / den;
    const size_t vbase = ((size_t)s * (a.v_ld ? a.v_ld : a.N) + n) * d;
  #pragma unroll
    for (int f = 0; f < F; ++f) {
      const int j = (f * 32 + lane) * 4;
      st4(a.v + vbase + j, v[f]);
      // g_pre = beta*J_norm^T v = (a - (1 - beta)) * v - (w . v / den) * pre
      if (a.gpre) st4(a.gpre + e + j, (av[f] - f4(1.f - beta)) * v[f] - cs * pre[f]);
      if (a.nsg) st4(nsacc + (size_t)s * d + j, (beta * inv) * (v[f] * pre[f]));
      if (a.nsg_cta) nsv[f] = fma4(f4(beta * inv), v[f] * pre[f], nsv[f]);
    }
    if (a.nsg) {
      __syncthreads();
      for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float t = 0.f;
        for (int q = 0; q < h; ++q) t += nsacc[(size_t)q * d + j];
        a.nsg[(size_t)n * d + j] = t;
      }
      __syncthreads();  // nsacc (this stage) is read before thread 0 refills it
    }
  }
  if (a.nsg_cta) {
    // sum the slots' partials through shared memory (every stage is consumed)
    __syncthreads();
#pragma unroll
    for (int f = 0; f < F; ++f) st4(stage0 + (size_t)s * d + (f * 32 + lane) * 4, nsv[f]);
    __syncthreads();
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
      float t = 0.f;
      for (int q = 0; q < h; ++q) t += stage0[(size_t)q * d + j];
      a.nsg_cta[(size_t)blockIdx.x * d + j] = t;
    }
  }
}

template <int F, int MA, int MAXT, int MINB, bool HS = false>
static cudaError_t adjoint_launch(const AdjointArgs &a, cudaStream_t st, int *grid_out) {
  const size_t hd = (size_t)a.h * a.d;
  const size_t stage_f = hd * (1 + (a.pre_b != nullptr) + (a.rhs_slot != nullptr)) +
                         (a.rhs_tok ? (size_t)a.d : 0);
  const size_t smem = 128 + 192 * 4 + 2 * stage_f * 4 + (HS ? (size_t)MA * hd * 4 : 0);
  auto k = adjoint_kernel<F, MA, MAXT, MINB, HS>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0, dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 32 * a.h, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int cap = (a.max_ctas > 0 && a.max_ctas < sms ? a.max_ctas : sms) * per_sm;
  const int grid = a.N < cap ? a.N : cap;
  if (grid_out) *grid_out = grid;
  k<<<grid, 32 * a.h, smem, st>>>(a);
  return cudaGetLastError();
}

template <int F>
static cudaError_t adjoint_dispatch_m(const AdjointArgs &a, cudaStream_t st, int *g) {
  const int ma = a.anderson_m <= 2 ? 0 : a.anderson_m;  // m <= 2 never mixes (n_res < 2)
  const bool small = a.h <= 8;
  switch (ma) {
    case 0: return small ? adjoint_launch<F, 0, 256, 2>(a, st, g) : adjoint_launch<F, 0, 512, 1>(a, st, g);
    case 3: return small ? adjoint_launch<F, 3, 256, 1>(a, st, g) : adjoint_launch<F, 3, 512, 1>(a, st, g);
    case 4:
      // iterates in shared memory (two tokens per SM) while two CTAs' rings and
      // stages fit: 4 x h x d floats of ring per CTA
      if (small && 4 * (size_t)a.h * a.d <= 16384 && !adj_reg_hist())
        return adjoint_launch<F, 4, 256, 2, true>(a, st, g);
      return small ? adjoint_launch<F, 4, 256, 1>(a, st, g) : adjoint_launch<F, 4, 512, 1>(a, st, g);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_adjoint(const AdjointArgs &a0, cudaStream_t st, int *g) {
  if (g) *g = 0;
  if (a0.N <= 0) return cudaSuccess;
  AdjointArgs a = a0;
  // AIDEEN_ADJ_SPIN_LIMIT shortens the stage waits (0: every first wait gives
  // up at once), so tests can drive the timeout path without a fault
  a.spin_limit = kSpinLimit;
  if (const char *e = getenv("AIDEEN_ADJ_SPIN_LIMIT")) a.spin_limit = (uint32_t)strtoul(e, nullptr, 10);
  switch (a.d) {
    case 128: return adjoint_dispatch_m<1>(a, st, g);
    case 256: return adjoint_dispatch_m<2>(a, st, g);
    case 512: return adjoint_dispatch_m<4>(a, st, g);
    case 1024: return adjoint_dispatch_m<8>(a, st, g);
    default: return cudaErrorInvalidValue;
  }
}

unsigned int *adjoint_error_dev() {
  void *p = nullptr;
  return cudaGetSymbolAddress(&p, g_adjoint_error) == cudaSuccess ? static_cast<unsigned int *>(p) : nullptr;
}

cudaError_t adjoint_error_async(unsigned int *host_flag, cudaStream_t st) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(host_flag, g_adjoint_error, sizeof(unsigned int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  static const unsigned int zero = 0;
  return cudaMemcpyToSymbolAsync(g_adjoint_error, &zero, sizeof(unsigned int), 0, cudaMemcpyHostToDevice, st);
}

size_t adjoint_smem_bytes(int h, int d, bool has_b, bool has_rs, bool has_tok, int anderson_m) {
  const size_t hd = (size_t)h * d;
  const size_t stage_f = hd * (1 + has_b + has_rs) + (has_tok ? (size_t)d : 0);
  const bool hs = anderson_m == 4 && h <= 8 && 4 * hd <= 16384 && !adj_reg_hist();
  return 128 + 192 * 4 + 2 * stage_f * 4 + (hs ? 4 * hd * 4 : 0);
}

__global__ void source_grad_kernel(const float *__restrict__ gpre, float *__restrict__ out, int h,
                                   int d) {
  const int n = blockIdx.x;
  for (int j = threadIdx.x * 4; j < d; j += blockDim.x * 4) {
    float4 acc = f4(0.f);
    for (int s = 0; s < h; ++s) acc = acc + ld4(gpre + ((size_t)n * h + s) * d + j);
    st4(out + (size_t)n * d + j, acc);
  }
}

cudaError_t launch_source_grad(const float *gpre, float *out, int N, int h, int d, cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  source_grad_kernel<<<N, d / 4, 0, st>>>(gpre, out, h, d);
  return cudaGetLastError();
}

// One warp per (token, slot): backward of A = attn * max(R,1e-3)/max(rho,1e-6).
__global__ void attn_bwd_scale_kernel(AttnBwdArgs a, int rows) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const int d = a.d;
  const float *gA = a.gpre + (size_t)w * d;
  const float *am = a.amat + (size_t)w * d;
  float ds = 0.f;
  for (int j = lane * 4; j < d; j += 128) ds += dot4(ld4(gA + j), ld4(am + j));
  ds = warp_sum(ds);
  const float sc = a.scale[w], rho = a.rho[w], R = a.Rsrc[w];
  const float rhoc = fmaxf(rho, 1e-6f);
  const float drho = rho > 1e-6f ? -ds * sc / rhoc : 0.f;
  const float ca = drho / ((float)d * rho);
  for (int j = lane * 4; j < d; j += 128)
    st4(a.da + (size_t)w * d + j, sc * ld4(gA + j) + ca * ld4(am + j));
  if (lane == 0) {
    const float dR = R > 1e-3f ? ds / rhoc : 0.f;
    a.dRc[w] = dR / ((float)d * R);
  }
}

cudaError_t launch_attn_bwd_scale(const AttnBwdArgs &a, int rows, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  attn_bwd_scale_kernel<<<(rows + 7) / 8, 256, 0, st>>>(a, rows);
  return cudaGetLastError();
}

// One block per token, warp per slot.  From dn (grad of the normalised mix)
// to dQ, dK, dV of the 32-wide head.
__global__ void attn_bwd_softmax_kernel(AttnBwdArgs a) {
  __shared__ float Ks[16][33], Qs[16][33], Vs[16][33], dmix[16][33], al[16][17], dlg[16][17];
  const int n = blockIdx.x, s = threadIdx.x >> 5, c = threadIdx.x & 31;
  const int h = a.h, d = a.d;
  const size_t row = ((size_t)n * h + s) * kHeadDim + c;
  const size_t qrow = ((size_t)n * h + s) * a.qkv_ld + c;
  Ks[s][c] = a.Kh[qrow] + a.W[a.off_kb + (size_t)s * d + c];
  Qs[s][c] = a.Qh[qrow] + a.W[a.off_qb + (size_t)s * d + c];
  Vs[s][c] = a.Vh[qrow];
  if (c < h) al[s][c] = a.alpha[((size_t)n * h + s) * h + c];
  const float nn = a.nmix[row], dnn = a.dn[row], r = a.rmix[(size_t)n * h + s];
  const float ndn = warp_sum(nn * dnn);
  dmix[s][c] = (dnn - nn * ndn / (float)kHeadDim) / r;
  __syncthreads();
  // query slot s: dalpha, softmax backward, dQ
  float dal[16];
  float adot = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < h) {
      dal[k] = warp_sum(dmix[s][c] * Vs[k][c]);
      adot += al[s][k] * dal[k];
    }
  const float gain = 2.0f * rsqrtf((float)kHeadDim);
  float dq = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (k < h) {
      const float dl = al[s][k] * (dal[k] - adot);
      dq += dl * Ks[k][c];
      if (c == 0) dlg[s][k] = dl;
    }
  a.dQ[qrow] = gain * dq;
  __syncthreads();
  // key/value slot s
  float dk = 0.f, dv = 0.f;
  const float ih = 1.f / (float)h;
  for (int q = 0; q < h; ++q) {
    dk += dlg[q][s] * Qs[q][c];
    dv += (al[q][s] - ih) * dmix[q][c];
  }
  a.dK[qrow] = gain * dk;
  a.dV[qrow] = dv;
}

cudaError_t launch_attn_bwd_softmax(const AttnBwdArgs &a, int N, cudaStream_t st) {
  if (N <= 0) return cudaSuccess;
  attn_bwd_softmax_kernel<<<N, 32 * a.h, 0, st>>>(a);
  return cudaGetLastError();
}

__global__ void dsig_init_kernel(AttnBwdArgs a, float *__restrict__ dsig, int rows, int slot_coord) {
  const size_t total4 = (size_t)rows * a.d / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t idx = i * 4;
    const size_t w = idx / a.d;
    const int j = (int)(idx % a.d);
    float4 g = ld4(a.gpre + idx);
    if (slot_coord) {
      const int s = (int)(w % a.h);
      const float4 src = ld4(a.signal + idx) + ld4(a.W + a.off_anchor + (size_t)s * a.d + j);
      g = g + a.dRc[w] * src;
    }
    st4(dsig + idx, g);
  }
}

static int grid_for(size_t n4) {
  size_t blocks = (n4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return blocks < 1 ? 1 : (int)blocks;
}

cudaError_t launch_dsig_init(const AttnBwdArgs &a, float *dsig, int rows, int slot_coord,
                             cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  dsig_init_kernel<<<grid_for((size_t)rows * a.d / 4), 256, 0, st>>>(a, dsig, rows, slot_coord);
  return cudaGetLastError();
}

__global__ void sub_upper_slots_kernel(float *__restrict__ dsig, const float *__restrict__ gpre, int N, int h,
                                       int d) {
  const int hu = h - h / 2;             // upper slots h/2 .. h-1
  const size_t row4 = (size_t)hu * d / 4;  // float4 per token over the upper slots
  const size_t total4 = (size_t)N * row4;
  const size_t off = (size_t)(h / 2) * d;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total4;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t n = i / row4, k = (i % row4) * 4;
    const size_t idx = n * (size_t)h * d + off + k;
    st4(dsig + idx, ld4(dsig + idx) - ld4(gpre + idx));
  }
}

cudaError_t launch_sub_upper_slots(float *dsig, const float *gpre, int N, int h, int d, cudaStream_t st) {
  if (N <= 0 || h < 2) return cudaSuccess;
  sub_upper_slots_kernel<<<grid_for((size_t)N * (h - h / 2) * d / 4), 256, 0, st>>>(dsig, gpre, N, h, d);
  return cudaGetLastError();
}

// One CTA per upper slot; a warp per token row, fixed striding and a fixed
// block reduction order (deterministic).
__global__ void __launch_bounds__(256) assoc_alpha_grad_kernel(const float *__restrict__ v,
                                                               const float *__restrict__ vread,
                                                               const float *__restrict__ alpha_raw, int N, int h,
                                                               int d, float *__restrict__ g_alpha) {
  __shared__ float red[8];
  const int s = h / 2 + blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc = 0.f;
  for (int n = warp; n < N; n += 8) {
    const float *vr = v + ((size_t)s * N + n) * d;
    const float *br = vread + ((size_t)n * h + s) * d;
    float dot = 0.f, vv = 0.f;
    for (int j = lane * 4; j < d; j += 128) {
      float4 g = ld4(vr + j);
      const float4 q = ld4(br + j);
      if (!finite4(g)) g = make_float4(isfinite(g.x) ? g.x : 0.f, isfinite(g.y) ? g.y : 0.f,
                                       isfinite(g.z) ? g.z : 0.f, isfinite(g.w) ? g.w : 0.f);
      dot += dot4(g, q);
      vv += dot4(q, q);
    }
    dot = warp_sum(dot);
    vv = warp_sum(vv);
    acc += dot / fmaxf(sqrtf(vv / (float)d), 0.1f);
  }
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += red[w];
    const float a = 1.f / (1.f + expf(-alpha_raw[s]));
    g_alpha[s] = a * (1.f - a) * t;
  }
}

cudaError_t launch_assoc_alpha_grad(const float *v, const float *vread, const float *alpha_raw, int N, int h, int d,
                                    float *g_alpha, cudaStream_t st) {
  if (N <= 0 || h < 2) return cudaSuccess;
  assoc_alpha_grad_kernel<<<h - h / 2, 256, 0, st>>>(v, vread, alpha_raw, N, h, d, g_alpha);
  return cudaGetLastError();
}

__global__ void add_kernel(float *__restrict__ dst, const float *__restrict__ x,
                           const float *__restrict__ y, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x)
    st4(dst + 4 * i, ld4(x + 4 * i) + ld4(y + 4 * i));
}

cudaError_t launch_add(float *dst, const float *a, const float *b, size_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  add_kernel<<<grid_for(n / 4), 256, 0, st>>>(dst, a, b, n / 4);
  return cudaGetLastError();
}

__global__ void permute_rows_kernel(const uint32_t *__restrict__ src, uint32_t *__restrict__ dst, int B, int T,
                                    size_t len, int to_internal) {
  const size_t N = (size_t)B * T;
  const size_t r = blockIdx.x % N, blk = blockIdx.x / N;  // destination row
  // destination row r in the target order -> source row in the other order
  size_t sr;
  if (to_internal) { const size_t t = r / B, b = r % B; sr = b * T + t; }
  else { const size_t b = r / T, t = r % T; sr = t * B + b; }
  const uint32_t *s = src + (blk * N + sr) * len;
  uint32_t *dd = dst + (blk * N + r) * len;
  if ((len & 3) == 0 && ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(dd)) & 15) == 0) {
    for (size_t i = threadIdx.x; i < len / 4; i += blockDim.x)
      reinterpret_cast<uint4 *>(dd)[i] = reinterpret_cast<const uint4 *>(s)[i];
  } else {
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) dd[i] = s[i];
  }
}

cudaError_t launch_permute_rows(const void *src, void *dst, int B, int T, int blocks, size_t len,
                                bool to_internal, cudaStream_t st) {
  const size_t rows = (size_t)B * T * blocks;
  if (rows == 0 || len == 0) return cudaSuccess;
  const int threads = len >= 512 ? 128 : 32;
  permute_rows_kernel<<<(unsigned)rows, threads, 0, st>>>(reinterpret_cast<const uint32_t *>(src),
                                                         reinterpret_cast<uint32_t *>(dst), B, T, len,
                                                         to_internal ? 1 : 0);
  return cudaGetLastError();
}

// dst[r][c] = x[r][c] + bias[c] over rows of `len` floats (len % 4 == 0).
__global__ void add_rowbias_kernel(float *__restrict__ dst, const float *__restrict__ x,
                                   const float *__restrict__ bias, size_t n4, size_t len4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x)
    st4(dst + 4 * i, ld4(x + 4 * i) + ld4(bias + 4 * (i % len4)));
}

cudaError_t launch_add_rowbias(float *dst, const float *x, const float *bias, size_t rows, size_t len,
                               cudaStream_t st) {
  const size_t n4 = rows * len / 4;
  if (n4 == 0) return cudaSuccess;
  add_rowbias_kernel<<<grid_for(n4), 256, 0, st>>>(dst, x, bias, n4, len / 4);
  return cudaGetLastError();
}

__global__ void colsum_kernel(const float *__restrict__ X, int rows, int ncols, long ld,
                              float *__restrict__ out, int seg, long ostride, int accumulate, long istride) {
  __shared__ float red[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  const long ic = (long)(c / seg) * istride + c % seg;
  // eight independent partial sums per thread: the row loads of a thread are in
  // flight together instead of one after another
  float acc = 0.f;
  if (c < ncols) {
    float p[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int r = ty;
    for (; r + 7 * 32 < rows; r += 8 * 32) {
#pragma unroll
      for (int q = 0; q < 8; ++q) p[q] += X[(size_t)(r + q * 32) * ld + ic];
    }
    for (; r < rows; r += 32) p[0] += X[(size_t)r * ld + ic];
    acc = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  }
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < ncols) {
    float t = 0.f;
    for (int q = 0; q < 32; ++q) t += red[q][tx];
    const long o = (long)(c / seg) * ostride + (c % seg);
    out[o] = accumulate ? out[o] + t : t;
  }
}

cudaError_t launch_colsum(const float *X, int rows, int ncols, long ld, float *out, int seg,
                          long ostride, bool accumulate, cudaStream_t st, long istride) {
  if (ncols <= 0) return cudaSuccess;
  colsum_kernel<<<(ncols + 31) / 32, 1024, 0, st>>>(X, rows, ncols, ld, out, seg, ostride,
                                                     accumulate ? 1 : 0, istride > 0 ? istride : seg);
  return cudaGetLastError();
}

}  // namespace aideen
