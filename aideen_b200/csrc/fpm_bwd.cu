// FPM memory backward (token-major rows: row (t, b) = t * B + b): the reverse-time pass through the post-solve memory
// write, with the reference's gradient formulas
// (aideen-backbone/src/shaders/fused_fpm_retain_bwd.wgsl:364-2095) and its
// shared W_out / diag W_x gradients (fused_fpm_shared_update.wgsl:129-256).
//
// The reference runs one 64-lane workgroup per slot, serial over every
// sequence and token, recomputing four d x 32 matvecs per token.  Here the
// pass is split by what actually depends on what:
//
//   * every forward-side quantity of token t (the retain / write-gate
//     pre-activations, the proposal, novelty and norms) depends only on the
//     stored h*, signal and memory history, so the low-rank projections are
//     batched tensor-core GEMMs over all tokens and `row_coefs` turns them
//     into per-element coefficients, one warp per (token, slot);
//   * in those formulas dL/dM[t-1] is an elementwise-linear function of
//     dL/dM[t]:  g[t-1] = alpha[t] * g[t] + 0.5 * v[t]  (the reference's
//     retain, decay and per-dimension novelty terms all act elementwise), so
//     the serial part is a diagonal linear reverse scan.  It runs chunked:
//     every chunk of CH tokens composes its steps into g -> A g + U
//     (parallel over chunks), a short pass carries g across the chunks, and
//     every chunk then replays its steps from its entry value;
//   * every parameter gradient is linear in g, so the elementwise ones are
//     summed per chunk and reduced deterministically, and the matrix ones are
//     outer-product GEMMs over all tokens.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.cuh"

namespace aideen {
namespace {

constexpr float kResidualScale = 0.1f;   // FPM_RESIDUAL_SCALE
constexpr float kGateBias = -1.5f;       // FPM_GATE_BIAS
constexpr float kReadGradScale = 0.5f;   // FPM_READ_GRAD_SCALE

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

// c = 0.5 * (h* + signal), [rows][d] with rows = N*h.
__global__ void fpm_c_kernel(const float4 *__restrict__ hs, const float4 *__restrict__ sig,
                             float4 *__restrict__ c, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    c[i] = 0.5f * (hs[i] + sig[i]);
}

// Coefficients of one (token, slot) row, computed by WPR warps; row thread
// rl = 32 * (warp % WPR) + lane owns the float4 columns rl + 32 * WPR * i, and
// the row's four sums are combined in `red` ([WPR][4], in warp order) behind
// the pair's named barrier `bar` (WPR > 1).  Every gradient term of the reference's token
// step is linear in g = dL/dM[t]:
//   alpha: g[t-1] = alpha * g + 0.5 v[t]      cpre:  g_pre (b_retain, W_retain_*)
//   cbd:   b_delta term                       calog: a_log term
//   cwx:   diag-W_x carrier term (before the tanh chain)
//   cgz:   per-element weight of the write-gate sum, rz = raw_z (1 - raw_z)
// and m_inner (the W_out operand) does not depend on g.  FULL = false stores
// alpha only.
// prm: the slot's parameters staged in shared memory,
//   [0,d) b_retain  [d,2d) b_delta  [2d,3d) W_write_gate  [3d,4d) a = sigmoid(-a_log)
//   [4d,5d) 0.5 tanh(diag W_x)
__device__ __forceinline__ void pair_sync(int bar, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
}

template <int NV, int WPR, bool FULL>
__device__ __forceinline__ void row_coefs(const FpmBwdArgs &a, const float *prm, int n, int s, int t,
                                          float *sm_row, size_t plane, float *rz_out, float *red, int bar) {
  const int lane = threadIdx.x & 31;
  const int wp = (threadIdx.x >> 5) % WPR;
  const int rl = 32 * wp + lane;
  const int d = a.d, h = a.h;
  const size_t row = ((size_t)n * h + s) * d;
  float4 hv[NV], mp[NV], pr[NV], rt[NV];
  float hsq = 0.f, gdot = 0.f, psq = 0.f, dsq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (rl + 32 * WPR * i);
    hv[i] = ld4(a.hstar + row + k);
    mp[i] = t > 0 ? ld4(a.hist + row - (size_t)a.B * h * d + k) : f4(0.f);  // token t-1, token-major rows
    const float4 dl = ld4(a.dpre + row + k) + ld4(prm + d + k);
    pr[i] = tanh4(dl);
    const float4 rp = ld4(a.rpre + row + k) + ld4(prm + k);
    rt[i] = make_float4(sigm(rp.x), sigm(rp.y), sigm(rp.z), sigm(rp.w));
    hsq += dot4(hv[i], hv[i]);
    gdot += dot4(ld4(prm + 2 * d + k), ld4(a.c + row + k));
    psq += dot4(mp[i], mp[i]);
    const float4 df = pr[i] - mp[i];
    dsq += dot4(df, df);
  }
  hsq = warp_sum(hsq);
  gdot = warp_sum(gdot);
  psq = warp_sum(psq);
  dsq = warp_sum(dsq);
  if (WPR > 1) {
    if (lane == 0) {
      red[4 * wp + 0] = hsq;
      red[4 * wp + 1] = gdot;
      red[4 * wp + 2] = psq;
      red[4 * wp + 3] = dsq;
    }
    pair_sync(bar, 32 * WPR);
    hsq = gdot = psq = dsq = 0.f;
#pragma unroll
    for (int q = 0; q < WPR; ++q) {
      hsq += red[4 * q + 0];
      gdot += red[4 * q + 1];
      psq += red[4 * q + 2];
      dsq += red[4 * q + 3];
    }
  }
  const float raw_z = sigm(gdot * rsqrtf((float)d) + a.W[a.off_bwrite + s] + kGateBias);
  const float z = fminf(fmaxf(raw_z, 0.f), 1.f);
  const float prev_norm = sqrtf(fmaxf(psq, 1e-6f));
  const float diff_norm = sqrtf(fmaxf(dsq, 1e-6f));
  const float denom = diff_norm + prev_norm + 1e-6f;
  const float nov = diff_norm / denom;
  const float dnov_ddiff = prev_norm / (denom * denom);
  const float dnov_dprev = -diff_norm / (denom * denom);
  const float inv_hrms = 1.f / sqrtf(fmaxf(hsq / (float)d, 1e-6f));
  const float inv_dn = 1.f / fmaxf(diff_norm, 1e-6f);
  const float inv_pn = 1.f / fmaxf(prev_norm, 1e-6f);
  const float zs = 0.5f / sqrtf(fmaxf(z, 1e-6f));
  if (FULL && rl == 0) *rz_out = raw_z * (1.f - raw_z);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (rl + 32 * WPR * i);
    const float4 am4 = ld4(prm + 3 * d + k), wx4 = ld4(prm + 4 * d + k);
    float o_alpha[4], o_pre[4], o_bd[4], o_alog[4], o_gz[4], o_wx[4], o_min[4];
    const float hvv[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
    const float mpv[4] = {mp[i].x, mp[i].y, mp[i].z, mp[i].w};
    const float prv[4] = {pr[i].x, pr[i].y, pr[i].z, pr[i].w};
    const float rtv[4] = {rt[i].x, rt[i].y, rt[i].z, rt[i].w};
    const float amv[4] = {am4.x, am4.y, am4.z, am4.w};
    const float wxv[4] = {wx4.x, wx4.y, wx4.z, wx4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float wx = wxv[e], am = amv[e];
      const float hu = hvv[e] * inv_hrms;
      const float r = rtv[e], p = prv[e], m = mpv[e];
      const float ret = 1.f - nov * (1.f - r);
      const float xp = hu + wx * hu + z * kResidualScale * p;
      const float base = am * m + (1.f - am) * xp;
      const float q = nov * r * (1.f - r);
      const float cpre = (m - base) * q;                          // g_pre / g
      const float cnov = -(cpre / fmaxf(q, 1e-6f)) * (1.f - r);   // g_novelty / g
      const float udiff = (p - m) * inv_dn;
      const float cdn = cnov * dnov_ddiff;
      const float gx = (1.f - am) * (1.f - ret);
      o_alpha[e] = ret + (1.f - ret) * am + cnov * dnov_dprev * m * inv_pn - cdn * udiff;
      o_pre[e] = cpre;
      o_bd[e] = (gx * z * kResidualScale + cdn * udiff) * (1.f - p * p);
      o_alog[e] = -am * (1.f - am) * (1.f - ret) * (m - xp);
      o_gz[e] = gx * (kResidualScale * p + hu * zs);
      o_wx[e] = (1.f - am) * hu;
      o_min[e] = ret * m + (1.f - ret) * base;
    }
    st4(sm_row + k, make_float4(o_alpha[0], o_alpha[1], o_alpha[2], o_alpha[3]));
    if (FULL) {
      st4(sm_row + plane + k, make_float4(o_pre[0], o_pre[1], o_pre[2], o_pre[3]));
      st4(sm_row + 2 * plane + k, make_float4(o_bd[0], o_bd[1], o_bd[2], o_bd[3]));
      st4(sm_row + 3 * plane + k, make_float4(o_alog[0], o_alog[1], o_alog[2], o_alog[3]));
      st4(sm_row + 4 * plane + k, make_float4(o_wx[0], o_wx[1], o_wx[2], o_wx[3]));
      st4(sm_row + 5 * plane + k, make_float4(o_gz[0], o_gz[1], o_gz[2], o_gz[3]));
      st4(a.minner + row + k, make_float4(o_min[0], o_min[1], o_min[2], o_min[3]));
    }
  }
}

// One CTA per (chunk of CH tokens, slot, sequence); warps WPR*w .. WPR*w+WPR-1
// compute token w's coefficients into shared memory, then one thread per
// dimension walks the chunk backwards.
//   FULL = false: chunk composite  g_in -> A * g_in + U  (alpha products and
//                 the accumulated read seeds), written to a.cA / a.cU.
//   FULL = true:  from the chunk's entry value a.gin, emit dm and g_pre, the
//                 per-chunk sums of every elementwise gradient term, and the
//                 write-gate terms (W_write_gate, b_write_mem).
template <int NV, int CH, int WPR, bool FULL>
__global__ void __launch_bounds__(32 * CH * WPR) fpm_chunk_kernel(FpmBwdArgs a) {
  extern __shared__ __align__(16) float sm[];
  const int ch = (FULL ? 0 : a.ch0) + blockIdx.x, s = blockIdx.y, b = blockIdx.z;
  const int d = a.d, h = a.h, T = a.T, nch = a.nch;
  const size_t plane = (size_t)CH * d;
  float *vs = sm + (FULL ? 6 : 1) * plane;   // 0.5 * v of the chunk's tokens
  float *rz = vs + plane;
  float *graw = rz + CH;
  float *prm = graw + CH;   // 5 * d staged slot parameters (CH is even)
  float *red = prm + 5 * d;  // [CH][WPR][4] row sums
  {
    const float4 *src = reinterpret_cast<const float4 *>(a.slot_prm + (size_t)s * 5 * d);
    for (int k = threadIdx.x; k < 5 * d / 4; k += blockDim.x) reinterpret_cast<float4 *>(prm)[k] = src[k];
  }
  __syncthreads();
  const int w = (threadIdx.x >> 5) / WPR;  // token of the chunk this warp works on
  const int rl = threadIdx.x % (32 * WPR);
  const int t0 = ch * CH;
  const int nt = min(CH, T - t0);
  const size_t N = (size_t)a.B * T;
  if (w < nt) {
    const size_t n = (size_t)(t0 + w) * a.B + b;
    const float *vrow = a.v + ((size_t)s * N + n) * d;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int k = 4 * (rl + 32 * WPR * i);
      const float4 x = ld4(vrow + k);
      st4(vs + (size_t)w * d + k, make_float4(isfinite(x.x) ? kReadGradScale * x.x : 0.f,
                                              isfinite(x.y) ? kReadGradScale * x.y : 0.f,
                                              isfinite(x.z) ? kReadGradScale * x.z : 0.f,
                                              isfinite(x.w) ? kReadGradScale * x.w : 0.f));
    }
    row_coefs<NV, WPR, FULL>(a, prm, (int)n, s, t0 + w, sm + (size_t)w * d, plane, rz + w, red + 4 * WPR * w,
                             1 + w);
  }
  __syncthreads();
  const size_t bc = ((size_t)b * nch + ch) * h + s;   // (sequence, chunk, slot) row of the partials
  const size_t P = (size_t)a.B * nch * h * d;
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    if (!FULL) {
      float A = 1.f, U = 0.f;
      for (int tl = nt - 1; tl >= 0; --tl) {
        const float al = sm[(size_t)tl * d + k];
        A = al * A;
        U = al * U + vs[(size_t)tl * d + k];
      }
      const size_t o = (((size_t)b * h + s) * nch + ch) * d + k;
      a.cA[o] = A;
      a.cU[o] = U;
    } else {
      float g = a.gin[(((size_t)b * h + s) * nch + ch) * d + k];
      float s_pre = 0.f, s_bd = 0.f, s_alog = 0.f, s_wx = 0.f;
      for (int tl = nt - 1; tl >= 0; --tl) {
        const size_t n = (size_t)(t0 + tl) * a.B + b;
        const size_t idx = (n * h + s) * d + k;
        float *c = sm + (size_t)tl * d + k;
        const float al = c[0];
        a.dm[idx] = g;
        c[0] = g;                               // dm, for the write-gate sum below
        const float gp = c[plane] * g;
        a.gpre[idx] = gp;
        s_pre += gp;
        s_bd += c[2 * plane] * g;
        s_alog += c[3 * plane] * g;
        s_wx += c[4 * plane] * g;
        g = al * g + vs[(size_t)tl * d + k];
      }
      const size_t o = bc * d + k;
      a.part[o] = s_pre;
      a.part[P + o] = s_bd;
      a.part[2 * P + o] = s_alog;
      a.part[3 * P + o] = s_wx;
    }
  }
  if (!FULL) return;
  __syncthreads();
  if (w < nt) {
    const int lane = threadIdx.x & 31;
    const float *dm = sm + (size_t)w * d, *cg = dm + 5 * plane;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int k = 4 * (rl + 32 * WPR * i);
      acc += dot4(ld4(cg + k), ld4(dm + k));
    }
    acc = warp_sum(acc);
    if (WPR > 1) {
      float *r2 = red + 4 * WPR * w;  // free again: the row sums were consumed before the scan
      if (lane == 0) r2[rl >> 5] = acc;
      pair_sync(1 + w, 32 * WPR);
      acc = 0.f;
#pragma unroll
      for (int q = 0; q < WPR; ++q) acc += r2[q];
    }
    if (rl == 0) graw[w] = acc * rz[w];
  }
  __syncthreads();
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int tl = 0; tl < CH; ++tl) {
      if (tl < nt) {
        const size_t n = (size_t)(t0 + tl) * a.B + b;
        acc += graw[tl] * a.c[(n * h + s) * d + k];
      }
    }
    a.part[4 * P + bc * d + k] = acc;
  }
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int tl = 0; tl < nt; ++tl) acc += graw[tl];
    a.part_bw[bc] = acc;
  }
}

// Carry across chunks, one thread per (sequence, slot, dimension):
// gin[ch] = g;  g <- A[ch] g + U[ch], from the last chunk to the first.
__global__ void fpm_carry_kernel(FpmBwdArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int d = a.d, nch = a.nch;
  if (i >= a.B * a.h * d) return;
  const int k = i % d;
  const size_t base = (size_t)(i / d) * nch * d + k;
  const float *__restrict__ cA = a.cA;
  const float *__restrict__ cU = a.cU;
  float *__restrict__ gin = a.gin;
  float g = a.carry[i];
#pragma unroll 8
  for (int ch = nch - 1; ch >= 0; --ch) {
    const size_t o = base + (size_t)ch * d;
    gin[o] = g;
    g = cA[o] * g + cU[o];
  }
  a.carry[i] = g;
}

// Deterministic sums of the per-(sequence, chunk) partials into the gradient
// vector.  blockIdx.y picks the quantity; each block reduces 32 columns with
// 32 row-strided threads per column:
//   0..3: b_retain, b_delta, a_log, W_write_gate over [B*nch] rows of [h*d]
//   4:    diag W_x over [B*nch*h] rows of [d]     5: b_write_mem over rows of [h]
__global__ void __launch_bounds__(1024) fpm_finalize_kernel(FpmBwdArgs a, float *G) {
  __shared__ float red[32][33];
  const int d = a.d, h = a.h, q = blockIdx.y;
  const int R = a.B * a.nch;
  const size_t P = (size_t)R * h * d;
  const float *X;
  int rows, ncols;
  if (q < 4) { X = a.part + (size_t)(q == 3 ? 4 : q) * P; rows = R; ncols = h * d; }
  else if (q == 4) { X = a.part + 3 * P; rows = R * h; ncols = d; }
  else { X = a.part_bw; rows = R; ncols = h; }
  const int c0 = blockIdx.x * 32;
  if (c0 >= ncols) return;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = c0 + tx;
  float acc = 0.f;
  if (c < ncols)
    for (int r = ty; r < rows; r += 32) acc += X[(size_t)r * ncols + c];
  red[ty][tx] = acc;
  __syncthreads();
  if (ty != 0 || c >= ncols) return;
  float t = 0.f;
  for (int i = 0; i < 32; ++i) t += red[i][tx];
  switch (q) {
    case 0: G[a.off_bret + c] = t; break;
    case 1: G[a.off_bdelta + c] = t; break;
    case 2: G[a.off_alog + c] = t; break;
    case 3: G[a.off_wgate + c] = t * rsqrtf((float)d); break;
    case 4: {
      const float th = tanhf(a.W[a.off_wx + (size_t)c * d + c]);
      G[a.off_wx + (size_t)c * d + c] = t * 0.5f * (1.f - th * th);
      break;
    }
    default: G[a.off_bwrite + c] = t;
  }
}

}  // namespace

// The slot parameters every chunk CTA stages, once per backward:
//   [0,d) b_retain  [d,2d) b_delta  [2d,3d) W_write_gate  [3d,4d) sigmoid(-a_log)
//   [4d,5d) 0.5 tanh(diag W_x)
__global__ void fpm_slot_params_kernel(FpmBwdArgs a) {
  const int s = blockIdx.x, d = a.d;
  const float *W = a.W;
  float *o = a.slot_prm + (size_t)s * 5 * d;
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    o[k] = W[a.off_bret + (size_t)s * d + k];
    o[d + k] = W[a.off_bdelta + (size_t)s * d + k];
    o[2 * d + k] = W[a.off_wgate + (size_t)s * d + k];
    o[3 * d + k] = 1.f / (1.f + expf(W[a.off_alog + (size_t)s * d + k]));
    o[4 * d + k] = 0.5f * tanhf(W[a.off_wx + (size_t)k * d + k]);
  }
}

cudaError_t launch_fpm_c(const float *hstar, const float *signal, float *c, size_t n, cudaStream_t st) {
  const size_t n4 = n / 4;
  const int blocks = (int)((n4 + 255) / 256 < 148 * 16 ? (n4 + 255) / 256 : 148 * 16);
  fpm_c_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(hstar),
                                       reinterpret_cast<const float4 *>(signal),
                                       reinterpret_cast<float4 *>(c), n4);
  return cudaGetLastError();
}

int fpm_chunk_len(int d) { return d > 512 ? 2 : 4; }

size_t fpm_chunk_smem(int d, bool full) {
  const int CH = fpm_chunk_len(d);
  return ((full ? 7 : 2) * (size_t)CH * d + 2 * CH + 5 * (size_t)d + 8 * (size_t)CH) * sizeof(float);
}

template <int NV, int CH, int WPR, bool FULL>
static cudaError_t chunk_launch(const FpmBwdArgs &a, cudaStream_t st) {
  static_assert(CH <= 15, "one named barrier per token row");
  const size_t smem = fpm_chunk_smem(a.d, FULL);
  auto k = fpm_chunk_kernel<NV, CH, WPR, FULL>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int nx = (!FULL && a.ch1 > 0) ? a.ch1 - a.ch0 : a.nch;
  if (nx <= 0) return cudaSuccess;
  FpmBwdArgs b = a;
  if (FULL || a.ch1 <= 0) b.ch0 = 0;
  k<<<dim3(nx, a.h, a.B), 32 * CH * WPR, smem, st>>>(b);
  return cudaGetLastError();
}

template <bool FULL>
static cudaError_t chunk_dispatch(const FpmBwdArgs &a, cudaStream_t st) {
  if (a.nch != (a.T + fpm_chunk_len(a.d) - 1) / fpm_chunk_len(a.d)) return cudaErrorInvalidValue;
  switch (a.d / 128) {
    case 1: return chunk_launch<1, 4, 1, FULL>(a, st);
    case 2: return chunk_launch<1, 4, 2, FULL>(a, st);
    case 4: return chunk_launch<2, 4, 2, FULL>(a, st);
    case 8: return chunk_launch<4, 2, 2, FULL>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_fpm_slot_params(const FpmBwdArgs &a, cudaStream_t st) {
  fpm_slot_params_kernel<<<a.h, 256, 0, st>>>(a);
  return cudaGetLastError();
}
cudaError_t launch_fpm_composite(const FpmBwdArgs &a, cudaStream_t st) { return chunk_dispatch<false>(a, st); }
cudaError_t launch_fpm_chunks(const FpmBwdArgs &a, cudaStream_t st) { return chunk_dispatch<true>(a, st); }

cudaError_t launch_fpm_carry(const FpmBwdArgs &a, cudaStream_t st) {
  const int n = a.B * a.h * a.d;
  fpm_carry_kernel<<<(n + 127) / 128, 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_fpm_finalize(const FpmBwdArgs &a, float *G, cudaStream_t st) {
  fpm_finalize_kernel<<<dim3((a.h * a.d + 31) / 32, 6), 1024, 0, st>>>(a, G);
  return cudaGetLastError();
}

}  // namespace aideen
