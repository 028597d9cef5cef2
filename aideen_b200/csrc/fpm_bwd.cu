// FPM memory backward: the reverse-time pass through the post-solve memory
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
//     batched tensor-core GEMMs over all tokens and `fpm_coef_kernel` turns
//     them into per-element coefficients, fully parallel over (token, slot);
//   * in those formulas dL/dM[t-1] is an elementwise-linear function of
//     dL/dM[t]:  g[t-1] = alpha[t] * g[t] + 0.5 * v[t]  (the reference's
//     retain, decay and per-dimension novelty terms all act elementwise), so
//     the serial part is a diagonal linear reverse scan, one thread per
//     (sequence, slot, dimension): `fpm_scan_kernel`;
//   * every parameter gradient is linear in g, so after the scan they are
//     column sums and outer-product GEMMs over all tokens.
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

// One warp per (token, slot) row; lane owns float4 columns lane + 32*i.
template <int NV>
__global__ void __launch_bounds__(256) fpm_coef_kernel(FpmBwdArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int rows = a.B * a.T * a.h;
  if (warp >= rows) return;
  const int d = a.d, h = a.h;
  const int n = warp / h, s = warp - n * h;
  const int t = n % a.T;
  const size_t row = (size_t)warp * d;
  const float *W = a.W;
  float4 hv[NV], cv[NV], mp[NV], pr[NV], rt[NV];
  float hsq = 0.f, gdot = 0.f, psq = 0.f, dsq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (lane + 32 * i);
    hv[i] = ld4(a.hstar + row + k);
    cv[i] = ld4(a.c + row + k);
    mp[i] = t > 0 ? ld4(a.hist + row - (size_t)h * d + k) : f4(0.f);
    const float4 dl = ld4(a.dpre + row + k) + ld4(W + a.off_bdelta + (size_t)s * d + k);
    pr[i] = tanh4(dl);
    const float4 rp = ld4(a.rpre + row + k) + ld4(W + a.off_bret + (size_t)s * d + k);
    rt[i] = make_float4(sigm(rp.x), sigm(rp.y), sigm(rp.z), sigm(rp.w));
    hsq += dot4(hv[i], hv[i]);
    gdot += dot4(ld4(W + a.off_wgate + (size_t)s * d + k), cv[i]);
    psq += dot4(mp[i], mp[i]);
    const float4 df = pr[i] - mp[i];
    dsq += dot4(df, df);
  }
  hsq = warp_sum(hsq);
  gdot = warp_sum(gdot);
  psq = warp_sum(psq);
  dsq = warp_sum(dsq);
  const float raw_z = sigm(gdot * rsqrtf((float)d) + W[a.off_bwrite + s] + kGateBias);
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
  if (lane == 0) a.rz[warp] = raw_z * (1.f - raw_z);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (lane + 32 * i);
    const float4 alog = ld4(W + a.off_alog + (size_t)s * d + k);
    float o_alpha[4], o_pre[4], o_bd[4], o_alog[4], o_gz[4], o_wx[4], o_min[4];
    const float hvv[4] = {hv[i].x, hv[i].y, hv[i].z, hv[i].w};
    const float mpv[4] = {mp[i].x, mp[i].y, mp[i].z, mp[i].w};
    const float prv[4] = {pr[i].x, pr[i].y, pr[i].z, pr[i].w};
    const float rtv[4] = {rt[i].x, rt[i].y, rt[i].z, rt[i].w};
    const float alv[4] = {alog.x, alog.y, alog.z, alog.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int kk = k + e;
      const float wx = 0.5f * tanhf(W[a.off_wx + (size_t)kk * d + kk]);
      const float am = 1.f / (1.f + expf(alv[e]));
      const float hu = hvv[e] * inv_hrms;
      const float r = rtv[e], p = prv[e], m = mpv[e];
      const float ret = 1.f - nov * (1.f - r);
      const float xp = hu + wx * hu + z * kResidualScale * p;
      const float base = am * m + (1.f - am) * xp;
      const float q = nov * r * (1.f - r);
      const float cpre = (m - base) * q;                    // g_pre / g
      const float cnov = -(cpre / fmaxf(q, 1e-6f)) * (1.f - r);   // g_nov / g
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
    st4(a.alpha + row + k, make_float4(o_alpha[0], o_alpha[1], o_alpha[2], o_alpha[3]));
    st4(a.cpre + row + k, make_float4(o_pre[0], o_pre[1], o_pre[2], o_pre[3]));
    st4(a.cbd + row + k, make_float4(o_bd[0], o_bd[1], o_bd[2], o_bd[3]));
    st4(a.calog + row + k, make_float4(o_alog[0], o_alog[1], o_alog[2], o_alog[3]));
    st4(a.cgz + row + k, make_float4(o_gz[0], o_gz[1], o_gz[2], o_gz[3]));
    st4(a.cwx + row + k, make_float4(o_wx[0], o_wx[1], o_wx[2], o_wx[3]));
    st4(a.minner + row + k, make_float4(o_min[0], o_min[1], o_min[2], o_min[3]));
  }
}

// Reverse scan, one thread per (sequence b, slot s, dimension k):
//   dm[t] = g;  g_pre[t] = cpre[t] * g;  g <- alpha[t] * g + 0.5 * v[t]
// with per-thread sums of the elementwise gradient terms over the chunk.
__global__ void __launch_bounds__(128) fpm_scan_kernel(FpmBwdArgs a) {
  const int d = a.d, h = a.h, T = a.T;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.B * h * d) return;
  const int k = i % d;
  const int s = (i / d) % h;
  const int b = i / (d * h);
  const size_t N = (size_t)a.B * T;
  float g = a.carry[i];
  float s_pre = 0.f, s_bd = 0.f, s_alog = 0.f, s_wx = 0.f;
#pragma unroll 4
  for (int t = T - 1; t >= 0; --t) {
    const size_t n = (size_t)b * T + t;
    const size_t idx = (n * h + s) * d + k;
    const float al = a.alpha[idx];
    const float cp = a.cpre[idx];
    float vv = a.v[((size_t)s * N + n) * d + k];
    vv = isfinite(vv) ? vv : 0.f;
    a.dm[idx] = g;
    const float gp = cp * g;
    a.gpre[idx] = gp;
    s_pre += gp;
    s_bd += a.cbd[idx] * g;
    s_alog += a.calog[idx] * g;
    s_wx += a.cwx[idx] * g;
    g = al * g + kReadGradScale * vv;
  }
  a.carry[i] = g;
  const size_t P = (size_t)a.B * h * d;
  a.part[i] = s_pre;
  a.part[P + i] = s_bd;
  a.part[2 * P + i] = s_alog;
  a.part[3 * P + i] = s_wx;
}

// Per (token, slot): dL/d(raw gate) = raw_z (1 - raw_z) * sum_k cgz * dm.
template <int NV>
__global__ void __launch_bounds__(256) fpm_gate_kernel(FpmBwdArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.B * a.T * a.h) return;
  const size_t row = (size_t)warp * a.d;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (lane + 32 * i);
    acc += dot4(ld4(a.cgz + row + k), ld4(a.dm + row + k));
  }
  acc = warp_sum(acc);
  if (lane == 0) a.graw[warp] = acc * a.rz[warp];
}

// Sum the per-sequence partials and scatter into the gradient vector:
// b_retain, b_delta, a_log per (slot, k) and the diagonal of W_x per k.
__global__ void fpm_finalize_kernel(FpmBwdArgs a, float *G) {
  const int d = a.d, h = a.h, B = a.B;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const size_t P = (size_t)B * h * d;
  if (i < h * d) {
    float sp = 0.f, sb = 0.f, sa = 0.f;
    for (int b = 0; b < B; ++b) {
      const size_t j = (size_t)b * h * d + i;
      sp += a.part[j];
      sb += a.part[P + j];
      sa += a.part[2 * P + j];
    }
    G[a.off_bret + i] = sp;
    G[a.off_bdelta + i] = sb;
    G[a.off_alog + i] = sa;
  }
  if (i < d) {
    float sw = 0.f;
    for (int b = 0; b < B; ++b)
      for (int s = 0; s < h; ++s) sw += a.part[3 * P + ((size_t)b * h + s) * d + i];
    const float th = tanhf(a.W[a.off_wx + (size_t)i * d + i]);
    G[a.off_wx + (size_t)i * d + i] = sw * 0.5f * (1.f - th * th);
  }
}

}  // namespace

cudaError_t launch_fpm_c(const float *hstar, const float *signal, float *c, size_t n, cudaStream_t st) {
  const size_t n4 = n / 4;
  const int blocks = (int)((n4 + 255) / 256 < 148 * 16 ? (n4 + 255) / 256 : 148 * 16);
  fpm_c_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(hstar),
                                       reinterpret_cast<const float4 *>(signal),
                                       reinterpret_cast<float4 *>(c), n4);
  return cudaGetLastError();
}

cudaError_t launch_fpm_coef(const FpmBwdArgs &a, cudaStream_t st) {
  const int rows = a.B * a.T * a.h;
  const int blocks = (rows * 32 + 255) / 256;
  switch (a.d / 128) {
    case 1: fpm_coef_kernel<1><<<blocks, 256, 0, st>>>(a); break;
    case 2: fpm_coef_kernel<2><<<blocks, 256, 0, st>>>(a); break;
    case 4: fpm_coef_kernel<4><<<blocks, 256, 0, st>>>(a); break;
    case 8: fpm_coef_kernel<8><<<blocks, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_fpm_scan(const FpmBwdArgs &a, cudaStream_t st) {
  const int n = a.B * a.h * a.d;
  fpm_scan_kernel<<<(n + 127) / 128, 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_fpm_gate(const FpmBwdArgs &a, cudaStream_t st) {
  const int rows = a.B * a.T * a.h;
  const int blocks = (rows * 32 + 255) / 256;
  switch (a.d / 128) {
    case 1: fpm_gate_kernel<1><<<blocks, 256, 0, st>>>(a); break;
    case 2: fpm_gate_kernel<2><<<blocks, 256, 0, st>>>(a); break;
    case 4: fpm_gate_kernel<4><<<blocks, 256, 0, st>>>(a); break;
    case 8: fpm_gate_kernel<8><<<blocks, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_fpm_finalize(const FpmBwdArgs &a, float *G, cudaStream_t st) {
  const int n = a.h * a.d;
  fpm_finalize_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, G);
  return cudaGetLastError();
}

}  // namespace aideen
