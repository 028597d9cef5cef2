// The simple temporal carrier: the memory scan of the reference's CPU DEQ
// (fixed_point_memory_reasoning.rs:1455-1486) and of its hist_v2 GPU mode
// (hist_v2_temporal.wgsl:60-108), run token by token over a chunk of fixed
// points:
//   M_t = (I + W_out^T)(a * M_{t-1} + (1 - a) * (1 + 0.5 tanh(diag W_x)) * h_t / rms(h_t)),
//   a = sigmoid(-a_log[slot]).
// One CTA per (sequence, slot) walks the tokens; each thread owns two
// elements.  W_out (d x d, shared by every slot) is read from L2 every token:
// the scan is a chain of d x d matrix-vector products, bound by that read and
// by the per-token reduction, not by HBM.
#include "common.cuh"
#include "kernels.cuh"

namespace aideen {
namespace {

__global__ void __launch_bounds__(512) temporal_scan_kernel(TemporalArgs a) {
  extern __shared__ __align__(16) float xs[];  // [d] this token's pre-projection memory
  __shared__ __align__(16) float red[2 * 8 * 32];
  const int d = a.d, h = a.h;
  const int b = blockIdx.x / h, s = blockIdx.x % h;
  const int j0 = 2 * threadIdx.x;
  BlockReducer R(red);
  const float *W = a.W;
  const float2 al = ld2(W + a.off_alog + (size_t)s * d + j0);
  const float2 av = make_float2(1.f / (1.f + expf(al.x)), 1.f / (1.f + expf(al.y)));
  const float2 wx = make_float2(0.5f * tanhf(W[a.off_wx + (size_t)j0 * d + j0]),
                                0.5f * tanhf(W[a.off_wx + (size_t)(j0 + 1) * d + j0 + 1]));
  const float *Wo = W + a.off_wout;
  float2 m = ld2(a.mstate + ((size_t)b * h + s) * d + j0);
  for (int t = 0; t < a.T; ++t) {
    const size_t e = (((size_t)t * a.B + b) * h + s) * d + j0;  // token-major rows
    const float2 hv = ld2(a.hstar + e);
    float v[1] = {dot2(hv, hv)};
    R.sum(v);
    const float hr = sqrtf(v[0] / (float)d + 1e-6f);
    const float ih = 1.f / fmaxf(hr, 1e-6f);
    const float2 hu = ih * hv;
    const float2 x = hu + wx * hu;
    const float2 mn = av * m + (f2(1.f) - av) * x;
    st2(xs + j0, mn);
    __syncthreads();
    // out[i] = mn[i] + sum_j W_out[j][i] mn[j]
    float2 acc0 = mn, acc1 = f2(0.f);
#pragma unroll 4
    for (int j = 0; j < d; j += 2) {
      const float2 w0 = __ldg(reinterpret_cast<const float2 *>(Wo + (size_t)j * d + j0));
      const float2 w1 = __ldg(reinterpret_cast<const float2 *>(Wo + (size_t)(j + 1) * d + j0));
      acc0 = fma2(f2(xs[j]), w0, acc0);
      acc1 = fma2(f2(xs[j + 1]), w1, acc1);
    }
    m = acc0 + acc1;
    st2(a.hist + e, m);
    __syncthreads();  // xs is rewritten by the next token
  }
  st2(a.mstate + ((size_t)b * h + s) * d + j0, m);
}

}  // namespace

cudaError_t launch_temporal_scan(const TemporalArgs &a, cudaStream_t st) {
  if (a.B <= 0 || a.T <= 0) return cudaSuccess;
  temporal_scan_kernel<<<a.B * a.h, a.d / 2, (size_t)a.d * sizeof(float), st>>>(a);
  return cudaGetLastError();
}

}  // namespace aideen
