// Allocation-free variant of the fused clean adjoint.
//
// Some callers cannot allocate device memory: allocators that forbid
// cudaMalloc once start-up is over, embedders that hand over pre-sized
// buffers and own every other byte of the device, or host code that must not
// take the allocator's lock on its latency path.  aideen_adjoint_noalloc
// serves them: the caller passes every input and output as a device pointer,
// no context is created, and the only extra memory the computation needs
// (per-token partial sums of the NormScale gradient) lives in the fixed array
// below.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/aideen_b200.h"
#include "kernels.cuh"

namespace aideen {
namespace {

// At most this many floats of per-token partials (tokens * d_model): 4 Mi
// floats = 16 MiB, e.g. 8192 tokens at d_model = 512.  Every GPU that loads the
// library holds this array until the process exits.
constexpr size_t kNoAllocScratchFloats = size_t(1) << 22;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float *g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  In host code
// `g_noalloc_scratch` names a host-side stand-in, not device memory, so the
// address is looked up once per device with that device current.
int scratch_for_current_device(float **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AIDEEN_E_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return AIDEEN_E_CUDA;
    g_scratch_ptr[dev] = static_cast<float *>(p);
  }
  *out = g_scratch_ptr[dev];
  return AIDEEN_OK;
}

}  // namespace
}  // namespace aideen

extern "C" int aideen_adjoint_noalloc(const float *hstar, const float *branch, const float *dl_dh,
                                      const float *rhs_slot, const float *norm_scale,
                                      uint32_t n_tokens, uint32_t h_slots, uint32_t d_model,
                                      uint32_t iters, float damping, uint32_t anderson_m,
                                      float *v_out, float *gpre_out, float *ns_grad_out,
                                      void *stream) {
  using namespace aideen;
  if (!hstar || !branch || !norm_scale || !v_out || !gpre_out) return AIDEEN_E_INVALID;
  if (!(d_model == 128 || d_model == 256 || d_model == 512 || d_model == 1024)) return AIDEEN_E_INVALID;
  if (h_slots < 1 || h_slots > 16 || n_tokens == 0 || anderson_m > 4) return AIDEEN_E_INVALID;
  if (ns_grad_out && (size_t)n_tokens * d_model > kNoAllocScratchFloats)
    return AIDEEN_E_INVALID;  // beyond the fixed scratch: split the tokens over several calls
  // The kernel stages its inputs with 16-byte bulk copies and float4 accesses:
  // a misaligned pointer (e.g. a view at an odd element offset) is refused
  // here instead of faulting on the device.
  const void *ptrs[] = {hstar, branch, dl_dh, rhs_slot, norm_scale, v_out, gpre_out, ns_grad_out};
  for (const void *p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return AIDEEN_E_INVALID;
  // One CTA double-buffers every staged input of a token (h_slots * d_model
  // floats each for hstar, branch and rhs_slot): shapes whose two stages exceed
  // the device's shared memory per block are refused.
  {
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      return AIDEEN_E_CUDA;
    if (adjoint_smem_bytes((int)h_slots, (int)d_model, true, rhs_slot != nullptr, dl_dh != nullptr,
                           (int)anderson_m) > (size_t)optin)
      return AIDEEN_E_INVALID;
  }
  float *scratch = nullptr;
  if (ns_grad_out) {
    const int rc = scratch_for_current_device(&scratch);
    if (rc != AIDEEN_OK) return rc;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AdjointArgs a{};
  a.N = (int)n_tokens; a.h = (int)h_slots; a.d = (int)d_model; a.iters = (int)iters;
  a.anderson_m = (int)anderson_m; a.beta = damping;
  a.pre_a = hstar; a.pre_b = branch; a.rhs_tok = dl_dh; a.rhs_slot = rhs_slot; a.NS = norm_scale;
  a.v = v_out; a.gpre = gpre_out;
  // The adjoint writes every partial row it covers before colsum reads it, so
  // the scratch needs no clearing between calls.
  a.nsg = scratch;
  if (launch_adjoint(a, st) != cudaSuccess) return AIDEEN_E_CUDA;
  if (ns_grad_out &&
      launch_colsum(scratch, (int)n_tokens, (int)d_model, d_model, ns_grad_out, (int)d_model, 0,
                    false, st) != cudaSuccess)
    return AIDEEN_E_CUDA;
  // Wait for the work and report a bounded stage wait of the kernel that ran
  // out.  A stream that is being captured cannot be waited on; its check is
  // left to the first later call that can wait.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return AIDEEN_E_CUDA;
  if (cap != cudaStreamCaptureStatusNone) return AIDEEN_OK;
  unsigned int timed_out = 0;
  if (adjoint_error_async(&timed_out, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
    return AIDEEN_E_CUDA;
  return timed_out ? AIDEEN_E_TIMEOUT : AIDEEN_OK;
}
