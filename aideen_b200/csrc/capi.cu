// C ABI of libaideen_b200: context lifetime, buffer ownership and the
// orchestration of one training step.  Mirrors the reference's
// GpuDeqBackend (aideen-backbone/src/gpu_deq.rs:80-218) call sequence:
// forward (:3855) -> LM head (lm_train.wgsl) -> clean adjoint (:4736) ->
// fused weight gradients + update (:4980) -> spectral renorm (:5568).
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string.h>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/aideen_b200.h"
#include "kernels.cuh"

using namespace aideen;

namespace {

struct DevBufs {
  float *W = nullptr, *G = nullptr, *M1 = nullptr, *M2 = nullptr;
  float *S_in = nullptr;
  int32_t *tokens = nullptr, *targets = nullptr;
  float *signal = nullptr, *A = nullptr, *amat = nullptr;
  float *src = nullptr;  // [N][h][d] signal + slot anchor (attention source rows)
  // associative branch (AIDEEN_CFG_ASSOC): per (sequence, upper slot) bank value,
  // previous source [B][h][d] and usage [B][h], carried like MState; the stored
  // signal [N][h][d] (the payload on the upper slots) the FPM backward reads
  float *assoc_v = nullptr, *assoc_p = nullptr, *assoc_u = nullptr, *sig_store = nullptr;
  float *assoc_read = nullptr;  // [N][h][d] bank value each token read (upper slots)
  float *perm = nullptr;  // row-permutation scratch, max_tokens * h * d floats (on first use)
  float *Qh = nullptr, *Kh = nullptr, *Vh = nullptr, *alpha = nullptr, *nmix = nullptr,
        *rmix = nullptr, *scale = nullptr, *rho = nullptr, *Rsrc = nullptr;
  float *hstar = nullptr, *pre = nullptr, *pooled = nullptr, *hist = nullptr, *fpmctx = nullptr,
        *mstate = nullptr;
  int32_t *iters = nullptr;
  float *v = nullptr, *gpre = nullptr, *dl_dh = nullptr, *rhs_slot = nullptr, *nsg = nullptr;
  // Q | K | V head projections (and their gradients) of a (token, slot) row side
  // by side, [N][h][96]; Qh..Vh / dQ..dV point into them; Wcat [h][d][96] is
  // the matching operand of W_q | W_k | W_v (refreshed at every forward)
  float *qkv = nullptr, *dqkv = nullptr, *Wcat = nullptr;
  float *da = nullptr, *dn = nullptr, *dQ = nullptr, *dK = nullptr, *dV = nullptr,
        *dsig = nullptr, *dRc = nullptr, *dS = nullptr;
  float *lmp = nullptr, *Glm = nullptr, *Mlm1 = nullptr, *Mlm2 = nullptr;  // [V*d | V | d]
  float *y = nullptr, *lrms = nullptr, *logits = nullptr, *dy = nullptr, *ggp = nullptr,
        *loss_rows = nullptr, *scal = nullptr;  // scal: [n_active, loss]
  float *emb = nullptr;
  // pre-split LM-head GEMM operands: dlogits remainder [N][Vp]; y and y^T
  // halves [N][d], [d][N4]; W_lm halves [V][d]
  float *dlog_lo = nullptr, *yhi = nullptr, *ylo = nullptr, *yThi = nullptr, *yTlo = nullptr;
  float *whi = nullptr, *wlo = nullptr;
  float *colpart = nullptr;  // [blocks][Vp] per-block column sums of dlogits
  float2 *rowstats = nullptr;  // [N][ceil(V / 256)] softmax statistics from the logits GEMM
  unsigned long long *stats = nullptr;
  float *sigmas = nullptr;
  float *stage = nullptr;  // packed AllWeights staging for upload/download
  float *ws = nullptr;     // split-K partial sums of the tensor-core GEMM
  float *ws2 = nullptr;    // the same for GEMMs on the FPM-backward stream
  float *ws3 = nullptr;    // and for the attention-gradient side stream
  float *ws4 = nullptr;    // and for the FPM backward's second stream
  // FPM backward (allocated on first use): [N][h][d] unless noted
  float *fc = nullptr, *frp = nullptr, *fdl = nullptr, *fminner = nullptr, *fdm = nullptr,
        *fgpre = nullptr;
  float *fup = nullptr, *fkw = nullptr, *fdup = nullptr;  // [N][h][32]
  float *fA = nullptr, *fU = nullptr, *fgin = nullptr;    // [max_batch][h][nch][d]
  float *fcarry = nullptr;                                // [max_batch][h][d] TBPTT carry
  float *fprm = nullptr;                                   // [h][5][d] FPM slot parameters
  float *fpart = nullptr, *fpart_bw = nullptr;            // [5][max_batch*nch][h][d], [max_batch*nch][h]
  // sampled-softmax LM head and embedding update (allocated on first use)
  int32_t *lS = nullptr;     // [lcap] sampled vocabulary ids
  float *lWS = nullptr;      // [lcap][d] gathered (then updated) W_lm rows
  int *ints = nullptr;       // [0] K, [1] distinct tokens U
  unsigned int *lerr = nullptr;
  int32_t *tg_all = nullptr, *tok_all = nullptr;  // allgathered targets / tokens (data parallel)
  float *grad_all = nullptr;                       // allgathered embedding-gradient rows
  int32_t *cuniq = nullptr, *coff = nullptr, *cpos = nullptr;  // token CSR
  float *Me1 = nullptr, *Me2 = nullptr;             // embedding Adam moments [V][d]
};

}  // namespace

struct aideen_ctx {
  aideen_cfg cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  // side stream for the LM-head update (+ its hi/lo split), which only the
  // next LM-head call needs: it overlaps the next step's forward
  cudaStream_t side = nullptr;
  cudaEvent_t ev_grads = nullptr, ev_lm_done = nullptr;
  bool lm_pending = false;
  // training-step pipeline: Picard token chunks on a high-priority stream,
  // the LM head and adjoint of each finished chunk on the context stream
  static constexpr int kMaxChunks = 8;
  cudaStream_t pic = nullptr;
  cudaEvent_t ev_prep = nullptr, ev_pic[kMaxChunks] = {};
  // FPM backward stream: runs beside the attention-branch weight gradients
  cudaStream_t fst = nullptr;
  cudaStream_t fst2 = nullptr;  // the FPM backward's W_out gradient beside its other GEMMs
  cudaEvent_t ev_f0 = nullptr, ev_f2 = nullptr;
  cudaEvent_t ev_g0 = nullptr, ev_fdone = nullptr;
  // last pipeline chunk: dW_lm and the LM-head bias / gain sums on their own
  // stream beside the weight gradients; joined before the gradients are used
  cudaStream_t lmst = nullptr;
  cudaEvent_t ev_adj = nullptr, ev_lmg = nullptr;
  // attention-branch weight gradients: the GEMMs off the dsig chain run on ast
  cudaStream_t ast = nullptr;
  cudaEvent_t ev_da = nullptr, ev_dqkv = nullptr, ev_adone = nullptr;
  cudaEvent_t ev_dsig = nullptr;
  bool lmg_pending = false;
  // embedding update on its own stream (one GPU): the token CSR from the step's
  // start, the row Adam once dL/dpooled exists; the next gather joins it
  cudaStream_t est = nullptr;
  cudaEvent_t ev_e0 = nullptr, ev_emb = nullptr;
  cudaEvent_t ev_gz0 = nullptr, ev_gz = nullptr;  // gradient buffer zeroed on the embedding stream
  bool g_zeroed = false;                           // ... for this step's weight gradients
  bool emb_pending = false, emb_csr_ready = false;
  bool emb_done = false;  // this step's embedding update is already queued
  // The Adam moments are zero wherever the gradient always is (the columns
  // 32..d-1 of W_q/W_k/W_v and the rows 32..d-1 of W_o, which the 32-wide
  // heads never read): the update may skip those entries (Adam leaves an
  // entry with zero gradient and zero moments exactly unchanged).
  bool adam_dead_zero = true;
  // pinned mailbox of the synchronising reads: [0] adjoint error word,
  // [1] Picard error word, [2] loss; device addresses of the two words
  uint32_t *hbox = nullptr;
  unsigned int *d_adj_err = nullptr, *d_pic_err = nullptr;
  bool lm_reduced = false;  // this step's LM-head gradients were already summed over ranks
  // data-parallel train step with Adam: the core gradients are reduce-scattered
  // in two buckets (the attention-branch block as soon as its chain ends,
  // beside the FPM backward; the rest after it), each rank steps its own shard,
  // and the weights are all-gathered
  bool shard_step = false;
  bool fpm_prepared = false;  // the FPM backward's forward-only stage already ran this step
  bool assoc = false;         // AIDEEN_CFG_ASSOC: associative branch on the upper slots with FPM
  int fpm_comp_done = 0;  // FPM chunk composites [0, this) already formed this step
  int sm_budget = 0;      // SMs the GEMM / softmax / adjoint launches may use (0: all)
  // optional stage timeline of the pipelined step (AIDEEN_PIPE_TIMELINE=1, stderr)
  std::vector<std::pair<std::string, cudaEvent_t>> tl;
  std::vector<double> tl_host;  // host microseconds at each mark
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0;
  std::string err;
  unsigned long long launches = 0;
  size_t W_len = 0, lm_len = 0, max_tokens = 0;
  size_t lm_b = 0, lm_g = 0;  // offsets of b_lm and g_lm in the padded LM block
  long Vp = 0;            // logits row stride (vocab rounded up to 4 floats)
  size_t ws_floats = 0;   // capacity of each split-K workspace
  float signal_scale = 1.f;
  bool signal_zero = false;
  aideen_run last_run{};
  uint32_t N = 0;         // tokens of the last forward (B*T)
  // Activation rows are token-major inside the library (row t*B + b) so that a
  // run of tokens is a contiguous row range; the ABI keeps the caller's order
  // (row b*T + t) and permutes at the boundary.  (perm_B, perm_T) describe the
  // rows currently held (perm_B = 1: caller order, e.g. after aideen_adjoint_on).
  int perm_B = 1, perm_T = 0;
  uint32_t adj_N = 0;     // tokens of the last adjoint
  int nsg_rows = 0;       // rows of per-CTA NormScale-gradient partials the last adjoint wrote
  float adj_beta = 0.85f;
  bool lm_ready = false, emb_ready = false;
  size_t lcap = 0, gcap = 0;  // capacity of the sampled-set buffers / allgather buffers (rows)
  size_t lcur = 0;            // sampled-set bound of the current step (row stride of its logits)
  int *hK = nullptr;          // pinned host copy of the sampled-set size
  bool lk_pending = false;    // hK's copy is in flight
  cudaEvent_t ev_K = nullptr;
  bool lm_split_stale = true;  // W_lm changed since its hi/lo copies were made
  bool use_tc = true;     // tcgen05 GEMMs where the operand shapes allow
  DevBufs b;
  // opt-in per-kernel-class timing (aideen_profile): events around each launch
  bool prof = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> pev;
  int prof_phase = -1;    // >= 0: every launch is charged to this class
  double prof_ms[AIDEEN_PROF_CLASSES] = {};
  unsigned long long prof_n[AIDEEN_PROF_CLASSES] = {};
  Layout P{128, 1, 64};   // device (padded) layout
  Layout Lx{128, 1};      // packed reference layout at the boundary
};

namespace {

int set_err(aideen_ctx *c, int code, const std::string &msg) {
  if (c) c->err = msg;
  return code;
}

// Wait for the context stream, then report a bounded device-side wait that ran
// out since the last check (adjoint stage loads, Picard memory-row exchange).
// The flags are per device, so a context also sees another context's timeout
// on the same device.
int sync_and_check(aideen_ctx *ctx) {
  unsigned int adj = 0, pic = 0;
  cudaError_t e = cudaSuccess;
  if (ctx->hbox && ctx->d_adj_err && ctx->d_pic_err) {
    // both words into pinned memory and cleared on the stream, one wait
    cudaStream_t st = ctx->stream;
    e = cudaMemcpyAsync(&ctx->hbox[0], ctx->d_adj_err, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&ctx->hbox[1], ctx->d_pic_err, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_adj_err, 0, 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_pic_err, 0, 4, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    adj = ctx->hbox[0];
    pic = ctx->hbox[1];
  } else {
    e = adjoint_error_async(&adj, ctx->stream);
    if (e == cudaSuccess) e = picard_error_async(&pic, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  }
  if (e != cudaSuccess) return set_err(ctx, AIDEEN_E_CUDA, std::string("sync: ") + cudaGetErrorString(e));
  if (adj) return set_err(ctx, AIDEEN_E_TIMEOUT, "adjoint: a bounded stage wait ran out (its outputs are invalid)");
  if (pic) return set_err(ctx, AIDEEN_E_TIMEOUT, "Picard memory-row exchange: a bounded wait ran out");
  return AIDEEN_OK;
}

// Make the context stream wait for a deferred embedding update.
cudaError_t join_emb(aideen_ctx *c) {
  if (!c->emb_pending) return cudaSuccess;
  c->emb_pending = false;
  return cudaStreamWaitEvent(c->stream, c->ev_emb, 0);
}

// Make the context stream wait for a deferred LM-head update on the side stream.
cudaError_t join_side(aideen_ctx *c) {
  if (!c->lm_pending) return cudaSuccess;
  c->lm_pending = false;
  return cudaStreamWaitEvent(c->stream, c->ev_lm_done, 0);
}

#define CU(expr)                                                                       \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess)                                                             \
      return set_err(ctx, AIDEEN_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)
int prof_class(const char *expr, int phase) {
  if (phase >= 0) return phase;
  if (strstr(expr, "launch_picard")) return AIDEEN_PROF_PICARD;
  if (strstr(expr, "launch_adjoint")) return AIDEEN_PROF_ADJOINT;
  if (strstr(expr, "source_grad")) return AIDEEN_PROF_OTHER;
  if (strstr(expr, "gemm_any") || strstr(expr, "gemm_split")) return AIDEEN_PROF_GEMM;
  if (strstr(expr, "launch_softmax_ce")) return AIDEEN_PROF_LM_SOFTMAX;
  if (strstr(expr, "launch_adam") || strstr(expr, "launch_clipped_sgd")) return AIDEEN_PROF_OPTIMIZER;
  return AIDEEN_PROF_OTHER;
}

// A launch of one of this library's kernels (timed per class when profiling).
#define KL(expr)                                                                       \
  do {                                                                                 \
    ctx->launches++;                                                                   \
    cudaEvent_t _e0 = nullptr, _e1 = nullptr;                                          \
    if (ctx->prof) {                                                                   \
      cudaEventCreate(&_e0);                                                           \
      cudaEventCreate(&_e1);                                                           \
      cudaEventRecord(_e0, ctx->stream);                                               \
    }                                                                                  \
    cudaError_t _e = (expr);                                                           \
    ctx->launches += tc_take_extra_launches();                                         \
    if (ctx->prof) {                                                                   \
      cudaEventRecord(_e1, ctx->stream);                                               \
      ctx->pev.push_back({prof_class(#expr, ctx->prof_phase), {_e0, _e1}});                            \
    }                                                                                  \
    if (_e != cudaSuccess)                                                             \
      return set_err(ctx, AIDEEN_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)
#define CHK(expr)                  \
  do {                             \
    int _r = (expr);               \
    if (_r != AIDEEN_OK) return _r; \
  } while (0)

template <typename T>
cudaError_t dalloc(T **p, size_t n) {
  if (n == 0) n = 1;
  return cudaMalloc((void **)p, n * sizeof(T));
}

int copy_in(aideen_ctx *ctx, void *dst, const void *src, size_t bytes, int where) {
  if (bytes == 0) return AIDEEN_OK;
  if (!src) return set_err(ctx, AIDEEN_E_INVALID, "null input pointer");
  CU(cudaMemcpyAsync(dst, src, bytes,
                     where == AIDEEN_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                     ctx->stream));
  return AIDEEN_OK;
}

cudaError_t ensure_perm(aideen_ctx *ctx) {
  if (ctx->b.perm) return cudaSuccess;
  return dalloc(&ctx->b.perm, ctx->max_tokens * ctx->cfg.h_slots * ctx->cfg.d_model);
}

// Copy `blocks` sets of B*T rows (len 4-byte words each) from the caller's
// order into the library's token-major order.
int copy_in_rows(aideen_ctx *ctx, void *dst, const void *src, int B, int T, int blocks, size_t len, int where) {
  const size_t bytes = (size_t)B * T * blocks * len * 4;
  if (bytes == 0) return AIDEEN_OK;
  if (!src) return set_err(ctx, AIDEEN_E_INVALID, "null input pointer");
  if (B == 1 || T == 1) return copy_in(ctx, dst, src, bytes, where);
  const void *from = src;
  if (where != AIDEEN_DEVICE) {
    CU(ensure_perm(ctx));
    CU(cudaMemcpyAsync(ctx->b.perm, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    from = ctx->b.perm;
  }
  KL(launch_permute_rows(from, dst, B, T, blocks, len, true, ctx->stream));
  return AIDEEN_OK;
}

bool no_sharded_update() { return getenv("AIDEEN_NO_SHARDED_UPDATE") != nullptr; }  // per step (tests toggle it)

bool tf32_grads_enabled() {
  static const bool on = getenv("AIDEEN_GRAD_3XTF32") == nullptr;
  return on;
}

GemmArgs gemm(int M, int N, int K, int batch, const float *A, long lda, long sA, bool tA,
              const float *B, long ldb, long sB, bool tB, float *C, long ldc, long sC,
              float alpha = 1.f, float beta = 0.f, const float *abias = nullptr, long sbias = 0) {
  GemmArgs g;
  g.M = M; g.N = N; g.K = K; g.batch = batch;
  g.A = A; g.lda = lda; g.strideA = sA; g.transA = tA;
  g.B = B; g.ldb = ldb; g.strideB = sB; g.transB = tB;
  g.C = C; g.ldc = ldc; g.strideC = sC;
  g.alpha = alpha; g.beta = beta; g.abias = abias; g.strideAbias = sbias;
  g.tf32 = false;
  g.col_group = 0; g.group_stride = 0;
  return g;
}

// The same GEMM with single TF32 products (weight gradients, whose 1e-3
// accuracy bar TF32 rounding meets; the forward keeps 3xTF32)
GemmArgs tf32(GemmArgs g) {
  g.tf32 = tf32_grads_enabled();
  return g;
}

// Pre-split GEMM (operands as tf32 high parts in g.A / g.B plus remainders).
cudaError_t gemm_split(aideen_ctx *ctx, const GemmArgs &g, const float *A_lo, const float *B_lo,
                       const float *row_bias = nullptr, float2 *row_stats = nullptr) {
  if (!tc_split_supported(g, A_lo, B_lo)) return cudaErrorInvalidValue;
  return tc_gemm_split(g, A_lo, B_lo, ctx->stream, ctx->b.ws, ctx->ws_floats, ctx->sm_budget, row_bias,
                       row_stats);
}

// GEMM dispatch: tcgen05 (3xTF32) when supported for these operands, else CUDA cores.
cudaError_t gemm_any(aideen_ctx *ctx, const GemmArgs &g) {
  if (ctx->use_tc && tc_gemm_supported(g)) {
    if (g.col_group > 0 && (size_t)g.batch * g.M * g.N > ctx->ws_floats) {
      // the grouped output needs the workspace: one GEMM per column group instead
      for (int c0 = 0; c0 < g.N; c0 += g.col_group) {
        GemmArgs gg = g;
        gg.N = g.N - c0 < g.col_group ? g.N - c0 : g.col_group;
        gg.B = g.transB ? g.B + (size_t)c0 * g.ldb : g.B + c0;
        gg.C = g.C + (size_t)(c0 / g.col_group) * g.group_stride;
        gg.col_group = 0;
        const cudaError_t e = tc_gemm(gg, ctx->stream, ctx->b.ws, ctx->ws_floats);
        if (e != cudaSuccess) return e;
        if (c0 + g.col_group < g.N) ++tc_extra_launches;
      }
      return cudaSuccess;
    }
    return tc_gemm(g, ctx->stream, ctx->b.ws, ctx->ws_floats);
  }
  return gemm_f32(g, ctx->stream);
}

int check_run(aideen_ctx *ctx, const aideen_run *r) {
  if (!r) return set_err(ctx, AIDEEN_E_INVALID, "null run");
  if (r->batch == 0 || r->seq_len == 0 || r->batch > ctx->cfg.max_batch ||
      r->seq_len > ctx->cfg.max_seq_len)
    return set_err(ctx, AIDEEN_E_INVALID, "batch/seq_len outside the context caps");
  if (r->max_iters == 0) return set_err(ctx, AIDEEN_E_INVALID, "max_iters must be >= 1");
  if (r->anderson_m > 3) return set_err(ctx, AIDEEN_E_UNSUPPORTED, "forward anderson_m > 3");
  return AIDEEN_OK;
}

// Everything after S_in is resident: projection, slot attention, Picard, pool.
// Projection and slot attention of a forward (everything before the Picard solve).
// Projection and slot attention of rows [r0, r0 + R) (every op is row-local).
int run_forward_prep_rows(aideen_ctx *ctx, const aideen_run *r, long r0, int R) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const Layout &L = ctx->P;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const float *W = b.W;
  const long hd = (long)h * d, H32 = (long)h * kHeadDim;
  float *signal = b.signal + r0 * hd;
  if (ctx->signal_zero) {
    CU(cudaMemsetAsync(signal, 0, (size_t)R * hd * sizeof(float), st));
  } else {
    // signal[n][s][:] = sigma * S_in[n] . W_in[s]   (deq_slot_attn_unified_clean.wgsl:762-804)
    KL(gemm_any(ctx, gemm(R, d, d, h, b.S_in + r0 * d, d, 0, false, W + L.win, d, (long)d * d, false, signal,
                     hd, d, ctx->signal_scale)));
  }
  if (r->slot_coord) {
    // 32-wide K/V/Q heads of src = signal + anchor (:281-355); src is kept for the backward
    float *src = b.src + r0 * hd;
    KL(launch_add_rowbias(src, signal, W + L.slot_anchor, R, (size_t)hd, st));
    // Q | K | V heads in one GEMM against the packed [d][96] operand
    const long H96 = (long)h * 96;
    if (r0 == 0) KL(launch_pack_qkv(W, L.wq, L.wk, L.wv, h, d, b.Wcat, st));
    KL(gemm_any(ctx, gemm(R, 96, d, h, src, hd, d, false, b.Wcat, 96, (long)d * 96, false, b.qkv + r0 * H96, H96,
                          96)));
    AttnArgs a{};
    a.h = h; a.d = d; a.W = W; a.off_qb = L.q_bias; a.off_kb = L.k_bias; a.off_anchor = L.slot_anchor;
    a.Qh = b.Qh + r0 * H96; a.Kh = b.Kh + r0 * H96; a.Vh = b.Vh + r0 * H96; a.qkv_ld = 96;
    a.alpha = b.alpha + r0 * h * h; a.nmix = b.nmix + r0 * H32; a.rmix = b.rmix + r0 * h;
    a.signal = signal; a.amat = b.amat + r0 * hd; a.A = b.A + r0 * hd;
    a.scale = b.scale + r0 * h; a.rho = b.rho + r0 * h; a.Rsrc = b.Rsrc + r0 * h;
    KL(launch_attn_softmax(a, R, st));
    // attn[o] = sum_k W_o[s][k*d + o] n[k]  (:452-470)
    KL(gemm_any(ctx, gemm(R, d, kHeadDim, h, a.nmix, H32, kHeadDim, false, W + L.wo, d,
                     (long)d * d, false, b.amat + r0 * hd, hd, d)));
    KL(launch_attn_scale(a, R * h, st));
  }
  if (!r->fpm) CU(cudaMemsetAsync(b.hist + r0 * hd, 0, (size_t)R * hd * sizeof(float), st));
  return AIDEEN_OK;
}

// Projection and slot attention of a forward (everything before the Picard solve).
int run_forward_prep(aideen_ctx *ctx, const aideen_run *r) {
  ctx->perm_B = r->batch;
  ctx->perm_T = r->seq_len;
  return run_forward_prep_rows(ctx, r, 0, r->batch * r->seq_len);
}

PicardArgs picard_args(aideen_ctx *ctx, const aideen_run *r) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const Layout &L = ctx->P;
  DevBufs &b = ctx->b;
  const float *W = b.W;
  PicardArgs p{};
  p.B = r->batch; p.T = r->seq_len; p.h = h; p.d = d; p.max_iters = r->max_iters;
  p.slot_coord = r->slot_coord ? 1 : 0;
  p.eps = r->epsilon; p.blend = r->fpm ? 0.2f : r->damping;
  p.alpha_m = r->fpm_alpha_m; p.tau = r->fpm_tau; p.gate_min = r->fpm_read_gate_min;
  p.W = W;
  p.off_ns = L.nscale; p.off_anchor = L.slot_anchor; p.off_hscale = L.hist_scale;
  p.off_hbias = L.hist_bias; p.off_wkm = L.w_k_mem; p.off_wqm = L.w_q_mem; p.off_bread = L.b_read_mem;
  p.off_wgate = L.w_write_gate; p.off_bwrite = L.b_write_mem; p.off_wkw = L.w_k_write;
  p.off_wvw = L.w_v_write; p.off_bdelta = L.b_delta; p.off_wup = L.w_retain_up;
  p.off_wdown = L.w_retain_down; p.off_bret = L.b_retain; p.off_alog = L.alog; p.off_wx = L.wx;
  p.signal = b.signal; p.A = b.A;
  p.hstar = b.hstar; p.pre = b.pre; p.hist = b.hist; p.fpmctx = b.fpmctx; p.mstate = b.mstate;
  p.iters = b.iters;
  p.t0 = 0;
  p.t1 = r->seq_len;
  p.assoc = ctx->assoc && r->fpm ? 1 : 0;
  p.off_alpha_assoc = L.alpha_assoc;
  p.s_in = b.S_in;
  p.assoc_v = b.assoc_v; p.assoc_p = b.assoc_p; p.assoc_u = b.assoc_u; p.sig_store = b.sig_store;
  p.assoc_read = b.assoc_read;
  p.anderson_m = r->anderson_m >= 2 ? (int)r->anderson_m : 0;  // depth 1 never mixes
  return p;
}

int read_solve_stats(aideen_ctx *ctx, const aideen_run *r, aideen_stats *stats) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const int N = r->batch * r->seq_len;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  CU(cudaMemsetAsync(b.stats, 0, 4 * sizeof(unsigned long long), st));
  KL(launch_solve_stats(b.iters, b.hstar, N * h, d, r->max_iters, b.stats, st));
  unsigned long long hs[4];
  CU(cudaMemcpyAsync(hs, b.stats, sizeof(hs), cudaMemcpyDeviceToHost, st));
  unsigned int pic_err = 0;
  CU(picard_error_async(&pic_err, st));
  CU(cudaStreamSynchronize(st));
  if (pic_err) return set_err(ctx, AIDEEN_E_TIMEOUT, "Picard memory-row exchange: a bounded wait ran out");
  stats->total_iters = hs[0];
  stats->max_iters_seen = (uint32_t)hs[1];
  stats->unconverged = (uint32_t)hs[2];
  stats->nonfinite = (uint32_t)hs[3];
  stats->solves = (uint32_t)(N * h);
  return AIDEEN_OK;
}

int run_forward(aideen_ctx *ctx, const aideen_run *r, aideen_stats *stats) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const int N = r->batch * r->seq_len;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  CHK(run_forward_prep(ctx, r));
  const PicardArgs p = picard_args(ctx, r);
  KL(launch_picard(p, r->fpm != 0, st));
  KL(launch_pool_rmsnorm(b.hstar, ctx->lm_ready ? b.lmp + ctx->lm_g : nullptr,
                         b.pooled, ctx->lm_ready ? b.y : nullptr, b.lrms, N, h, d, st));
  ctx->last_run = *r;
  ctx->N = N;
  return stats ? read_solve_stats(ctx, r, stats) : AIDEEN_OK;
}

int run_lm_head(aideen_ctx *ctx, int N, float *loss_out) {
  if (!ctx->lm_ready) return set_err(ctx, AIDEEN_E_INVALID, "LM head not uploaded");
  ctx->prof_phase = AIDEEN_PROF_LM_SOFTMAX;  // every LM-head launch in one profile class
  struct PhaseReset { aideen_ctx *c; ~PhaseReset() { c->prof_phase = -1; } } phase_reset{ctx};
  const int d = ctx->cfg.d_model, V = ctx->cfg.vocab;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const float *Wlm = b.lmp, *glm = b.lmp + ctx->lm_g;
  const long Vp = ctx->Vp;
  CU(join_side(ctx));
  KL(launch_count_active(b.targets, N, b.scal, st));
  // The three LM-head GEMMs run on pre-split operands: W_lm halves are
  // refreshed once per change of W_lm, y and y^T halves per call (y^T makes
  // dW_lm's B operand K-major), and the softmax writes dlogits already split.
  if (ctx->lm_split_stale) {
    KL(launch_split_hilo(Wlm, b.whi, b.wlo, (size_t)V * d, st));
    ctx->lm_split_stale = false;
  }
  const long N4 = (N + 3) / 4 * 4;
  KL(launch_split_hilo(b.y, b.yhi, b.ylo, (size_t)N * d, st));
  KL(launch_transpose_split(b.y, N, d, d, b.yThi, b.yTlo, N4, st));
  // logits[n][v] = y[n] . W_lm[v]
  KL(gemm_split(ctx, gemm(N, V, d, 1, b.yhi, d, 0, false, b.whi, d, 0, true, b.logits, Vp, 0), b.ylo, b.wlo));
  // vocabularies whose column accumulator fits one block's shared memory fuse
  // the b_lm column sums into the softmax; larger ones sum dlogits afterwards
  const bool fused_colsum = Vp * 4 <= 227 * 1024;
  const int nrb = softmax_rows_blocks(N);
  if (fused_colsum)
    KL(launch_softmax_ce_split(b.logits, b.lmp + ctx->lm_b, b.targets, b.scal, N, V, Vp, b.loss_rows,
                               b.dlog_lo, b.colpart, st));
  else
    KL(launch_softmax_ce(b.logits, b.lmp + ctx->lm_b, b.targets, b.scal, N, V, Vp, b.loss_rows, b.dlog_lo, st));
  KL(launch_sum(b.loss_rows, N, b.scal + 1, st));
  // dy[n][j] = sum_v dlogits[n][v] W_lm[v][j]
  KL(gemm_split(ctx, gemm(N, d, V, 1, b.logits, Vp, 0, false, b.whi, d, 0, false, b.dy, d, 0), b.dlog_lo,
                b.wlo));
  // dW_lm[v][j] = sum_n dlogits[n][v] y^T[j][n]
  KL(gemm_split(ctx, gemm(V, d, N, 1, b.logits, Vp, 0, true, b.yThi, N4, 0, true, b.Glm, d, 0), b.dlog_lo,
                b.yTlo));
  // b_lm gradient: column sums of dlogits from the softmax's per-block partials
  if (fused_colsum) {
    KL(launch_colsum(b.colpart, nrb, V, Vp, b.Glm + ctx->lm_b, V, 0, false, st));
  } else {
    KL(launch_colsum(b.logits, N, V, Vp, b.Glm + ctx->lm_b, V, 0, false, st));
    KL(launch_colsum(b.dlog_lo, N, V, Vp, b.Glm + ctx->lm_b, V, 0, true, st));
  }
  KL(launch_rmsnorm_bwd(b.dy, b.pooled, b.lrms, glm, b.dl_dh, b.ggp, N, d, st));
  KL(launch_colsum(b.ggp, N, d, d, b.Glm + ctx->lm_g, d, 0, false, st));
  if (loss_out) {
    if (ctx->hbox) {
      CU(cudaMemcpyAsync(&ctx->hbox[2], b.scal + 1, sizeof(float), cudaMemcpyDeviceToHost, st));
      CU(cudaStreamSynchronize(st));
      memcpy(loss_out, &ctx->hbox[2], sizeof(float));
    } else {
      CU(cudaMemcpyAsync(loss_out, b.scal + 1, sizeof(float), cudaMemcpyDeviceToHost, st));
      CU(cudaStreamSynchronize(st));
    }
  }
  return AIDEEN_OK;
}

int run_adjoint(aideen_ctx *ctx, int N, const float *pre_a, const float *pre_b,
                const float *rhs_tok, const float *rhs_slot, uint32_t iters, float beta,
                uint32_t anderson_m) {
  if (anderson_m > 4) return set_err(ctx, AIDEEN_E_UNSUPPORTED, "anderson_m > 4");
  AdjointArgs a{};
  a.N = N; a.h = ctx->cfg.h_slots; a.d = ctx->cfg.d_model; a.iters = iters;
  a.anderson_m = anderson_m; a.beta = beta;
  a.pre_a = pre_a; a.pre_b = pre_b; a.rhs_tok = rhs_tok; a.rhs_slot = rhs_slot;
  a.NS = ctx->b.W + ctx->P.nscale; a.v = ctx->b.v; a.gpre = ctx->b.gpre; a.nsg_cta = ctx->b.nsg;
  int grid = 0;
  KL(launch_adjoint(a, ctx->stream, &grid));
  ctx->nsg_rows = grid;
  ctx->adj_N = N;
  ctx->adj_beta = beta;
  return AIDEEN_OK;
}

int run_fpm_backward(aideen_ctx *ctx, bool prepare_only = false);
int fpm_args(aideen_ctx *ctx, FpmBwdArgs &a);
void tl_mark(aideen_ctx *ctx, const char *name, cudaStream_t s);

// Gradient buckets of the sharded update: [0, W_x) holds W_q..W_in and their
// biases (the attention-branch chain writes them), [W_x, end) the rest.
void grad_buckets(const aideen_ctx *ctx, size_t off[2], size_t len[2]) {
  off[0] = 0;
  len[0] = ctx->P.wx;
  off[1] = ctx->P.wx;
  len[1] = ctx->W_len - ctx->P.wx;
}

// Sum bucket [off, off + len) of the gradients over ranks, leaving this rank's
// shard [off + rank*cnt, +cnt) summed (cnt = len / nranks) and the remainder
// past cnt*nranks summed on every rank.
int reduce_scatter_bucket(aideen_ctx *ctx, size_t off, size_t len) {
  const size_t n = (size_t)ctx->nranks, cnt = len / n, rem = len - cnt * n;
  float *G = ctx->b.G + off;
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess && cnt)
    r = ncclReduceScatter(G, G + (size_t)ctx->rank * cnt, cnt, ncclFloat, ncclSum, ctx->comm, ctx->stream);
  if (r == ncclSuccess && rem) r = ncclAllReduce(G + cnt * n, G + cnt * n, rem, ncclFloat, ncclSum, ctx->comm, ctx->stream);
  const ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess)
    return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclReduceScatter: ") +
                                           ncclGetErrorString(r != ncclSuccess ? r : r2));
  return AIDEEN_OK;
}

int run_weight_grads(aideen_ctx *ctx, bool want_ds) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const int N = ctx->N;
  if (N == 0 || ctx->adj_N != ctx->N)
    return set_err(ctx, AIDEEN_E_INVALID, "weight grads need a forward and an adjoint over the same tokens");
  const Layout &L = ctx->P;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const float *W = b.W;
  float *G = b.G;
  const bool sc = ctx->last_run.slot_coord != 0;
  const int H32 = h * kHeadDim;
  if (ctx->g_zeroed) {
    CU(cudaStreamWaitEvent(st, ctx->ev_gz, 0));
    ctx->g_zeroed = false;
  } else {
    CU(cudaMemsetAsync(G, 0, ctx->W_len * sizeof(float), st));
  }
  // The FPM backward writes only its own gradient segments: without
  // profiling it runs on its own stream (and split-K workspace) beside the
  // attention-branch gradients below.
  const bool fork_fpm = ctx->last_run.fpm && !ctx->prof && ctx->fst;
  if (fork_fpm) {
    CU(cudaEventRecord(ctx->ev_g0, st));
    CU(cudaStreamWaitEvent(ctx->fst, ctx->ev_g0, 0));
    cudaStream_t keep_st = ctx->stream;
    float *keep_ws = ctx->b.ws;
    ctx->stream = ctx->fst;
    ctx->b.ws = ctx->b.ws2;
    const int rc = run_fpm_backward(ctx);
    ctx->stream = keep_st;
    ctx->b.ws = keep_ws;
    CHK(rc);
    tl_mark(ctx, "fpm_bwd", ctx->fst);
    CU(cudaEventRecord(ctx->ev_fdone, ctx->fst));
  }
  // Off the dsig chain (attn scale -> dn -> softmax backward -> dsig -> dsrc
  // -> W_in gradient), the W_o / W_q,k,v gradient GEMMs and the bias sums run
  // on a side stream with their own split-K workspace.
  const bool fork_attn = sc && !ctx->prof && ctx->ast;
  cudaStream_t sst = fork_attn ? ctx->ast : st;
  auto on_side = [&](auto &&f) -> cudaError_t {
    if (!fork_attn) return f();
    float *keep_ws = b.ws;
    ctx->stream = ctx->ast;
    b.ws = b.ws3;
    const cudaError_t e = f();
    ctx->stream = st;
    b.ws = keep_ws;
    return e;
  };
  if (fork_attn) {
    if (!fork_fpm) CU(cudaEventRecord(ctx->ev_g0, st));
    CU(cudaStreamWaitEvent(ctx->ast, ctx->ev_g0, 0));
  }
  KL(launch_colsum(b.nsg, ctx->nsg_rows, d, d, G + L.nscale, d, 0, false, sst));
  AttnBwdArgs a{};
  a.h = h; a.d = d; a.W = W; a.off_qb = L.q_bias; a.off_kb = L.k_bias; a.off_anchor = L.slot_anchor;
  a.gpre = b.gpre; a.amat = b.amat; a.scale = b.scale; a.rho = b.rho; a.Rsrc = b.Rsrc;
  a.signal = b.signal; a.da = b.da; a.dRc = b.dRc; a.dn = b.dn; a.nmix = b.nmix; a.rmix = b.rmix;
  a.alpha = b.alpha; a.Qh = b.Qh; a.Kh = b.Kh; a.Vh = b.Vh; a.dQ = b.dQ; a.dK = b.dK; a.dV = b.dV;
  a.qkv_ld = 96;
  const long H96 = (long)h * 96;
  if (sc) {
    KL(launch_attn_bwd_scale(a, N * h, st));
    if (fork_attn) {
      CU(cudaEventRecord(ctx->ev_da, st));
      CU(cudaStreamWaitEvent(ctx->ast, ctx->ev_da, 0));
      // dsig's initial value needs only g_pre and attn_bwd_scale's dRc: on
      // the side stream beside dn and the softmax backward
      KL(launch_dsig_init(a, b.dsig, N * h, 1, sst));
      CU(cudaEventRecord(ctx->ev_dsig, sst));
    }
    // gW_o[s][c][o] = sum_n n[n][s][c] da[n][s][o]
    KL(on_side([&] {
      return gemm_any(ctx, tf32(gemm(kHeadDim, d, N, h, b.nmix, H32, kHeadDim, true, b.da, (long)h * d, d, false,
                                     G + L.wo, d, (long)d * d)));
    }));
    // dn[n][s][c] = sum_o da[n][s][o] W_o[s][c*d + o]
    KL(gemm_any(ctx, gemm(N, kHeadDim, d, h, b.da, (long)h * d, d, false, W + L.wo, d, (long)d * d, true,
                     b.dn, H32, kHeadDim)));
    tl_mark(ctx, "wg_o", st);
    KL(launch_attn_bwd_softmax(a, N, st));
    if (fork_attn) {
      CU(cudaEventRecord(ctx->ev_dqkv, st));
      CU(cudaStreamWaitEvent(ctx->ast, ctx->ev_dqkv, 0));
    }
    // gW_{q,k,v}[s][j][c] = sum_n src[n][s][j] d{Q,K,V}[n][s][c]
    // as one product of width 96 whose column groups of 32 land in W_q, W_k, W_v
    KL(on_side([&] {
      GemmArgs gq = tf32(gemm(d, 96, N, h, b.src, (long)h * d, d, true, b.dqkv, H96, 96, false, G + L.wq, d,
                              (long)d * d));
      gq.col_group = kHeadDim;
      gq.group_stride = (long)(L.wk - L.wq);
      return gemm_any(ctx, gq);
    }));
    KL(launch_colsum(b.dQ, N, H32, H96, G + L.q_bias, kHeadDim, d, false, sst, 96));
    KL(launch_colsum(b.dK, N, H32, H96, G + L.k_bias, kHeadDim, d, false, sst, 96));
    tl_mark(ctx, "wg_qkv", st);
    if (fork_attn) CU(cudaStreamWaitEvent(st, ctx->ev_dsig, 0));
    else KL(launch_dsig_init(a, b.dsig, N * h, 1, st));
    // dsrc[n][s][j] += sum_c d{Q|K|V}[n][s][c] Wcat[s][j][c], one GEMM of depth 96
    KL(gemm_any(ctx, gemm(N, d, 96, h, b.dqkv, H96, 96, false, b.Wcat, 96, (long)d * 96, true, b.dsig,
                          (long)h * d, d, 1.f, 1.f)));
    tl_mark(ctx, "dsrc", st);
    if (fork_attn) CU(cudaEventRecord(ctx->ev_adone, ctx->ast));
    KL(launch_colsum(b.dsig, N, h * d, (long)h * d, G + L.slot_anchor, h * d, 0, false, st));
  } else {
    KL(launch_dsig_init(a, b.dsig, N * h, 0, st));
  }
  // associative slots: their branch holds the payload, not their signal, so the
  // direct term g_pre reaches W_in and S_in from the lower slots only (the
  // anchor above keeps it)
  if (ctx->assoc && ctx->last_run.fpm) {
    KL(launch_sub_upper_slots(b.dsig, b.gpre, N, h, d, st));
    // the reference's alpha_assoc gradient from the adjoint and the values read
    KL(launch_assoc_alpha_grad(b.v, b.assoc_read, W + L.alpha_assoc, N, h, d, G + L.alpha_assoc, st));
  }
  if (!ctx->signal_zero) {
    // gW_in[s][j][o] = sigma * sum_n S_in[n][j] dsig[n][s][o]
    KL(gemm_any(ctx, tf32(gemm(d, d, N, h, b.S_in, d, 0, true, b.dsig, (long)h * d, d, false, G + L.win, d,
                               (long)d * d, ctx->signal_scale))));
    tl_mark(ctx, "wg_in", st);
    if (want_ds) {
      // the source gradient (not a weight gradient: profiled with "other")
      auto source_grad_gemm = [&](int s) {
        return gemm_any(ctx, gemm(N, d, d, 1, b.dsig + (size_t)s * d, (long)h * d, 0, false,
                                  W + L.win + (size_t)s * d * d, d, 0, true, b.dS, d, 0, ctx->signal_scale,
                                  s == 0 ? 0.f : 1.f));
      };
      for (int s = 0; s < h; ++s) KL(source_grad_gemm(s));
    }
  } else if (want_ds) {
    CU(cudaMemsetAsync(b.dS, 0, (size_t)N * d * sizeof(float), st));
  }
  if (fork_attn) CU(cudaStreamWaitEvent(st, ctx->ev_adone, 0));
  tl_mark(ctx, "attn_grads", st);
  size_t boff[2], blen[2];
  grad_buckets(ctx, boff, blen);
  if (ctx->shard_step) CHK(reduce_scatter_bucket(ctx, boff[0], blen[0]));  // beside the FPM backward
  if (ctx->shard_step) tl_mark(ctx, "rs0", st);
  if (fork_fpm) CU(cudaStreamWaitEvent(st, ctx->ev_fdone, 0));
  else if (ctx->last_run.fpm) CHK(run_fpm_backward(ctx));
  if (ctx->shard_step) CHK(reduce_scatter_bucket(ctx, boff[1], blen[1]));
  if (ctx->shard_step) tl_mark(ctx, "rs1", st);
  return AIDEEN_OK;
}

// FPM backward arguments over the last forward (allocates the FPM buffers once).
int fpm_args(aideen_ctx *ctx, FpmBwdArgs &a) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const int B = ctx->last_run.batch, T = ctx->last_run.seq_len;
  const Layout &L = ctx->P;
  DevBufs &b = ctx->b;
  const size_t Nhd = ctx->max_tokens * h * d, NH32 = ctx->max_tokens * h * kRank;
  const int CH = fpm_chunk_len(d);
  const size_t nch_max = (ctx->cfg.max_seq_len + CH - 1) / CH;
  const size_t chunk_rows = (size_t)ctx->cfg.max_batch * nch_max;
  if (!b.fc) {
    cudaError_t e = cudaSuccess;
    auto A = [&](float **p, size_t n) { if (e == cudaSuccess) e = dalloc(p, n); };
    A(&b.fc, Nhd); A(&b.frp, Nhd); A(&b.fdl, Nhd); A(&b.fminner, Nhd); A(&b.fdm, Nhd); A(&b.fgpre, Nhd);
    A(&b.fup, NH32); A(&b.fkw, NH32); A(&b.fdup, NH32);
    A(&b.fA, chunk_rows * h * d); A(&b.fU, chunk_rows * h * d); A(&b.fgin, chunk_rows * h * d);
    A(&b.fpart, 5 * chunk_rows * h * d); A(&b.fpart_bw, chunk_rows * h); A(&b.fprm, (size_t)5 * h * d);
    CU(e);
  }
  const float *W = b.W;
  a = FpmBwdArgs{};
  a.B = B; a.T = T; a.h = h; a.d = d; a.nch = (T + CH - 1) / CH; a.W = W;
  a.off_bdelta = L.b_delta; a.off_bret = L.b_retain; a.off_wgate = L.w_write_gate;
  a.off_bwrite = L.b_write_mem; a.off_alog = L.alog; a.off_wx = L.wx;
  a.hstar = b.hstar; a.hist = b.hist; a.c = b.fc; a.rpre = b.frp; a.dpre = b.fdl; a.v = b.v;
  a.minner = b.fminner; a.cA = b.fA; a.cU = b.fU; a.gin = b.fgin; a.dm = b.fdm; a.gpre = b.fgpre;
  a.carry = b.fcarry; a.part = b.fpart; a.part_bw = b.fpart_bw; a.slot_prm = b.fprm;
  a.ch0 = 0;
  a.ch1 = 0;
  return AIDEEN_OK;
}

// FPM memory backward over the last forward's chunk (fpm_bwd.cu); adds the
// FPM parameters' gradients to G and advances the TBPTT carry.
int run_fpm_backward(aideen_ctx *ctx, bool prepare_only) {
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const int B = ctx->last_run.batch, T = ctx->last_run.seq_len, N = B * T;
  const Layout &L = ctx->P;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  FpmBwdArgs a;
  CHK(fpm_args(ctx, a));
  const float *W = b.W;
  float *G = b.G;
  const int R = kRank, HR = h * kRank;
  const long hd = (long)h * d;
  ctx->prof_phase = AIDEEN_PROF_FPM_BWD;
  struct PhaseReset { aideen_ctx *c; ~PhaseReset() { c->prof_phase = -1; } } phase_reset{ctx};
  if (!ctx->fpm_prepared || prepare_only) {
  // forward-only stage: c and the rank-32 projections (needs h*, not v)
  // c = (h* + stored signal) / 2: the payload on the associative slots
  KL(launch_fpm_c(b.hstar, ctx->assoc ? b.sig_store : b.signal, b.fc, (size_t)N * h * d, st));
  // up[n][s][r] = sum_j c W_retain_up[s][j][r];  kw = same with W_k_write
  KL(gemm_any(ctx, gemm(N, R, d, h, b.fc, hd, d, false, W + L.w_retain_up, R, (long)d * R, false,
                   b.fup, HR, R)));
  KL(gemm_any(ctx, gemm(N, R, d, h, b.fc, hd, d, false, W + L.w_k_write, R, (long)d * R, false,
                   b.fkw, HR, R)));
  // retain / proposal pre-activations (biases are added by the chunk kernels)
  KL(gemm_any(ctx, gemm(N, d, R, h, b.fup, HR, R, false, W + L.w_retain_down, d, (long)R * d, false,
                   b.frp, hd, d)));
  KL(gemm_any(ctx, gemm(N, d, R, h, b.fkw, HR, R, false, W + L.w_v_write, d, (long)R * d, false,
                   b.fdl, hd, d)));
  }
  if (prepare_only) {
    ctx->fpm_prepared = true;
    return AIDEEN_OK;
  }
  ctx->fpm_prepared = false;
  if (ctx->fpm_comp_done == 0) KL(launch_fpm_slot_params(a, st));
  // chunk composites not already formed during the pipelined step
  a.ch0 = ctx->fpm_comp_done;
  a.ch1 = a.nch;
  KL(launch_fpm_composite(a, st));
  a.ch0 = 0;
  a.ch1 = 0;
  ctx->fpm_comp_done = 0;
  tl_mark(ctx, "f_comp", st);
  KL(launch_fpm_carry(a, st));
  KL(launch_fpm_chunks(a, st));
  tl_mark(ctx, "f_chunks", st);
  // W_out[r][c] = sum_{n,s} dm[n][s][r] m_inner[n][s][c]: needs only the
  // replay's outputs, so it runs on a second stream (own split-K workspace)
  // beside the finalize and the rank-32 gradient GEMMs below
  const bool wout_side = ctx->fst2 && st == ctx->fst && !ctx->prof;
  auto wout_gemm = [&] {
    return gemm_any(ctx, tf32(gemm(d, d, N * h, 1, b.fdm, d, 0, true, b.fminner, d, 0, false, G + L.wout, d, 0)));
  };
  if (wout_side) {
    CU(cudaEventRecord(ctx->ev_f0, st));
    CU(cudaStreamWaitEvent(ctx->fst2, ctx->ev_f0, 0));
    float *keep_ws = b.ws;
    ctx->stream = ctx->fst2;
    b.ws = b.ws4;
    const cudaError_t we = wout_gemm();
    ctx->stream = st;
    b.ws = keep_ws;
    ctx->launches++;
    ctx->launches += tc_take_extra_launches();
    CU(we);
    CU(cudaEventRecord(ctx->ev_f2, ctx->fst2));
  }
  KL(launch_fpm_finalize(a, G, st));
  tl_mark(ctx, "f_fin", st);
  // W_retain_down[s][r][k] = sum_n up[n][s][r] g_pre[n][s][k]
  KL(gemm_any(ctx, tf32(gemm(R, d, N, h, b.fup, HR, R, true, b.fgpre, hd, d, false, G + L.w_retain_down, d,
                             (long)R * d))));
  // dup[n][s][r] = sum_k g_pre[n][s][k] W_retain_down[s][r][k]
  KL(gemm_any(ctx, gemm(N, R, d, h, b.fgpre, hd, d, false, W + L.w_retain_down, d, (long)R * d, true,
                   b.fdup, HR, R)));
  tl_mark(ctx, "f_dup", st);
  // W_retain_up[s][j][r] = sum_n c[n][s][j] dup[n][s][r]
  KL(gemm_any(ctx, tf32(gemm(d, R, N, h, b.fc, hd, d, true, b.fdup, HR, R, false, G + L.w_retain_up, R,
                             (long)d * R))));
  if (wout_side) CU(cudaStreamWaitEvent(st, ctx->ev_f2, 0));
  else KL(wout_gemm());
  return AIDEEN_OK;
}

void tl_mark(aideen_ctx *ctx, const char *name, cudaStream_t s) {
  static const bool on = getenv("AIDEEN_PIPE_TIMELINE") != nullptr;
  if (!on) return;
  cudaEvent_t e;
  cudaEventCreate(&e);
  cudaEventRecord(e, s);
  ctx->tl.push_back({name, e});
  ctx->tl_host.push_back(
      std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now().time_since_epoch()).count());
}

void tl_flush(aideen_ctx *ctx) {
  if (ctx->tl.empty()) return;
  cudaDeviceSynchronize();
  std::string line = "[timeline r" + std::to_string(ctx->rank) + "]";
  for (size_t i = 0; i < ctx->tl.size(); ++i) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->tl.front().second, ctx->tl[i].second);
    char buf[96];
    snprintf(buf, sizeof(buf), " %s=%.3f", ctx->tl[i].first.c_str(), ms);
    line += buf;
  }
  // the host clock at each mark (ms after the first): when the host enqueued it
  line += " | host:";
  for (size_t i = 0; i < ctx->tl_host.size(); ++i) {
    char buf[96];
    snprintf(buf, sizeof(buf), " %s=%.3f", ctx->tl[i].first.c_str(), (ctx->tl_host[i] - ctx->tl_host[0]) / 1e3);
    line += buf;
  }
  line += "\n";
  ctx->tl_host.clear();
  fputs(line.c_str(), stderr);  // one write per step, whole lines from every rank
  for (auto &m : ctx->tl) cudaEventDestroy(m.second);
  ctx->tl.clear();
}

// Token boundary of chunk j of nch: proportional to cumulative weights.  A
// small first chunk lets the consumers start early; the default weights are
// 1,2,3,... (three chunks 1,2,3 measured best of the tried splits at the bench
// shape; AIDEEN_PIPELINE_WEIGHTS overrides, comma-separated).
int chunk_bound(int j, int nch, int T) {
  int w[aideen_ctx::kMaxChunks] = {0};
  int tot = 0;
  static const char *const weights = getenv("AIDEEN_PIPELINE_WEIGHTS");
  const char *e = weights;
  for (int i = 0; i < nch; ++i) {
    int wi = i + 1;
    if (e && *e) {
      wi = atoi(e);
      while (*e && *e != ',') ++e;
      if (*e == ',') ++e;
    }
    w[i] = wi > 0 ? wi : 1;
    tot += w[i];
  }
  int acc = 0;
  for (int i = 0; i < j; ++i) acc += w[i];
  return (int)((long)acc * T / tot);
}

// chunk_bound rounded so every chunk's rows (tokens x B) fill whole 128-row
// GEMM tiles where B divides 128 (the first and last bounds stay 0 and T)
int chunk_bound_aligned(int j, int nch, int T, int B) {
  const int t = chunk_bound(j, nch, T);
  if (j == 0 || j == nch || B <= 0 || 128 % B != 0) return t;
  const int q = 128 / B;
  const int r = (t + q / 2) / q * q;
  return r > 0 && r < T ? r : t;
}

// Token chunks of the training step for the pipelined schedule (0: run the
// step sequentially).  Pipelining pays when the Picard solve leaves SMs idle.
int pipeline_chunks(aideen_ctx *ctx, const aideen_run *r) {
  if (ctx->prof || getenv("AIDEEN_NO_PIPELINE")) return 0;  // read per step (tests toggle it)
  int nsm = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int picard_ctas = (int)(r->batch * ctx->cfg.h_slots);
  if (nsm - picard_ctas < 32) return 0;
  if (r->batch % 4 != 0) return 0;  // chunk row offsets must keep 16-byte alignment of y^T columns
  int nch = 3;
  static const char *const chunks = getenv("AIDEEN_PIPELINE_CHUNKS");
  if (chunks) nch = atoi(chunks);
  if (nch > aideen_ctx::kMaxChunks) nch = aideen_ctx::kMaxChunks;
  if (nch < 2) return 0;
  for (int j = 0; j < nch; ++j)  // every chunk holds at least one token
    if (chunk_bound_aligned(j + 1, nch, r->seq_len, r->batch) <=
        chunk_bound_aligned(j, nch, r->seq_len, r->batch))
      return 0;
  return nch;
}

// Forward, LM head and adjoint of one training step with the Picard solve cut
// into token chunks on the high-priority stream: when chunk j's fixed points
// exist, pooling, the LM head (logits, softmax-CE, dy, dW_lm accumulated) and
// the adjoint of its rows run on the context stream, capped to the SMs the
// solve leaves free, while the solve continues with chunk j+1.  Results equal
// the sequential schedule's (each stage is row-local or a sum over rows).
int lm_sampled_prepare(aideen_ctx *ctx, int N, const aideen_step_args *a);
int lm_sampled_rows(aideen_ctx *ctx, long r0, int R, bool first);
int lm_sampled_finish(aideen_ctx *ctx, int N, const aideen_step_args *a);
int run_emb_update(aideen_ctx *ctx, int N, const aideen_step_args *a);
int emb_csr_early(aideen_ctx *ctx, int N);

int run_step_pipelined(aideen_ctx *ctx, const aideen_step_args *a, int nch, aideen_stats *stats) {
  const aideen_run *r = &a->run;
  // sampled head: per chunk only its logits / softmax / dW_S share; its Adam
  // step, dL/dh and the adjoint follow the last chunk (dL/dh needs the
  // updated rows, which need every row's coef)
  const bool sampled = a->lm_samples > 0;
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model, V = ctx->cfg.vocab;
  const int B = r->batch, T = r->seq_len, N = B * T;
  const long Vp = ctx->Vp, N4 = (N + 3) / 4 * 4;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const float *glm = b.lmp + ctx->lm_g, *Wlm = b.lmp;
  tl_mark(ctx, "start", st);
  // forward prep of the first chunk's rows; the rest is prepared while the
  // solve runs the first chunk
  ctx->perm_B = B;
  ctx->perm_T = T;
  const int R0 = chunk_bound_aligned(1, nch, T, B) * B;
  CHK(run_forward_prep_rows(ctx, r, 0, R0));
  tl_mark(ctx, "prep0", st);
  CU(cudaEventRecord(ctx->ev_prep, st));
  ctx->last_run = *r;
  ctx->N = N;
  int nsm = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int budget = nsm - B * h;
  // Picard chunks on the high-priority stream: chunk 0 after its rows' prep,
  // the others after the remaining rows' prep.  Chunk 0 is enqueued before
  // the host spends time on anything the solve does not wait for (when the
  // host has just synchronised, the GPU otherwise idles meanwhile).
  CU(cudaStreamWaitEvent(ctx->pic, ctx->ev_prep, 0));
  PicardArgs p = picard_args(ctx, r);
  p.t0 = 0;
  p.t1 = chunk_bound_aligned(1, nch, T, B);
  ctx->launches++;
  CU(launch_picard(p, r->fpm != 0, ctx->pic));
  CU(cudaEventRecord(ctx->ev_pic[0], ctx->pic));
  tl_mark(ctx, "pic0", ctx->pic);
  if (a->emb_update) CHK(emb_csr_early(ctx, N));
  // the gradient buffer is zeroed beside the solve instead of at the start of
  // the weight gradients (stream order: after the previous step's update)
  if (ctx->est && !ctx->prof) {
    CU(cudaEventRecord(ctx->ev_gz0, st));
    CU(cudaStreamWaitEvent(ctx->est, ctx->ev_gz0, 0));
    CU(cudaMemsetAsync(b.G, 0, ctx->W_len * sizeof(float), ctx->est));
    CU(cudaEventRecord(ctx->ev_gz, ctx->est));
    ctx->g_zeroed = true;
  }
  if (sampled) CHK(lm_sampled_prepare(ctx, N, a));
  else KL(launch_count_active(b.targets, N, b.scal, st));
  CU(cudaMemsetAsync(b.colpart, 0, (size_t)nsm * Vp * sizeof(float), st));
  // the last chunk's consumers run after the solve has finished: all SMs
  static const bool cap_last = getenv("AIDEEN_PIPELINE_CAP_LAST") != nullptr;
  CHK(run_forward_prep_rows(ctx, r, R0, N - R0));
  tl_mark(ctx, "prep", st);
  CU(cudaEventRecord(ctx->ev_prep, st));
  CU(cudaStreamWaitEvent(ctx->pic, ctx->ev_prep, 0));
  for (int j = 1; j < nch; ++j) {
    p.t0 = chunk_bound_aligned(j, nch, T, B);
    p.t1 = chunk_bound_aligned(j + 1, nch, T, B);
    ctx->launches++;
    CU(launch_picard(p, r->fpm != 0, ctx->pic));
    CU(cudaEventRecord(ctx->ev_pic[j], ctx->pic));
    tl_mark(ctx, ("pic" + std::to_string(j)).c_str(), ctx->pic);
  }
  // the FPM backward's forward-only stage once the solve is done, on its stream
  if (r->fpm && ctx->fst) {
    CU(cudaStreamWaitEvent(ctx->fst, ctx->ev_pic[nch - 1], 0));
    cudaStream_t keep_st = ctx->stream;
    float *keep_ws = ctx->b.ws;
    ctx->stream = ctx->fst;
    ctx->b.ws = ctx->b.ws2;
    const int rc = run_fpm_backward(ctx, true);
    ctx->stream = keep_st;
    ctx->b.ws = keep_ws;
    CHK(rc);
  }
  // per-chunk consumers on the context stream, within the SMs the solve leaves
  int colpart_rows = 0;
  int nsg_rows = 0;
  for (int j = 0; j < nch; ++j) {
    const int t0 = chunk_bound_aligned(j, nch, T, B), t1 = chunk_bound_aligned(j + 1, nch, T, B);
    const int bud = (j + 1 < nch || cap_last) ? budget : 0;
    ctx->sm_budget = bud;
    const long r0 = (long)t0 * B;
    const int R = (t1 - t0) * B;
    CU(cudaStreamWaitEvent(st, ctx->ev_pic[j], 0));
    if (sampled) {
      KL(launch_pool_rmsnorm(b.hstar + r0 * h * d, glm, b.pooled + r0 * d, b.y + r0 * d, b.lrms + r0, R, h, d,
                             st));
      CHK(lm_sampled_rows(ctx, r0, R, j == 0));
      tl_mark(ctx, ("cons" + std::to_string(j)).c_str(), st);
      continue;
    }
    if (j == 0) {  // the previous step's deferred LM-head update must be done before the logits
      CU(join_side(ctx));
      if (ctx->lm_split_stale) {
        KL(launch_split_hilo(Wlm, b.whi, b.wlo, (size_t)V * d, st));
        ctx->lm_split_stale = false;
      }
    }
    KL(launch_pool_rmsnorm(b.hstar + r0 * h * d, glm, b.pooled + r0 * d, b.y + r0 * d, b.lrms + r0, R, h, d, st));
    KL(launch_split_hilo(b.y + r0 * d, b.yhi + r0 * d, b.ylo + r0 * d, (size_t)R * d, st));
    KL(launch_transpose_split(b.y + r0 * d, R, d, d, b.yThi + r0, b.yTlo + r0, N4, st));
    // logits[n][v] = y[n] . W_lm[v]
    const long NT = (V + 255) / 256;
    KL(gemm_split(ctx, gemm(R, V, d, 1, b.yhi + r0 * d, d, 0, false, b.whi, d, 0, true, b.logits + r0 * Vp, Vp, 0),
                  b.ylo + r0 * d, b.wlo, b.lmp + ctx->lm_b, b.rowstats + r0 * NT));
    KL(launch_softmax_ce_split(b.logits + r0 * Vp, b.lmp + ctx->lm_b, b.targets + r0, b.scal, R, V, Vp,
                               b.loss_rows + r0, b.dlog_lo + r0 * Vp, b.colpart, st, bud, true,
                               b.rowstats + r0 * NT));
    const int blocks = softmax_rows_blocks(R, bud);
    colpart_rows = blocks > colpart_rows ? blocks : colpart_rows;
    // dy[n][j] = sum_v dlogits[n][v] W_lm[v][j]
    KL(gemm_split(ctx, gemm(R, d, V, 1, b.logits + r0 * Vp, Vp, 0, false, b.whi, d, 0, false, b.dy + r0 * d, d, 0),
                  b.dlog_lo + r0 * Vp, b.wlo));
    KL(launch_rmsnorm_bwd(b.dy + r0 * d, b.pooled + r0 * d, b.lrms + r0, glm, b.dl_dh + r0 * d,
                          b.ggp + r0 * d, R, d, st));
    // dW_lm[v][j] = sum_n dlogits[n][v] y^T[j][n], after the last chunk's
    // adjoint on its own stream (below)
    const bool tail_lm = j == nch - 1 && ctx->lmst && !ctx->prof;
    // dW_lm: the first `early` chunks' rows as each chunk's consumers finish
    // (they fill the consumers' slack while the solve runs), every later row in
    // one GEMM after the last adjoint, beside the weight gradients
    // (AIDEEN_DWLM_EARLY overrides the count; nch - 1 is fully per chunk)
    static const int early_env = getenv("AIDEEN_DWLM_EARLY") ? atoi(getenv("AIDEEN_DWLM_EARLY")) : 1;
    const int early = (ctx->lmst && !ctx->prof) ? (early_env < nch - 1 ? early_env : nch - 1) : nch;
    auto dwlm = [&]() {
      const long rr0 = tail_lm ? (long)chunk_bound_aligned(early, nch, T, B) * B : r0;
      const int RR = (int)((tail_lm ? N : r0 + R) - rr0);
      const bool first = rr0 == 0;
      return gemm_split(ctx, gemm(V, d, RR, 1, b.logits + rr0 * Vp, Vp, 0, true, b.yThi + rr0, N4, 0, true, b.Glm,
                                  d, 0, 1.f, first ? 0.f : 1.f),
                        b.dlog_lo + rr0 * Vp, b.yTlo + rr0);
    };
    if (!tail_lm && j < early) KL(dwlm());
    // adjoint of the chunk's rows
    AdjointArgs aa{};
    aa.N = R; aa.h = h; aa.d = d; aa.iters = a->adj_iters; aa.anderson_m = a->anderson_m;
    aa.beta = r->damping;
    aa.pre_a = b.pre + r0 * h * d; aa.pre_b = nullptr; aa.rhs_tok = b.dl_dh + r0 * d; aa.rhs_slot = nullptr;
    aa.NS = b.W + ctx->P.nscale; aa.v = b.v + r0 * d; aa.v_ld = N; aa.gpre = b.gpre + r0 * h * d;
    // per-CTA NormScale-gradient partials, the chunks' rows one after another
    // (a launch has at most as many CTAs as tokens, so N rows always suffice)
    aa.nsg_cta = b.nsg + (size_t)nsg_rows * d; aa.max_ctas = bud;
    if (a->anderson_m > 4) { ctx->sm_budget = 0; return set_err(ctx, AIDEEN_E_UNSUPPORTED, "anderson_m > 4"); }
    int grid = 0;
    KL(launch_adjoint(aa, st, &grid));
    nsg_rows += grid;
    tl_mark(ctx, ("cons" + std::to_string(j)).c_str(), st);
    // the FPM backward's chunk composites need only the forward and this
    // chunk's adjoint: form them on the FPM stream now (not for the last chunk,
    // whose composites start the backward proper)
    if (r->fpm && ctx->fst && ctx->fpm_prepared && j + 1 < nch && !ctx->prof) {
      FpmBwdArgs fa;
      CHK(fpm_args(ctx, fa));
      const int CH = fpm_chunk_len(d);
      if (t0 % CH == 0 && t1 % CH == 0 && t0 / CH == ctx->fpm_comp_done) {
        CU(cudaEventRecord(ctx->ev_adj, st));
        CU(cudaStreamWaitEvent(ctx->fst, ctx->ev_adj, 0));
        if (ctx->fpm_comp_done == 0) KL(launch_fpm_slot_params(fa, ctx->fst));
        fa.ch0 = t0 / CH;
        fa.ch1 = t1 / CH;
        KL(launch_fpm_composite(fa, ctx->fst));
        ctx->fpm_comp_done = t1 / CH;
      }
    }
    if (tail_lm) {
      CU(cudaEventRecord(ctx->ev_adj, st));
      CU(cudaStreamWaitEvent(ctx->lmst, ctx->ev_adj, 0));
      ctx->stream = ctx->lmst;
      // leave SMs to the FPM backward and attention-gradient chains that run
      // beside it (their kernels cannot share an SM with this GEMM's CTAs)
      // (48 SMs: best of the tried caps at the bench shape; AIDEEN_TAIL_LM_CAP overrides)
      ctx->sm_budget = getenv("AIDEEN_TAIL_LM_CAP") ? atoi(getenv("AIDEEN_TAIL_LM_CAP")) : nsm - 48;
      float *keep_ws = b.ws;
      b.ws = nullptr;  // no split-K here: the context stream's GEMMs own the workspace meanwhile
      const cudaError_t e = dwlm();
      b.ws = keep_ws;
      ctx->stream = st;
      KL(e);
    }
  }
  ctx->sm_budget = 0;
  if (sampled) {
    CHK(lm_sampled_finish(ctx, N, a));
    tl_mark(ctx, "lm_fin", st);
    // dL/dpooled is final here and nothing later in the step reads the
    // embedding: its row update runs on the embedding stream beside the
    // adjoint and the gradient chains (the same result as running it last).
    // With a communicator the gradient rows' all-gather is issued here on the
    // context stream, in the same place of every rank's collective sequence.
    if (a->emb_update == 1 && ctx->emb_csr_ready) {
      CHK(run_emb_update(ctx, N, a));
      ctx->emb_done = true;
    }
    AdjointArgs aa{};
    aa.N = N; aa.h = h; aa.d = d; aa.iters = a->adj_iters; aa.anderson_m = a->anderson_m;
    aa.beta = r->damping;
    aa.pre_a = b.pre; aa.rhs_tok = b.dl_dh;
    aa.NS = b.W + ctx->P.nscale; aa.v = b.v; aa.gpre = b.gpre; aa.nsg_cta = b.nsg;
    if (a->anderson_m > 4) return set_err(ctx, AIDEEN_E_UNSUPPORTED, "anderson_m > 4");
    int grid = 0;
    KL(launch_adjoint(aa, st, &grid));
    tl_mark(ctx, "adjoint", st);
    ctx->adj_N = N;
    ctx->adj_beta = r->damping;
    ctx->nsg_rows = grid;
    return stats ? read_solve_stats(ctx, r, stats) : AIDEEN_OK;
  }
  ctx->adj_N = N;
  ctx->adj_beta = r->damping;
  ctx->nsg_rows = nsg_rows;
  KL(launch_sum(b.loss_rows, N, b.scal + 1, st));
  const bool tail_lm = ctx->lmst && !ctx->prof;
  cudaStream_t lst = tail_lm ? ctx->lmst : st;
  KL(launch_colsum(b.colpart, colpart_rows, V, Vp, b.Glm + ctx->lm_b, V, 0, false, lst));
  KL(launch_colsum(b.ggp, N, d, d, b.Glm + ctx->lm_g, d, 0, false, lst));
  if (tail_lm) {
    // data parallel: the LM-head gradients are final here, so their sum over
    // ranks runs on the same stream, beside the weight gradients (every rank
    // issues it before the core-gradient allreduce, so the order matches)
    if (a->update.allreduce && ctx->comm && ctx->nranks > 1 && ctx->lm_ready) {
      const ncclResult_t nr =
          ncclAllReduce(b.Glm, b.Glm, ctx->lm_len, ncclFloat, ncclSum, ctx->comm, ctx->lmst);
      if (nr != ncclSuccess) return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllReduce: ") + ncclGetErrorString(nr));
      ctx->lm_reduced = true;
    }
    CU(cudaEventRecord(ctx->ev_lmg, ctx->lmst));
    ctx->lmg_pending = true;
  }
  return stats ? read_solve_stats(ctx, r, stats) : AIDEEN_OK;
}

// Sampled-softmax LM head over the last forward's pooled rows (the
// reference's lm_probs -> lm_update -> lm_backprop_h_t order): its Adam step
// on the sampled rows happens here, before dL/dh is formed from them.  With a
// communicator the sampled set is built from every rank's targets and the
// sampled-row gradients are summed over ranks before the clamp and the step,
// so every rank applies the same update.
// Sampled head, stage 1: the sampled set (from every rank's targets with a
// communicator) and the gathered rows W_S.  Depends only on the targets and
// W_lm, so it can run before the forward's rows exist.
int lm_sampled_prepare(aideen_ctx *ctx, int N, const aideen_step_args *a) {
  if (!ctx->lm_ready) return set_err(ctx, AIDEEN_E_INVALID, "LM head not uploaded");
  ctx->prof_phase = AIDEEN_PROF_LM_SOFTMAX;  // every LM-head launch in one profile class
  struct PhaseReset { aideen_ctx *c; ~PhaseReset() { c->prof_phase = -1; } } phase_reset{ctx};
  const int d = ctx->cfg.d_model, V = ctx->cfg.vocab;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const bool dp = ctx->comm && ctx->nranks > 1;
  const int Ng = dp ? N * ctx->nranks : N;
  const int ns = (int)a->lm_samples;
  // K <= max(min(max(ns, Ng), V, 2048), distinct targets) <= min(V, max(ns, Ng))
  size_t cap = (size_t)(ns > Ng ? ns : Ng);
  if (cap > (size_t)V) cap = V;
  cap = (cap + 3) / 4 * 4;
  if (cap > (size_t)ctx->Vp) return set_err(ctx, AIDEEN_E_INVALID, "sampled set larger than the logits rows");
  if (cap > ctx->lcap) {
    if (b.lS) { cudaFree(b.lS); cudaFree(b.lWS); b.lS = nullptr; b.lWS = nullptr; }
    CU(dalloc(&b.lS, cap));
    CU(dalloc(&b.lWS, cap * d));
    ctx->lcap = cap;
  }
  ctx->lcur = cap;
  if (!b.ints) {
    CU(dalloc(&b.ints, 8));
    CU(dalloc(&b.lerr, 1));
    CU(cudaMemsetAsync(b.lerr, 0, sizeof(unsigned int), st));
  }
  const int32_t *tg = b.targets;
  if (dp) {
    if ((size_t)Ng > ctx->gcap) {
      if (b.tg_all) { cudaFree(b.tg_all); cudaFree(b.tok_all); b.tg_all = b.tok_all = nullptr; }
      CU(dalloc(&b.tg_all, (size_t)Ng));
      CU(dalloc(&b.tok_all, (size_t)Ng));
      ctx->gcap = Ng;
    }
    const ncclResult_t nr = ncclAllGather(b.targets, b.tg_all, N, ncclInt32, ctx->comm, st);
    if (nr != ncclSuccess) return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
    tg = b.tg_all;
  }
  CU(join_side(ctx));
  const unsigned long long seed = a->sample_seed ? (unsigned long long)a->sample_seed : 0xA1DEEE5A4D5EED5Eull;
  KL(launch_sample_set(tg, Ng, V, ns, 2048, seed, a->update.step, b.lS, b.ints, b.scal, (int)cap, b.lerr, st));
  KL(launch_gather_rows(b.lmp, b.lS, b.ints, (int)cap, d, b.lWS, st));
  if (!ctx->hK) {
    CU(cudaMallocHost((void **)&ctx->hK, sizeof(int)));
    CU(cudaEventCreateWithFlags(&ctx->ev_K, cudaEventDisableTiming));
  }
  // the set holds max(desired, distinct targets) ids with desired =
  // min(max(ns, Ng), V, 2048): when desired already reaches the bound, that is
  // the size; otherwise the host reads it back to trim the GEMM width
  const int desired = std::min(std::min(ns > Ng ? ns : Ng, V), 2048);
  if ((size_t)(desired + 3) / 4 * 4 < cap) {
    CU(cudaMemcpyAsync(ctx->hK, b.ints, sizeof(int), cudaMemcpyDeviceToHost, st));
    CU(cudaEventRecord(ctx->ev_K, st));
    ctx->lk_pending = true;
  }
  return AIDEEN_OK;
}

// The sampled set's size as the GEMMs' width: the host waits for the set
// (built before the forward's rows exist; the caller has enqueued the solve
// by now, so the device keeps working) and trims the bound to it.
int lm_sampled_width(aideen_ctx *ctx) {
  if (!ctx->lk_pending) return AIDEEN_OK;
  ctx->lk_pending = false;
  CU(cudaEventSynchronize(ctx->ev_K));
  const size_t k = ((size_t)(*ctx->hK > 0 ? *ctx->hK : 1) + 3) / 4 * 4;
  if (k < ctx->lcur) ctx->lcur = k;
  return AIDEEN_OK;
}

// Stage 2, for token rows [r0, r0 + R) whose pooled state exists: sampled
// logits, softmax and coef in place, loss rows, and their share of dW_S and
// db_S (accumulated after the first row range).
int lm_sampled_rows(aideen_ctx *ctx, long r0, int R, bool first) {
  CHK(lm_sampled_width(ctx));
  ctx->prof_phase = AIDEEN_PROF_LM_SOFTMAX;
  struct PhaseReset { aideen_ctx *c; ~PhaseReset() { c->prof_phase = -1; } } phase_reset{ctx};
  const int d = ctx->cfg.d_model, V = ctx->cfg.vocab;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const int cap = (int)ctx->lcur;
  const long ld = cap;
  float *lg = b.logits + r0 * ld;
  const float *y = b.y + r0 * d;
  // logits[n][k] = y[n] . W_lm[S_k]
  KL(gemm_any(ctx, gemm(R, cap, d, 1, y, d, 0, false, b.lWS, d, 0, true, lg, ld, 0)));
  KL(launch_softmax_sampled(lg, ld, b.lmp + ctx->lm_b, b.lS, b.ints, b.targets + r0, V, b.scal,
                            b.loss_rows + r0, R, st));
  // dW_S[k][j] += sum_n coef[n][k] y[n][j]; db_S[k] += sum_n coef[n][k]
  KL(gemm_any(ctx, tf32(gemm(cap, d, R, 1, lg, ld, 0, true, y, d, 0, false, b.Glm, d, 0, 1.f, first ? 0.f : 1.f))));
  KL(launch_colsum(lg, R, cap, ld, b.Glm + ctx->lm_b, cap, 0, !first, st));
  return AIDEEN_OK;
}

// Stage 3, once every row's coef exists: (sum over ranks,) the clamped Adam
// step on the sampled rows, then dL/dy from the updated rows and the RMSNorm
// backward into dl_dh, and the loss.
int lm_sampled_finish(aideen_ctx *ctx, int N, const aideen_step_args *a) {
  ctx->prof_phase = AIDEEN_PROF_LM_SOFTMAX;
  struct PhaseReset { aideen_ctx *c; ~PhaseReset() { c->prof_phase = -1; } } phase_reset{ctx};
  const int d = ctx->cfg.d_model;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const int cap = (int)ctx->lcur;
  const long ld = cap;
  float *dW = b.Glm, *db = b.Glm + ctx->lm_b;
  KL(launch_sum(b.loss_rows, N, b.scal + 1, st));
  if (ctx->comm && ctx->nranks > 1) {
    // the sampled rows' gradients are the only LM-head gradients of the step:
    // the core-gradient sum must not sum the LM-head block again
    ctx->lm_reduced = true;
    ncclResult_t nr = ncclGroupStart();
    if (nr == ncclSuccess) nr = ncclAllReduce(dW, dW, (size_t)cap * d, ncclFloat, ncclSum, ctx->comm, st);
    if (nr == ncclSuccess) nr = ncclAllReduce(db, db, cap, ncclFloat, ncclSum, ctx->comm, st);
    const ncclResult_t n2 = ncclGroupEnd();
    if (nr != ncclSuccess || n2 != ncclSuccess)
      return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllReduce: ") +
                                             ncclGetErrorString(nr != ncclSuccess ? nr : n2));
  }
  const aideen_update *u = &a->update;
  const double t = u->step < 1 ? 1.0 : (double)u->step;
  const float bc1 = (float)(1.0 - std::pow((double)u->beta1, t));
  const float bc2 = (float)(1.0 - std::pow((double)u->beta2, t));
  KL(launch_lm_sampled_adam(b.lmp, b.lmp + ctx->lm_b, b.Mlm1, b.Mlm2, ctx->lm_b, dW, db, b.lS, b.ints, cap, d,
                            b.lWS, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2, st));
  ctx->lm_split_stale = true;
  // dL/dy[n][j] = sum_k coef[n][k] W_lm'[S_k][j], then through the RMSNorm
  KL(gemm_any(ctx, gemm(N, d, cap, 1, b.logits, ld, 0, false, b.lWS, d, 0, false, b.dy, d, 0)));
  KL(launch_rmsnorm_bwd(b.dy, b.pooled, b.lrms, b.lmp + ctx->lm_g, b.dl_dh, b.ggp, N, d, st));
  return AIDEEN_OK;
}

// Sampled-softmax LM head over the last forward's pooled rows (the
// reference's lm_probs -> lm_update -> lm_backprop_h_t order): its Adam step
// on the sampled rows happens here, before dL/dh is formed from them.  With a
// communicator the sampled set is built from every rank's targets and the
// sampled-row gradients are summed over ranks before the clamp and the step,
// so every rank applies the same update.
int run_lm_head_sampled(aideen_ctx *ctx, int N, const aideen_step_args *a) {
  CHK(lm_sampled_prepare(ctx, N, a));
  CHK(lm_sampled_rows(ctx, 0, N, true));
  return lm_sampled_finish(ctx, N, a);
}

// Embedding rows of the step's tokens: the mean gradient row of every
// distinct token (dL/dpooled, or dL/dS_in with source 2), then Adam on that
// row.  With a communicator every rank gathers all ranks' tokens and rows, so
// every rank applies the same update.
int run_emb_update(aideen_ctx *ctx, int N, const aideen_step_args *a) {
  const int d = ctx->cfg.d_model, V = ctx->cfg.vocab;
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  const bool dp = ctx->comm && ctx->nranks > 1;
  const int Ng = dp ? N * ctx->nranks : N;
  if (Ng > emb_csr_max_tokens())
    return set_err(ctx, AIDEEN_E_UNSUPPORTED, "embedding update: more tokens per step than the CSR sort holds");
  if (!b.Me1) {
    CU(dalloc(&b.Me1, (size_t)V * d));
    CU(dalloc(&b.Me2, (size_t)V * d));
    CU(cudaMemsetAsync(b.Me1, 0, (size_t)V * d * 4, st));
    CU(cudaMemsetAsync(b.Me2, 0, (size_t)V * d * 4, st));
  }
  if (!b.cuniq || (size_t)Ng > ctx->gcap) {
    if (b.cuniq) { cudaFree(b.cuniq); cudaFree(b.coff); cudaFree(b.cpos); }
    if (b.tg_all) { cudaFree(b.tg_all); cudaFree(b.tok_all); b.tg_all = b.tok_all = nullptr; }
    if (b.grad_all) { cudaFree(b.grad_all); b.grad_all = nullptr; }
    const size_t n = (size_t)Ng > ctx->gcap ? (size_t)Ng : ctx->gcap;
    CU(dalloc(&b.cuniq, n)); CU(dalloc(&b.coff, n + 1)); CU(dalloc(&b.cpos, n));
    CU(dalloc(&b.tg_all, n)); CU(dalloc(&b.tok_all, n));
    ctx->gcap = n;
  }
  if (!b.ints) {
    CU(dalloc(&b.ints, 8));
    CU(dalloc(&b.lerr, 1));
    CU(cudaMemsetAsync(b.lerr, 0, sizeof(unsigned int), st));
  }
  const float *grad = a->emb_update == 2 ? b.dS : b.dl_dh;
  const int32_t *tok = b.tokens;
  if (dp) {
    if (!b.grad_all) CU(dalloc(&b.grad_all, ctx->gcap * d));
    ncclResult_t nr = ncclGroupStart();
    // (with the CSR built early, every rank's tokens were gathered then)
    if (nr == ncclSuccess && !ctx->emb_csr_ready)
      nr = ncclAllGather(b.tokens, b.tok_all, N, ncclInt32, ctx->comm, st);
    if (nr == ncclSuccess) nr = ncclAllGather(grad, b.grad_all, (size_t)N * d, ncclFloat, ctx->comm, st);
    const ncclResult_t n2 = ncclGroupEnd();
    if (nr != ncclSuccess || n2 != ncclSuccess)
      return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllGather: ") +
                                             ncclGetErrorString(nr != ncclSuccess ? nr : n2));
    tok = b.tok_all;
    grad = b.grad_all;
    tl_mark(ctx, "emb_ag", st);
  }
  const aideen_update *u = &a->update;
  const double t = u->step < 1 ? 1.0 : (double)u->step;
  const float bc1 = (float)(1.0 - std::pow((double)u->beta1, t));
  const float bc2 = (float)(1.0 - std::pow((double)u->beta2, t));
  const float lr = a->emb_lr > 0.f ? a->emb_lr : u->lr;
  if (ctx->emb_csr_ready) {
    // the CSR was built on the embedding stream at the step's start; the row
    // update follows the gradient rows there and the next gather joins it
    ctx->emb_csr_ready = false;
    CU(cudaEventRecord(ctx->ev_e0, st));
    CU(cudaStreamWaitEvent(ctx->est, ctx->ev_e0, 0));
    ctx->launches++;
    CU(launch_emb_adam(b.emb, b.Me1, b.Me2, grad, b.cuniq, b.coff, b.cpos, b.ints + 1, Ng, d, lr, u->beta1,
                       u->beta2, u->eps, bc1, bc2, ctx->est));
    CU(cudaEventRecord(ctx->ev_emb, ctx->est));
    ctx->emb_pending = true;
    return AIDEEN_OK;
  }
  KL(launch_emb_csr(tok, Ng, V, b.cuniq, b.coff, b.cpos, b.ints + 1, st));
  KL(launch_emb_adam(b.emb, b.Me1, b.Me2, grad, b.cuniq, b.coff, b.cpos, b.ints + 1, Ng, d, lr, u->beta1,
                     u->beta2, u->eps, bc1, bc2, st));
  return AIDEEN_OK;
}

// No profiling: the step's token CSR on the embedding stream while the forward
// runs (it needs only the token ids; with a communicator, every rank's ids,
// gathered here on the context stream).
int emb_csr_early(aideen_ctx *ctx, int N) {
  DevBufs &b = ctx->b;
  const bool dp = ctx->comm && ctx->nranks > 1;
  const int Ng = dp ? N * ctx->nranks : N;
  if (ctx->prof || !ctx->est || !b.cuniq || (size_t)Ng > ctx->gcap || Ng > emb_csr_max_tokens())
    return AIDEEN_OK;  // the update builds it itself (first step, profiling)
  const int32_t *tok = b.tokens;
  if (dp) {
    const ncclResult_t nr = ncclAllGather(b.tokens, b.tok_all, N, ncclInt32, ctx->comm, ctx->stream);
    if (nr != ncclSuccess) return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllGather: ") + ncclGetErrorString(nr));
    tok = b.tok_all;
  }
  CU(cudaEventRecord(ctx->ev_e0, ctx->stream));
  CU(cudaStreamWaitEvent(ctx->est, ctx->ev_e0, 0));
  ctx->launches++;
  CU(launch_emb_csr(tok, Ng, (int)ctx->cfg.vocab, b.cuniq, b.coff, b.cpos, b.ints + 1, ctx->est));
  ctx->emb_csr_ready = true;
  return AIDEEN_OK;
}

int run_allreduce(aideen_ctx *ctx, int timeout_ms) {
  if (!ctx->comm || ctx->nranks <= 1) return AIDEEN_OK;
  ncclResult_t r = ncclGroupStart();
  if (r == ncclSuccess)
    r = ncclAllReduce(ctx->b.G, ctx->b.G, ctx->W_len, ncclFloat, ncclSum, ctx->comm, ctx->stream);
  if (r == ncclSuccess && ctx->lm_ready && !ctx->lm_reduced)
    r = ncclAllReduce(ctx->b.Glm, ctx->b.Glm, ctx->lm_len, ncclFloat, ncclSum, ctx->comm, ctx->stream);
  ctx->lm_reduced = false;
  ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess)
    return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllReduce: ") +
                                           ncclGetErrorString(r != ncclSuccess ? r : r2));
  if (timeout_ms <= 0) return AIDEEN_OK;  // stream-ordered, no host wait
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) return AIDEEN_OK;
    if (q != cudaErrorNotReady) CU(q);
    ncclResult_t ae = ncclSuccess;
    ncclCommGetAsyncError(ctx->comm, &ae);
    if (ae != ncclSuccess && ae != ncclInProgress) {
      ncclCommAbort(ctx->comm);
      ctx->comm = nullptr;
      return set_err(ctx, AIDEEN_E_NCCL, std::string("async NCCL error: ") + ncclGetErrorString(ae));
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      ncclCommAbort(ctx->comm);
      ctx->comm = nullptr;
      return set_err(ctx, AIDEEN_E_TIMEOUT, "gradient allreduce did not finish in time; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// LM-head update and the refresh of its pre-split copies.  Without profiling
// it runs on the side stream, ordered after the gradients (and their
// allreduce) on the context stream; the next LM-head call joins it.
int run_lm_update(aideen_ctx *ctx, const aideen_update *u, float bc1, float bc2) {
  DevBufs &b = ctx->b;
  const bool deferred = !ctx->prof;
  cudaStream_t ls = deferred ? ctx->side : ctx->stream;
  CU(join_side(ctx));
  if (deferred) {
    CU(cudaEventRecord(ctx->ev_grads, ctx->stream));
    CU(cudaStreamWaitEvent(ctx->side, ctx->ev_grads, 0));
  }
  if (u->rule == AIDEEN_RULE_ADAM)
    KL(launch_adam(b.lmp, b.Glm, b.Mlm1, b.Mlm2, ctx->lm_len, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2,
                   u->grad_scale, ls));
  else
    KL(launch_clipped_sgd(b.lmp, b.Glm, ctx->lm_len, ctx->lm_len, u->lr, u->weight_decay, u->grad_scale, ls));
  KL(launch_split_hilo(b.lmp, b.whi, b.wlo, (size_t)ctx->cfg.vocab * ctx->cfg.d_model, ls));
  ctx->lm_split_stale = false;
  if (deferred) {
    CU(cudaEventRecord(ctx->ev_lm_done, ctx->side));
    ctx->lm_pending = true;
  }
  return AIDEEN_OK;
}

// Adam on this rank's shard of both reduce-scattered buckets (and on the
// small remainders every rank holds summed), then the weights all-gathered.
int run_update_sharded(aideen_ctx *ctx, const aideen_update *u, float bc1, float bc2) {
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  size_t boff[2], blen[2];
  grad_buckets(ctx, boff, blen);
  const size_t n = (size_t)ctx->nranks;
  for (int k = 0; k < 2; ++k) {
    const size_t cnt = blen[k] / n, rem = blen[k] - cnt * n;
    const size_t o = boff[k] + (size_t)ctx->rank * cnt, orr = boff[k] + cnt * n;
    if (cnt) KL(launch_adam(b.W + o, b.G + o, b.M1 + o, b.M2 + o, cnt, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2,
                            u->grad_scale, st));
    if (rem) KL(launch_adam(b.W + orr, b.G + orr, b.M1 + orr, b.M2 + orr, rem, u->lr, u->beta1, u->beta2, u->eps,
                            bc1, bc2, u->grad_scale, st));
  }
  tl_mark(ctx, "adam_sh", st);
  ncclResult_t r = ncclGroupStart();
  for (int k = 0; k < 2 && r == ncclSuccess; ++k) {
    const size_t cnt = blen[k] / n;
    if (cnt)
      r = ncclAllGather(b.W + boff[k] + (size_t)ctx->rank * cnt, b.W + boff[k], cnt, ncclFloat, ctx->comm, st);
  }
  const ncclResult_t r2 = ncclGroupEnd();
  if (r != ncclSuccess || r2 != ncclSuccess)
    return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllGather: ") +
                                           ncclGetErrorString(r != ncclSuccess ? r : r2));
  return AIDEEN_OK;
}

int run_update(aideen_ctx *ctx, const aideen_update *u) {
  if (!u) return set_err(ctx, AIDEEN_E_INVALID, "null update");
  if (ctx->shard_step) {
    // the core gradients were reduce-scattered during the weight gradients;
    // the LM head's sum is still owed in dense mode
    ctx->shard_step = false;
    if (ctx->lm_ready && !ctx->lm_reduced && u->update_lm_head) {
      const ncclResult_t nr = ncclAllReduce(ctx->b.Glm, ctx->b.Glm, ctx->lm_len, ncclFloat, ncclSum, ctx->comm,
                                            ctx->stream);
      if (nr != ncclSuccess) return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclAllReduce: ") + ncclGetErrorString(nr));
    }
    ctx->lm_reduced = false;
    const double t = u->step < 1 ? 1.0 : (double)u->step;
    const float bc1 = (float)(1.0 - std::pow((double)u->beta1, t));
    const float bc2 = (float)(1.0 - std::pow((double)u->beta2, t));
    CHK(run_update_sharded(ctx, u, bc1, bc2));
    if (u->update_lm_head && ctx->lm_ready) CHK(run_lm_update(ctx, u, bc1, bc2));
    return AIDEEN_OK;
  }
  if (u->allreduce) CHK(run_allreduce(ctx, 0));
  DevBufs &b = ctx->b;
  cudaStream_t st = ctx->stream;
  if (u->rule == AIDEEN_RULE_ADAM) {
    const double t = u->step < 1 ? 1.0 : (double)u->step;
    const float bc1 = (float)(1.0 - std::pow((double)u->beta1, t));
    const float bc2 = (float)(1.0 - std::pow((double)u->beta2, t));
    if (ctx->adam_dead_zero && !getenv("AIDEEN_ADAM_FULL")) {
      // only the entries a gradient can reach: ~1/2.7 of the parameters
      const Layout &L = ctx->P;
      const size_t d = ctx->cfg.d_model, h = ctx->cfg.h_slots;
      AdamSegs sg{};
      auto add = [&](size_t off, size_t rows, size_t row_len, size_t stride) {
        sg.off[sg.n] = off;
        sg.rows[sg.n] = (int)rows;
        sg.row4[sg.n] = (int)(row_len / 4);
        sg.stride[sg.n] = (long)stride;
        sg.start4[sg.n + 1] = sg.start4[sg.n] + rows * (row_len / 4);
        ++sg.n;
      };
      const size_t tail = ctx->W_len - L.win, tail4 = tail / 4 * 4;
      add(L.wq, h * d, kHeadDim, d);                  // W_q: columns 0..31 of every row
      add(L.q_bias, 1, L.wk - L.q_bias, 0);           // q bias (and alignment padding)
      add(L.wk, h * d, kHeadDim, d);
      add(L.k_bias, 1, L.wv - L.k_bias, 0);
      add(L.wv, h * d, kHeadDim, d);
      add(L.wo, h, (size_t)kHeadDim * d, d * d);      // W_o: rows 0..31 of every slot
      add(L.win, 1, tail4, 0);                        // W_in and every later tensor
      KL(launch_adam_segs(b.W, b.G, b.M1, b.M2, sg, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2, u->grad_scale,
                          st));
      if (tail4 < tail)
        KL(launch_adam(b.W + L.win + tail4, b.G + L.win + tail4, b.M1 + L.win + tail4, b.M2 + L.win + tail4,
                       tail - tail4, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2, u->grad_scale, st));
    } else {
      KL(launch_adam(b.W, b.G, b.M1, b.M2, ctx->W_len, u->lr, u->beta1, u->beta2, u->eps, bc1, bc2,
                     u->grad_scale, st));
    }
    if (u->update_lm_head && ctx->lm_ready) CHK(run_lm_update(ctx, u, bc1, bc2));
  } else if (u->rule == AIDEEN_RULE_CLIPPED_SGD) {
    KL(launch_clipped_sgd(b.W, b.G, ctx->W_len, ctx->P.hist, u->lr, u->weight_decay, u->grad_scale, st));
    if (u->update_lm_head && ctx->lm_ready) CHK(run_lm_update(ctx, u, 0.f, 0.f));
  } else {
    return set_err(ctx, AIDEEN_E_INVALID, "unknown update rule");
  }
  return AIDEEN_OK;
}

}  // namespace

extern "C" {

size_t aideen_all_weights_len(uint32_t d, uint32_t h) { return Layout(d, h, 1).total; }

const char *aideen_last_error(const aideen_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t aideen_launch_count(const aideen_ctx *ctx) { return ctx ? ctx->launches : 0; }

aideen_ctx *aideen_create(const aideen_cfg *cfg, int device, int *status) {
  auto fail = [&](int code) -> aideen_ctx * {
    if (status) *status = code;
    return nullptr;
  };
  if (!cfg) return fail(AIDEEN_E_INVALID);
  const uint32_t d = cfg->d_model, h = cfg->h_slots;
  if (!(d == 128 || d == 256 || d == 512 || d == 1024) || h < 1 || h > 16 || cfg->max_batch == 0 ||
      cfg->max_seq_len == 0 || (cfg->flags & ~(uint32_t)AIDEEN_CFG_ASSOC) != 0 ||
      ((cfg->flags & AIDEEN_CFG_ASSOC) && h < 2))
    return fail(AIDEEN_E_INVALID);
  if (cudaSetDevice(device) != cudaSuccess) return fail(AIDEEN_E_CUDA);
  aideen_ctx *ctx = new aideen_ctx();
  ctx->cfg = *cfg;
  ctx->device = device;
  if (const char *gm = getenv("AIDEEN_GEMM")) ctx->use_tc = strcmp(gm, "simt") != 0;
  ctx->P = Layout(d, h, 64);
  ctx->Lx = Layout(d, h, 1);
  ctx->W_len = ctx->P.total;
  const size_t N = (size_t)cfg->max_batch * cfg->max_seq_len;
  ctx->max_tokens = N;
  const size_t V = cfg->vocab;
  ctx->Vp = (long)((V + 3) / 4 * 4);
  ctx->lm_b = V * d;
  ctx->lm_g = V * d + (V + 63) / 64 * 64;
  ctx->lm_len = V ? ctx->lm_g + d : 0;
  DevBufs &b = ctx->b;
  const size_t Nhd = N * h * d, NH32 = N * h * kHeadDim;
  cudaError_t e = cudaSuccess;
  auto A = [&](auto **p, size_t n) { if (e == cudaSuccess) e = dalloc(p, n); };
  A(&b.W, ctx->W_len); A(&b.G, ctx->W_len); A(&b.M1, ctx->W_len); A(&b.M2, ctx->W_len);
  A(&b.S_in, N * d); A(&b.tokens, N); A(&b.targets, N);
  A(&b.signal, Nhd); A(&b.A, Nhd); A(&b.amat, Nhd); A(&b.src, Nhd);
  A(&b.qkv, 3 * NH32); A(&b.dqkv, 3 * NH32); A(&b.Wcat, (size_t)h * d * 96);
  A(&b.nmix, NH32); A(&b.dn, NH32);
  b.Qh = b.qkv; b.Kh = b.qkv + 32; b.Vh = b.qkv + 64;
  b.dQ = b.dqkv; b.dK = b.dqkv + 32; b.dV = b.dqkv + 64;
  A(&b.alpha, N * h * h); A(&b.rmix, N * h); A(&b.scale, N * h); A(&b.rho, N * h);
  A(&b.Rsrc, N * h); A(&b.dRc, N * h); A(&b.iters, N * h);
  A(&b.hstar, Nhd); A(&b.pre, Nhd); A(&b.hist, Nhd); A(&b.fpmctx, Nhd);
  A(&b.v, Nhd); A(&b.gpre, Nhd); A(&b.dsig, Nhd); A(&b.da, Nhd);
  A(&b.mstate, (size_t)cfg->max_batch * h * d); A(&b.fcarry, (size_t)cfg->max_batch * h * d);
  ctx->assoc = (cfg->flags & AIDEEN_CFG_ASSOC) != 0;
  if (ctx->assoc) {
    A(&b.assoc_v, (size_t)cfg->max_batch * h * d); A(&b.assoc_p, (size_t)cfg->max_batch * h * d);
    A(&b.assoc_u, (size_t)cfg->max_batch * h); A(&b.sig_store, Nhd); A(&b.assoc_read, Nhd);
    if (e == cudaSuccess) e = cudaMemset(b.assoc_v, 0, (size_t)cfg->max_batch * h * d * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(b.assoc_p, 0, (size_t)cfg->max_batch * h * d * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(b.assoc_u, 0, (size_t)cfg->max_batch * h * sizeof(float));
  }
  A(&b.pooled, N * d); A(&b.dl_dh, N * d); A(&b.nsg, N * d); A(&b.dS, N * d);
  A(&b.y, N * d); A(&b.dy, N * d); A(&b.yhi, N * d); A(&b.ylo, N * d);
  A(&b.yThi, d * ((N + 3) / 4 * 4)); A(&b.yTlo, d * ((N + 3) / 4 * 4)); A(&b.ggp, N * d); A(&b.lrms, N); A(&b.loss_rows, N);
  A(&b.scal, 4); A(&b.stage, ctx->Lx.total);
  ctx->ws_floats = 16 * N * d;  // up to 16 splits of an [N][d] output
  A(&b.ws, ctx->ws_floats); A(&b.ws2, ctx->ws_floats); A(&b.ws3, ctx->ws_floats); A(&b.ws4, ctx->ws_floats); A(&b.stats, 4); A(&b.sigmas, 5 * h + 2);
  if (V) {
    A(&b.lmp, ctx->lm_len); A(&b.Glm, ctx->lm_len); A(&b.Mlm1, ctx->lm_len); A(&b.Mlm2, ctx->lm_len);
    A(&b.logits, N * (size_t)ctx->Vp); A(&b.emb, V * d);
    A(&b.dlog_lo, N * (size_t)ctx->Vp); A(&b.whi, V * d); A(&b.wlo, V * d);
    int nsm_dev = 0;
    cudaDeviceGetAttribute(&nsm_dev, cudaDevAttrMultiProcessorCount, device);
    A(&b.colpart, (size_t)(nsm_dev > 0 ? nsm_dev : 148) * ctx->Vp);  // <= one row per SM
    A(&b.rowstats, N * ((V + 255) / 256));
  }
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  ctx->own_stream = true;
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_grads, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_lm_done, cudaEventDisableTiming);
  if (e == cudaSuccess) {
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    e = cudaStreamCreateWithPriority(&ctx->pic, cudaStreamNonBlocking, hi);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_prep, cudaEventDisableTiming);
  if (e == cudaSuccess) {
    // the FPM backward is the longest chain after the adjoint: its CTAs go
    // ahead of the attention-branch GEMMs that run beside it
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    e = cudaStreamCreateWithPriority(&ctx->fst, cudaStreamNonBlocking, hi);
    if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&ctx->fst2, cudaStreamNonBlocking, hi);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_f0, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_f2, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_g0, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_fdone, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->lmst, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->ast, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->est, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_e0, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_emb, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_da, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_dqkv, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_dsig, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMallocHost((void **)&ctx->hbox, 4 * sizeof(uint32_t));
  ctx->d_adj_err = adjoint_error_dev();
  ctx->d_pic_err = picard_error_dev();
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_gz0, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_gz, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_adone, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_adj, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_lmg, cudaEventDisableTiming);
  for (int i = 0; i < aideen_ctx::kMaxChunks && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&ctx->ev_pic[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    aideen_destroy(ctx);
    return fail(AIDEEN_E_CUDA);
  }
  cudaMemsetAsync(b.mstate, 0, (size_t)cfg->max_batch * h * d * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.fcarry, 0, (size_t)cfg->max_batch * h * d * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.W, 0, ctx->W_len * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.G, 0, ctx->W_len * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.M1, 0, ctx->W_len * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.M2, 0, ctx->W_len * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.hist, 0, Nhd * sizeof(float), ctx->stream);
  cudaMemsetAsync(b.fpmctx, 0, Nhd * sizeof(float), ctx->stream);
  if (V) {
    cudaMemsetAsync(b.Mlm1, 0, ctx->lm_len * sizeof(float), ctx->stream);
    cudaMemsetAsync(b.Mlm2, 0, ctx->lm_len * sizeof(float), ctx->stream);
  }
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    aideen_destroy(ctx);
    return fail(AIDEEN_E_CUDA);
  }
  if (status) *status = AIDEEN_OK;
  return ctx;
}

void aideen_destroy(aideen_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->est) cudaStreamSynchronize(ctx->est);
  if (ctx->comm) ncclCommDestroy(ctx->comm);
  DevBufs &b = ctx->b;
  void *ptrs[] = {b.W, b.G, b.M1, b.M2, b.S_in, b.tokens, b.targets, b.signal, b.A, b.amat, b.qkv,
                  b.assoc_v, b.assoc_p, b.assoc_u, b.sig_store, b.assoc_read,
                  b.dqkv, b.Wcat, b.alpha, b.nmix, b.rmix, b.scale, b.rho, b.Rsrc, b.hstar, b.pre,
                  b.pooled, b.hist, b.fpmctx, b.mstate, b.iters, b.v, b.gpre, b.dl_dh, b.rhs_slot,
                  b.nsg, b.da, b.dn, b.dsig, b.dRc, b.dS, b.lmp, b.Glm, b.Mlm1,
                  b.Mlm2, b.y, b.lrms, b.logits, b.dy, b.ggp, b.loss_rows, b.scal, b.emb, b.stats,
                  b.sigmas, b.stage, b.ws, b.fc, b.frp, b.fdl, b.fminner, b.fdm, b.fgpre, b.fup,
                  b.fkw, b.fdup, b.fA, b.fU, b.fgin, b.fcarry, b.fpart, b.fpart_bw, b.fprm, b.src,
                  b.dlog_lo, b.yhi, b.ylo, b.yThi, b.yTlo, b.whi, b.wlo, b.colpart, b.perm, b.ws2, b.ws3, b.ws4, b.rowstats,
                  b.lS, b.lWS, b.ints, b.lerr, b.tg_all, b.tok_all, b.grad_all, b.cuniq, b.coff, b.cpos,
                  b.Me1, b.Me2};
  for (void *p : ptrs)
    if (p) cudaFree(p);
  if (ctx->side) cudaStreamSynchronize(ctx->side);
  if (ctx->stream && ctx->own_stream) cudaStreamDestroy(ctx->stream);
  if (ctx->side) cudaStreamDestroy(ctx->side);
  if (ctx->pic) { cudaStreamSynchronize(ctx->pic); cudaStreamDestroy(ctx->pic); }
  if (ctx->ev_prep) cudaEventDestroy(ctx->ev_prep);
  if (ctx->fst) { cudaStreamSynchronize(ctx->fst); cudaStreamDestroy(ctx->fst); }
  if (ctx->fst2) { cudaStreamSynchronize(ctx->fst2); cudaStreamDestroy(ctx->fst2); }
  if (ctx->ev_f0) cudaEventDestroy(ctx->ev_f0);
  if (ctx->ev_f2) cudaEventDestroy(ctx->ev_f2);
  if (ctx->ev_g0) cudaEventDestroy(ctx->ev_g0);
  if (ctx->ev_fdone) cudaEventDestroy(ctx->ev_fdone);
  if (ctx->lmst) { cudaStreamSynchronize(ctx->lmst); cudaStreamDestroy(ctx->lmst); }
  if (ctx->ast) { cudaStreamSynchronize(ctx->ast); cudaStreamDestroy(ctx->ast); }
  if (ctx->est) cudaStreamDestroy(ctx->est);
  if (ctx->hK) cudaFreeHost(ctx->hK);
  if (ctx->hbox) cudaFreeHost(ctx->hbox);
  if (ctx->ev_K) cudaEventDestroy(ctx->ev_K);
  if (ctx->ev_e0) cudaEventDestroy(ctx->ev_e0);
  if (ctx->ev_gz0) cudaEventDestroy(ctx->ev_gz0);
  if (ctx->ev_gz) cudaEventDestroy(ctx->ev_gz);
  if (ctx->ev_emb) cudaEventDestroy(ctx->ev_emb);
  if (ctx->ev_da) cudaEventDestroy(ctx->ev_da);
  if (ctx->ev_dqkv) cudaEventDestroy(ctx->ev_dqkv);
  if (ctx->ev_dsig) cudaEventDestroy(ctx->ev_dsig);
  if (ctx->ev_adone) cudaEventDestroy(ctx->ev_adone);
  if (ctx->ev_adj) cudaEventDestroy(ctx->ev_adj);
  if (ctx->ev_lmg) cudaEventDestroy(ctx->ev_lmg);
  for (auto &ev : ctx->ev_pic)
    if (ev) cudaEventDestroy(ev);
  if (ctx->ev_grads) cudaEventDestroy(ctx->ev_grads);
  if (ctx->ev_lm_done) cudaEventDestroy(ctx->ev_lm_done);
  delete ctx;
}

int aideen_set_stream(aideen_ctx *ctx, void *s) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  CU(join_emb(ctx));
  CU(cudaStreamSynchronize(ctx->stream));
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  ctx->stream = (cudaStream_t)s;
  ctx->own_stream = false;
  return AIDEEN_OK;
}

int aideen_profile(aideen_ctx *ctx, int enable) {
  if (!ctx) return AIDEEN_E_INVALID;
  ctx->prof = enable != 0;
  return AIDEEN_OK;
}

int aideen_profile_read(aideen_ctx *ctx, float *ms, uint64_t *launches, int reset) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(cudaStreamSynchronize(ctx->stream));
  for (auto &pe : ctx->pev) {
    float t = 0.f;
    cudaEventElapsedTime(&t, pe.second.first, pe.second.second);
    ctx->prof_ms[pe.first] += t;
    ctx->prof_n[pe.first] += 1;
    cudaEventDestroy(pe.second.first);
    cudaEventDestroy(pe.second.second);
  }
  ctx->pev.clear();
  for (int i = 0; i < AIDEEN_PROF_CLASSES; ++i) {
    if (ms) ms[i] = (float)ctx->prof_ms[i];
    if (launches) launches[i] = ctx->prof_n[i];
    if (reset) { ctx->prof_ms[i] = 0; ctx->prof_n[i] = 0; }
  }
  return AIDEEN_OK;
}

int aideen_join(aideen_ctx *ctx) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  CU(join_emb(ctx));
  return AIDEEN_OK;
}

int aideen_sync(aideen_ctx *ctx) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  CU(join_emb(ctx));
  return sync_and_check(ctx);
}

// Packed reference layout <-> padded device layout, one copy per tensor.
static int repack(aideen_ctx *ctx, float *dst, const float *src, bool to_device, cudaMemcpyKind kind) {
  for (int k = 0; k < kSegments; ++k) {
    const size_t len = ctx->P.seg_len[k];
    const size_t dof = to_device ? ctx->P.seg_off[k] : ctx->Lx.seg_off[k];
    const size_t sof = to_device ? ctx->Lx.seg_off[k] : ctx->P.seg_off[k];
    CU(cudaMemcpyAsync(dst + dof, src + sof, len * sizeof(float), kind, ctx->stream));
  }
  return AIDEEN_OK;
}

int aideen_upload_weights(aideen_ctx *ctx, const float *w, size_t n, int where) {
  if (!ctx) return AIDEEN_E_INVALID;
  if (n != ctx->Lx.total) return set_err(ctx, AIDEEN_E_INVALID, "AllWeights length mismatch");
  if (!w) return set_err(ctx, AIDEEN_E_INVALID, "null weights");
  if (where == AIDEEN_DEVICE) {
    CHK(repack(ctx, ctx->b.W, w, true, cudaMemcpyDeviceToDevice));
  } else {
    CU(cudaMemcpyAsync(ctx->b.stage, w, n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    CHK(repack(ctx, ctx->b.W, ctx->b.stage, true, cudaMemcpyDeviceToDevice));
  }
  float fl[2];
  CU(cudaMemcpyAsync(&fl[0], ctx->b.W + ctx->P.signal_scale, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  CU(cudaMemcpyAsync(&fl[1], ctx->b.W + ctx->P.signal_zero, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  CU(cudaStreamSynchronize(ctx->stream));
  ctx->signal_scale = fl[0];
  ctx->signal_zero = fl[1] > 0.5f;
  return AIDEEN_OK;
}

static int download_packed(aideen_ctx *ctx, const float *src, float *out, size_t n) {
  if (!out || n > ctx->Lx.total) return set_err(ctx, AIDEEN_E_INVALID, "bad download size");
  CHK(repack(ctx, ctx->b.stage, src, false, cudaMemcpyDeviceToDevice));
  CU(cudaMemcpyAsync(out, ctx->b.stage, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  CU(cudaStreamSynchronize(ctx->stream));
  return AIDEEN_OK;
}

int aideen_download_weights(aideen_ctx *ctx, float *out, size_t n) {
  if (!ctx) return AIDEEN_E_INVALID;
  return download_packed(ctx, ctx->b.W, out, n);
}

int aideen_download_grads(aideen_ctx *ctx, float *out, size_t n) {
  if (!ctx) return AIDEEN_E_INVALID;
  return download_packed(ctx, ctx->b.G, out, n);
}

// LM-head block [V*d | V (padded) | d] <-> packed [V*d + V + d] host array.
static int lm_block_copy(aideen_ctx *ctx, float *dev, float *host, bool to_host) {
  const size_t V = ctx->cfg.vocab, d = ctx->cfg.d_model;
  const size_t seg[3][2] = {{0, V * d}, {ctx->lm_b, V}, {ctx->lm_g, d}};
  size_t o = 0;
  for (auto &sg : seg) {
    if (to_host) CU(cudaMemcpyAsync(host + o, dev + sg[0], sg[1] * 4, cudaMemcpyDeviceToHost, ctx->stream));
    else CU(cudaMemcpyAsync(dev + sg[0], host + o, sg[1] * 4, cudaMemcpyHostToDevice, ctx->stream));
    o += sg[1];
  }
  return AIDEEN_OK;
}

int aideen_download_adam(aideen_ctx *ctx, float *m_core, float *v_core, size_t n_core, float *m_lm, float *v_lm) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  if (m_core) CHK(download_packed(ctx, ctx->b.M1, m_core, n_core));
  if (v_core) CHK(download_packed(ctx, ctx->b.M2, v_core, n_core));
  if (ctx->lm_len) {
    if (m_lm) CHK(lm_block_copy(ctx, ctx->b.Mlm1, m_lm, true));
    if (v_lm) CHK(lm_block_copy(ctx, ctx->b.Mlm2, v_lm, true));
  }
  return sync_and_check(ctx);
}

int aideen_upload_adam(aideen_ctx *ctx, const float *m_core, const float *v_core, size_t n_core, const float *m_lm,
                       const float *v_lm) {
  if (!ctx) return AIDEEN_E_INVALID;
  if ((m_core || v_core) && n_core != ctx->Lx.total) return set_err(ctx, AIDEEN_E_INVALID, "bad moment length");
  CU(join_side(ctx));
  {
    // moments that are non-zero where no gradient reaches keep the full Adam sweep
    const Layout &L = ctx->Lx;
    const size_t d = ctx->cfg.d_model, h = ctx->cfg.h_slots;
    auto dead_zero = [&](const float *m) {
      if (!m) return true;
      for (size_t blk : {L.wq, L.wk, L.wv})
        for (size_t r = 0; r < h * d; ++r)
          for (size_t c = kHeadDim; c < d; ++c)
            if (m[blk + r * d + c] != 0.f) return false;
      for (size_t s = 0; s < h; ++s)
        for (size_t i = (size_t)kHeadDim * d; i < d * d; ++i)
          if (m[L.wo + s * d * d + i] != 0.f) return false;
      return true;
    };
    const bool ok = dead_zero(m_core) && dead_zero(v_core);
    ctx->adam_dead_zero = (m_core && v_core) ? ok : (ctx->adam_dead_zero && ok);
  }
  for (int i = 0; i < 2; ++i) {
    const float *src = i ? v_core : m_core;
    if (!src) continue;
    CU(cudaMemcpyAsync(ctx->b.stage, src, n_core * 4, cudaMemcpyHostToDevice, ctx->stream));
    CHK(repack(ctx, i ? ctx->b.M2 : ctx->b.M1, ctx->b.stage, true, cudaMemcpyDeviceToDevice));
  }
  if (ctx->lm_len) {
    if (m_lm) CHK(lm_block_copy(ctx, ctx->b.Mlm1, const_cast<float *>(m_lm), false));
    if (v_lm) CHK(lm_block_copy(ctx, ctx->b.Mlm2, const_cast<float *>(v_lm), false));
  }
  return sync_and_check(ctx);
}

int aideen_upload_lm_head(aideen_ctx *ctx, const float *w_lm, const float *b_lm, const float *g_lm) {
  if (!ctx) return AIDEEN_E_INVALID;
  const size_t V = ctx->cfg.vocab, d = ctx->cfg.d_model;
  if (!V) return set_err(ctx, AIDEEN_E_INVALID, "context created with vocab = 0");
  CU(join_side(ctx));
  CHK(copy_in(ctx, ctx->b.lmp, w_lm, V * d * sizeof(float), AIDEEN_HOST));
  CHK(copy_in(ctx, ctx->b.lmp + ctx->lm_b, b_lm, V * sizeof(float), AIDEEN_HOST));
  CHK(copy_in(ctx, ctx->b.lmp + ctx->lm_g, g_lm, d * sizeof(float), AIDEEN_HOST));
  CU(cudaStreamSynchronize(ctx->stream));
  ctx->lm_ready = true;
  ctx->lm_split_stale = true;
  return AIDEEN_OK;
}

int aideen_download_lm_head(aideen_ctx *ctx, float *w_lm, float *b_lm, float *g_lm) {
  if (!ctx || !ctx->lm_ready) return set_err(ctx, AIDEEN_E_INVALID, "no LM head");
  CU(join_side(ctx));
  const size_t V = ctx->cfg.vocab, d = ctx->cfg.d_model;
  if (w_lm) CU(cudaMemcpyAsync(w_lm, ctx->b.lmp, V * d * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (b_lm) CU(cudaMemcpyAsync(b_lm, ctx->b.lmp + ctx->lm_b, V * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (g_lm) CU(cudaMemcpyAsync(g_lm, ctx->b.lmp + ctx->lm_g, d * 4, cudaMemcpyDeviceToHost, ctx->stream));
  CU(cudaStreamSynchronize(ctx->stream));
  return AIDEEN_OK;
}

int aideen_upload_embedding(aideen_ctx *ctx, const float *emb) {
  if (!ctx) return AIDEEN_E_INVALID;
  if (!ctx->cfg.vocab) return set_err(ctx, AIDEEN_E_INVALID, "context created with vocab = 0");
  CU(join_emb(ctx));
  CHK(copy_in(ctx, ctx->b.emb, emb, (size_t)ctx->cfg.vocab * ctx->cfg.d_model * 4, AIDEEN_HOST));
  CU(cudaStreamSynchronize(ctx->stream));
  ctx->emb_ready = true;
  return AIDEEN_OK;
}

int aideen_download_embedding(aideen_ctx *ctx, float *emb) {
  if (!ctx || !emb) return AIDEEN_E_INVALID;
  if (!ctx->emb_ready) return set_err(ctx, AIDEEN_E_INVALID, "embedding not uploaded");
  CU(join_emb(ctx));
  CU(cudaMemcpyAsync(emb, ctx->b.emb, (size_t)ctx->cfg.vocab * ctx->cfg.d_model * 4, cudaMemcpyDeviceToHost,
                     ctx->stream));
  return sync_and_check(ctx);
}

int aideen_reset_state(aideen_ctx *ctx) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(cudaMemsetAsync(ctx->b.mstate, 0,
                     (size_t)ctx->cfg.max_batch * ctx->cfg.h_slots * ctx->cfg.d_model * 4, ctx->stream));
  // the TBPTT carry of the FPM backward is cleared with the memory (gpu_deq.rs:3147)
  CU(cudaMemsetAsync(ctx->b.fcarry, 0,
                     (size_t)ctx->cfg.max_batch * ctx->cfg.h_slots * ctx->cfg.d_model * 4, ctx->stream));
  if (ctx->assoc) {  // the banks and the previous source (gpu_deq.rs:3141-3160)
    const size_t bh = (size_t)ctx->cfg.max_batch * ctx->cfg.h_slots;
    CU(cudaMemsetAsync(ctx->b.assoc_v, 0, bh * ctx->cfg.d_model * 4, ctx->stream));
    CU(cudaMemsetAsync(ctx->b.assoc_p, 0, bh * ctx->cfg.d_model * 4, ctx->stream));
    CU(cudaMemsetAsync(ctx->b.assoc_u, 0, bh * 4, ctx->stream));
  }
  return AIDEEN_OK;
}

int aideen_reset_optimizer(aideen_ctx *ctx) {
  if (!ctx) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  ctx->adam_dead_zero = true;
  CU(cudaMemsetAsync(ctx->b.M1, 0, ctx->W_len * 4, ctx->stream));
  CU(cudaMemsetAsync(ctx->b.M2, 0, ctx->W_len * 4, ctx->stream));
  if (ctx->lm_len) {
    CU(cudaMemsetAsync(ctx->b.Mlm1, 0, ctx->lm_len * 4, ctx->stream));
    CU(cudaMemsetAsync(ctx->b.Mlm2, 0, ctx->lm_len * 4, ctx->stream));
  }
  return AIDEEN_OK;
}

int aideen_forward(aideen_ctx *ctx, const aideen_run *run, const float *s_in, int where,
                   aideen_stats *stats) {
  if (!ctx) return AIDEEN_E_INVALID;
  CHK(check_run(ctx, run));
  const size_t N = (size_t)run->batch * run->seq_len;
  CHK(copy_in_rows(ctx, ctx->b.S_in, s_in, run->batch, run->seq_len, 1, ctx->cfg.d_model, where));
  (void)N;
  return run_forward(ctx, run, stats);
}

int aideen_forward_tokens(aideen_ctx *ctx, const aideen_run *run, const int32_t *tokens, int where,
                          aideen_stats *stats) {
  if (!ctx) return AIDEEN_E_INVALID;
  CHK(check_run(ctx, run));
  if (!ctx->emb_ready) return set_err(ctx, AIDEEN_E_INVALID, "embedding not uploaded");
  const int N = run->batch * run->seq_len;
  CHK(copy_in_rows(ctx, ctx->b.tokens, tokens, run->batch, run->seq_len, 1, 1, where));
  CU(join_emb(ctx));
  tl_mark(ctx, "entry", ctx->stream);
  ctx->emb_done = false;
  KL(launch_embed(ctx->b.tokens, ctx->b.emb, ctx->b.S_in, N, ctx->cfg.d_model, ctx->cfg.vocab, ctx->stream));
  return run_forward(ctx, run, stats);
}

int aideen_lm_head_loss(aideen_ctx *ctx, uint32_t batch, uint32_t seq_len, const int32_t *targets,
                        int where, float *loss_out) {
  if (!ctx) return AIDEEN_E_INVALID;
  const uint32_t N = batch * seq_len;
  if (N == 0 || N != ctx->N) return set_err(ctx, AIDEEN_E_INVALID, "LM head must follow a forward of the same shape");
  CHK(copy_in_rows(ctx, ctx->b.targets, targets, ctx->perm_B, ctx->perm_T, 1, 1, where));
  return run_lm_head(ctx, N, loss_out);
}

int aideen_adjoint(aideen_ctx *ctx, const aideen_adjoint_args *a, const float *dl_dh,
                   const float *rhs_slot, int where) {
  if (!ctx || !a) return AIDEEN_E_INVALID;
  const uint32_t N = a->batch * a->seq_len;
  if (N == 0 || N != ctx->N) return set_err(ctx, AIDEEN_E_INVALID, "adjoint must follow a forward of the same shape");
  const size_t d = ctx->cfg.d_model, h = ctx->cfg.h_slots;
  if (dl_dh) CHK(copy_in_rows(ctx, ctx->b.dl_dh, dl_dh, ctx->perm_B, ctx->perm_T, 1, d, where));
  const float *rs = nullptr;
  if (rhs_slot) {
    if (!ctx->b.rhs_slot) CU(dalloc(&ctx->b.rhs_slot, ctx->max_tokens * h * d));
    CHK(copy_in_rows(ctx, ctx->b.rhs_slot, rhs_slot, ctx->perm_B, ctx->perm_T, 1, h * d, where));
    rs = ctx->b.rhs_slot;
  }
  return run_adjoint(ctx, N, ctx->b.pre, nullptr, ctx->b.dl_dh, rs, a->iters, a->damping, a->anderson_m);
}

int aideen_adjoint_on(aideen_ctx *ctx, const aideen_adjoint_args *a, const float *hstar,
                      const float *branch, const float *dl_dh, const float *rhs_slot, int where) {
  if (!ctx || !a || !hstar || !branch) return AIDEEN_E_INVALID;
  const uint32_t N = a->batch * a->seq_len;
  if (N == 0 || N > ctx->max_tokens) return set_err(ctx, AIDEEN_E_INVALID, "tokens beyond the context caps");
  const size_t d = ctx->cfg.d_model, h = ctx->cfg.h_slots, bytes = (size_t)N * h * d * 4;
  const float *pa = hstar, *pb = branch;
  if (where != AIDEEN_DEVICE) {
    CHK(copy_in(ctx, ctx->b.hstar, hstar, bytes, where));
    CHK(copy_in(ctx, ctx->b.signal, branch, bytes, where));
    pa = ctx->b.hstar;
    pb = ctx->b.signal;
  }
  const float *rt = nullptr, *rs = nullptr;
  if (dl_dh) {
    if (where != AIDEEN_DEVICE) { CHK(copy_in(ctx, ctx->b.dl_dh, dl_dh, (size_t)N * d * 4, where)); rt = ctx->b.dl_dh; }
    else rt = dl_dh;
  }
  if (rhs_slot) {
    if (where != AIDEEN_DEVICE) {
      if (!ctx->b.rhs_slot) CU(dalloc(&ctx->b.rhs_slot, ctx->max_tokens * h * d));
      CHK(copy_in(ctx, ctx->b.rhs_slot, rhs_slot, bytes, where));
      rs = ctx->b.rhs_slot;
    } else {
      rs = rhs_slot;
    }
  }
  ctx->N = 0;  // the forward state no longer matches this adjoint
  ctx->perm_B = 1;  // rows in the caller's order
  ctx->perm_T = (int)N;
  return run_adjoint(ctx, N, pa, pb, rt, rs, a->iters, a->damping, a->anderson_m);
}

int aideen_temporal_scan(aideen_ctx *ctx, uint32_t batch, uint32_t seq_len, const float *hstar, int where) {
  if (!ctx) return AIDEEN_E_INVALID;
  const int h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  if (batch == 0 || seq_len == 0 || batch > ctx->cfg.max_batch || seq_len > ctx->cfg.max_seq_len)
    return set_err(ctx, AIDEEN_E_INVALID, "batch/seq_len outside the context caps");
  if (hstar) {
    CHK(copy_in_rows(ctx, ctx->b.hstar, hstar, (int)batch, (int)seq_len, 1, (size_t)h * d, where));
    ctx->perm_B = (int)batch;
    ctx->perm_T = (int)seq_len;
    ctx->N = batch * seq_len;
  } else if (ctx->N != batch * seq_len || ctx->last_run.batch != batch) {
    return set_err(ctx, AIDEEN_E_INVALID, "no h* given and the last forward has another shape");
  }
  TemporalArgs a{};
  a.B = (int)batch; a.T = (int)seq_len; a.h = h; a.d = d; a.W = ctx->b.W;
  a.off_alog = ctx->P.alog; a.off_wx = ctx->P.wx; a.off_wout = ctx->P.wout;
  a.hstar = ctx->b.hstar; a.hist = ctx->b.hist; a.mstate = ctx->b.mstate;
  KL(launch_temporal_scan(a, ctx->stream));
  return AIDEEN_OK;
}

int aideen_source_grad(aideen_ctx *ctx, float *out, int where) {
  if (!ctx || !out) return AIDEEN_E_INVALID;
  const int N = ctx->adj_N, h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  if (N == 0) return set_err(ctx, AIDEEN_E_INVALID, "no adjoint has run");
  KL(launch_source_grad(ctx->b.gpre, ctx->b.dS, N, h, d, ctx->stream));  // dS doubles as staging
  const bool perm = ctx->perm_B > 1 && ctx->perm_T > 1;
  const float *res = ctx->b.dS;
  if (perm) {
    CU(ensure_perm(ctx));
    float *dst = where == AIDEEN_DEVICE ? out : ctx->b.perm;
    KL(launch_permute_rows(ctx->b.dS, dst, ctx->perm_B, ctx->perm_T, 1, d, false, ctx->stream));
    res = dst;
  }
  if (where != AIDEEN_DEVICE) {
    CU(cudaMemcpyAsync(out, res, (size_t)N * d * 4, cudaMemcpyDeviceToHost, ctx->stream));
    CHK(sync_and_check(ctx));
  } else if (!perm) {
    CU(cudaMemcpyAsync(out, res, (size_t)N * d * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  return AIDEEN_OK;
}

int aideen_weight_grads(aideen_ctx *ctx) {
  if (!ctx) return AIDEEN_E_INVALID;
  return run_weight_grads(ctx, true);
}

int aideen_apply_update(aideen_ctx *ctx, const aideen_update *u) {
  if (!ctx) return AIDEEN_E_INVALID;
  return run_update(ctx, u);
}

int aideen_renormalize_spectral(aideen_ctx *ctx, uint32_t n_iters, float attn, float win, float fpm,
                                float wv, float wo, float *sig) {
  if (!ctx) return AIDEEN_E_INVALID;
  KL(launch_spectral(ctx->b.W, ctx->cfg.d_model, ctx->cfg.h_slots, ctx->P, n_iters, attn, win, fpm,
                     wv, wo, ctx->b.sigmas, ctx->stream));
  if (sig) {
    CU(cudaMemcpyAsync(sig, ctx->b.sigmas, (5 * ctx->cfg.h_slots + 2) * 4, cudaMemcpyDeviceToHost,
                       ctx->stream));
    CU(cudaStreamSynchronize(ctx->stream));
  }
  return AIDEEN_OK;
}

int aideen_train_step(aideen_ctx *ctx, const aideen_step_args *a, const int32_t *tokens,
                      const int32_t *targets, int where, float *loss_out, aideen_stats *stats) {
  if (!ctx || !a) return AIDEEN_E_INVALID;
  // the early-zeroed gradient buffer belongs to this call only (also when it fails)
  struct GzGuard {
    aideen_ctx *c;
    ~GzGuard() { c->g_zeroed = false; }
  } gz_guard{ctx};
  CHK(check_run(ctx, &a->run));
  if (!ctx->emb_ready || !ctx->lm_ready)
    return set_err(ctx, AIDEEN_E_INVALID, "train step needs the embedding and the LM head");
  const int N = a->run.batch * a->run.seq_len;
  // a step that failed after summing its LM-head gradients must not make this
  // step skip the sum
  ctx->lm_reduced = false;
  CHK(copy_in_rows(ctx, ctx->b.tokens, tokens, a->run.batch, a->run.seq_len, 1, 1, where));
  CHK(copy_in_rows(ctx, ctx->b.targets, targets, a->run.batch, a->run.seq_len, 1, 1, where));
  if (a->emb_update > 2) return set_err(ctx, AIDEEN_E_INVALID, "emb_update must be 0, 1 or 2");
  CU(join_emb(ctx));
  tl_mark(ctx, "entry", ctx->stream);
  ctx->emb_done = false;
  KL(launch_embed(ctx->b.tokens, ctx->b.emb, ctx->b.S_in, N, ctx->cfg.d_model, ctx->cfg.vocab, ctx->stream));
  const bool sampled = a->lm_samples > 0;
  const int nch = pipeline_chunks(ctx, &a->run);
  // (the pipelined step builds the embedding CSR after its first solve launch)
  if (a->emb_update && nch <= 1) CHK(emb_csr_early(ctx, N));
  if (nch > 1) {
    CHK(run_step_pipelined(ctx, a, nch, stats));
  } else {
    CHK(run_forward(ctx, &a->run, stats));
    if (sampled) CHK(run_lm_head_sampled(ctx, N, a));
    else CHK(run_lm_head(ctx, N, nullptr));
    CHK(run_adjoint(ctx, N, ctx->b.pre, nullptr, ctx->b.dl_dh, nullptr, a->adj_iters, a->run.damping,
                    a->anderson_m));
  }
  // data parallel with Adam: sharded update (no profiling: its per-class
  // timing assumes one stream)
  ctx->shard_step = a->update.allreduce && ctx->comm && ctx->nranks > 1 && a->update.rule == AIDEEN_RULE_ADAM &&
                    !ctx->prof && !no_sharded_update();
  const int wg = run_weight_grads(ctx, a->emb_update == 2);
  if (wg != AIDEEN_OK) {
    ctx->shard_step = false;
    return wg;
  }
  if (ctx->lmg_pending) {  // the last chunk's dW_lm and LM-head sums
    CU(cudaStreamWaitEvent(ctx->stream, ctx->ev_lmg, 0));
    ctx->lmg_pending = false;
  }
  tl_mark(ctx, "wgrads", ctx->stream);
  aideen_update up = a->update;
  if (sampled) up.update_lm_head = 0;  // its rows were updated inside the LM stage
  CHK(run_update(ctx, &up));
  tl_mark(ctx, "update", ctx->stream);
  if (a->renorm)
    KL(launch_spectral(ctx->b.W, ctx->cfg.d_model, ctx->cfg.h_slots, ctx->P, 12, 0.10f, 0.30f, 0.70f,
                       0.50f, 0.50f, ctx->b.sigmas, ctx->stream));
  // the reference updates the embedding rows last (trainer.rs:3282-3300)
  if (a->emb_update && !ctx->emb_done) CHK(run_emb_update(ctx, N, a));
  ctx->emb_done = false;
  tl_mark(ctx, "end", ctx->stream);
  tl_flush(ctx);
  if (loss_out) {
    // through the pinned mailbox: one asynchronous copy, one wait (in
    // sync_and_check) instead of a blocking pageable copy
    float *dst = ctx->hbox ? reinterpret_cast<float *>(&ctx->hbox[2]) : loss_out;
    CU(cudaMemcpyAsync(dst, ctx->b.scal + 1, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    CHK(sync_and_check(ctx));
    if (ctx->hbox) memcpy(loss_out, dst, sizeof(float));
  }
  return AIDEEN_OK;
}

static void *buf_ptr(aideen_ctx *ctx, int which, size_t *count) {
  const size_t N = ctx->N ? ctx->N : ctx->adj_N, h = ctx->cfg.h_slots, d = ctx->cfg.d_model;
  const size_t Na = ctx->adj_N ? ctx->adj_N : N;
  DevBufs &b = ctx->b;
  switch (which) {
    case AIDEEN_BUF_HSTAR: *count = N * h * d; return b.hstar;
    case AIDEEN_BUF_POOLED: *count = N * d; return b.pooled;
    case AIDEEN_BUF_SIGNAL: *count = N * h * d; return b.signal;
    case AIDEEN_BUF_ATTN: *count = N * h * d; return b.A;
    case AIDEEN_BUF_ITERS: *count = N * h; return b.iters;
    case AIDEEN_BUF_ADJ_V: *count = Na * h * d; return b.v;
    case AIDEEN_BUF_GPRE: *count = Na * h * d; return b.gpre;
    case AIDEEN_BUF_DL_DH: *count = N * d; return b.dl_dh;
    case AIDEEN_BUF_HIST_CTX: *count = N * h * d; return b.hist;
    case AIDEEN_BUF_MSTATE: *count = (size_t)ctx->cfg.max_batch * h * d; return b.mstate;
    case AIDEEN_BUF_FPM_CTX: *count = N * h * d; return b.fpmctx;
    case AIDEEN_BUF_ALPHA: *count = N * h * h; return b.alpha;
    case AIDEEN_BUF_S_IN: *count = N * d; return b.S_in;
    case AIDEEN_BUF_DS_IN: *count = N * d; return b.dS;
    case AIDEEN_BUF_LM_GRADS: *count = ctx->lm_len ? ctx->lm_b + ctx->cfg.vocab + d : 0; return b.Glm;
    case AIDEEN_BUF_LM_SAMPLES: *count = ctx->lcap; return b.lS;
    case AIDEEN_BUF_PRE: *count = N * h * d; return b.pre;
    case AIDEEN_BUF_FPM_DM: *count = b.fdm ? N * h * d : 0; return b.fdm;
    case AIDEEN_BUF_FPM_CARRY: *count = (size_t)ctx->cfg.max_batch * h * d; return b.fcarry;
    default: *count = 0; return nullptr;
  }
}

int aideen_read(aideen_ctx *ctx, int which, void *dst, size_t n) {
  if (!ctx || !dst) return AIDEEN_E_INVALID;
  CU(join_side(ctx));
  size_t count = 0;
  void *p = buf_ptr(ctx, which, &count);
  if (!p) return set_err(ctx, AIDEEN_E_INVALID, "unknown or absent buffer");
  if (n > count) return set_err(ctx, AIDEEN_E_INVALID, "read beyond the buffer's valid extent");
  if (which == AIDEEN_BUF_LM_GRADS) {  // packed [gW | gb | gg] from the padded block
    const size_t segs[3][2] = {{0, ctx->lm_b}, {ctx->lm_b, ctx->cfg.vocab}, {ctx->lm_g, ctx->cfg.d_model}};
    size_t o = 0;
    for (auto &sg : segs) {
      const size_t m = sg[1] < n - o ? sg[1] : n - o;
      if (m) CU(cudaMemcpyAsync((float *)dst + o, ctx->b.Glm + sg[0], m * 4, cudaMemcpyDeviceToHost, ctx->stream));
      o += m;
    }
    CU(cudaStreamSynchronize(ctx->stream));
    return AIDEEN_OK;
  }
  // row-indexed buffers come back in the caller's row order
  size_t len = 0;
  int blocks = 1;
  const size_t hh = ctx->cfg.h_slots, dd = ctx->cfg.d_model;
  switch (which) {
    case AIDEEN_BUF_HSTAR: case AIDEEN_BUF_SIGNAL: case AIDEEN_BUF_ATTN: case AIDEEN_BUF_GPRE:
    case AIDEEN_BUF_HIST_CTX: case AIDEEN_BUF_FPM_CTX: case AIDEEN_BUF_PRE: case AIDEEN_BUF_FPM_DM:
      len = hh * dd; break;
    case AIDEEN_BUF_POOLED: case AIDEEN_BUF_DL_DH: case AIDEEN_BUF_S_IN: case AIDEEN_BUF_DS_IN:
      len = dd; break;
    case AIDEEN_BUF_ITERS: len = hh; break;
    case AIDEEN_BUF_ALPHA: len = hh * hh; break;
    case AIDEEN_BUF_ADJ_V: len = dd; blocks = (int)hh; break;
    default: break;
  }
  const int PB = ctx->perm_B, PT = ctx->perm_T;
  if (len && PB > 1 && PT > 1 && count == (size_t)PB * PT * blocks * len) {
    CU(ensure_perm(ctx));
    KL(launch_permute_rows(p, ctx->b.perm, PB, PT, blocks, len, false, ctx->stream));
    p = ctx->b.perm;
  }
  CU(cudaMemcpyAsync(dst, p, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
  return sync_and_check(ctx);
}

void *aideen_device_ptr(aideen_ctx *ctx, int which) {
  if (!ctx) return nullptr;
  join_side(ctx);
  size_t count = 0;
  return buf_ptr(ctx, which, &count);
}

namespace {
__global__ void fill_kernel(float *x, size_t n, uint32_t seed) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    uint32_t v = (uint32_t)i * 2654435761u ^ seed;
    v ^= v >> 13; v *= 0x5bd1e995u; v ^= v >> 15;
    x[i] = (float)(v & 0xFFFFFF) / 8388608.0f - 1.0f;
  }
}
__global__ void relerr_kernel(const float *a, const float *b, size_t n, double *out) {
  double num = 0, den = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const double d = (double)a[i] - b[i];
    num += d * d;
    den += (double)b[i] * b[i];
  }
  atomicAdd(&out[0], num);
  atomicAdd(&out[1], den);
}
}  // namespace

int aideen_gemm_selftest(aideen_ctx *ctx, int M, int N, int K, int batch, int trans_a, int trans_b,
                         int flags, float *rel_err, float *ms_tc, float *ms_simt) {
  if (!ctx || M <= 0 || N <= 0 || K <= 0 || batch <= 0) return AIDEEN_E_INVALID;
  const size_t na = (size_t)M * K * batch, nb = (size_t)K * N * batch, nc = (size_t)M * N * batch;
  float *A = nullptr, *B = nullptr, *C1 = nullptr, *C2 = nullptr;
  double *acc = nullptr;
  CU(cudaMalloc(&A, na * 4)); CU(cudaMalloc(&B, nb * 4)); CU(cudaMalloc(&C1, nc * 4));
  CU(cudaMalloc(&C2, nc * 4)); CU(cudaMalloc(&acc, 16));
  cudaStream_t st = ctx->stream;
  fill_kernel<<<256, 256, 0, st>>>(A, na, 1u);
  fill_kernel<<<256, 256, 0, st>>>(B, nb, 2u);
  CU(cudaMemsetAsync(acc, 0, 16, st));
  const long lda = trans_a ? M : K, ldb = trans_b ? K : N;
  GemmArgs g = gemm(M, N, K, batch, A, lda, (long)M * K, trans_a != 0, B, ldb, (long)K * N, trans_b != 0,
                    C1, N, (long)M * N);
  g.tf32 = (flags & AIDEEN_SELFTEST_TF32) != 0;
  int rc = AIDEEN_OK;
  const bool presplit = (flags & AIDEEN_SELFTEST_PRESPLIT) != 0;
  float *Alo = nullptr, *Blo = nullptr, *Ahi = nullptr, *Bhi = nullptr;
  if (presplit) {
    CU(cudaMalloc(&Ahi, na * 4)); CU(cudaMalloc(&Alo, na * 4));
    CU(cudaMalloc(&Bhi, nb * 4)); CU(cudaMalloc(&Blo, nb * 4));
    CU(launch_split_hilo(A, Ahi, Alo, na, st));
    CU(launch_split_hilo(B, Bhi, Blo, nb, st));
  }
  GemmArgs gs = g;
  gs.A = Ahi; gs.B = Bhi;
  auto run_tc = [&](float *wsp, size_t wsn) -> cudaError_t {
    return presplit ? tc_gemm_split(gs, Alo, Blo, st, wsp, wsn) : tc_gemm(g, st, wsp, wsn);
  };
  if (presplit ? !tc_split_supported(gs, Alo, Blo) : !tc_gemm_supported(g)) {
    rc = set_err(ctx, AIDEEN_E_UNSUPPORTED, "shape not supported by the tensor-core GEMM");
  } else {
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0); cudaEventCreate(&e1); cudaEventCreate(&e2);
    float *wsp = nullptr;
    const size_t wsn = 16 * (size_t)M * N * batch;  // up to 16 split-K partials of every output
    cudaMalloc(&wsp, wsn * 4);
    run_tc(wsp, wsn);  // warm-up
    const int reps = 10;
    cudaEventRecord(e0, st);
    cudaError_t ce = cudaSuccess;
    for (int i = 0; i < reps && ce == cudaSuccess; ++i) ce = run_tc(wsp, wsn);
    cudaEventRecord(e1, st);
    GemmArgs g2 = g;
    g2.C = C2;
    cudaError_t ce2 = gemm_f32(g2, st);
    cudaEventRecord(e2, st);
    relerr_kernel<<<256, 256, 0, st>>>(C1, C2, nc, acc);
    double h[2] = {0, 0};
    cudaMemcpyAsync(h, acc, 16, cudaMemcpyDeviceToHost, st);
    cudaError_t se = cudaStreamSynchronize(st);
    float t1 = 0, t2 = 0;
    cudaEventElapsedTime(&t1, e0, e1);
    cudaEventElapsedTime(&t2, e1, e2);
    cudaEventDestroy(e0); cudaEventDestroy(e1); cudaEventDestroy(e2);
    cudaFree(wsp);
    if (ce != cudaSuccess || ce2 != cudaSuccess || se != cudaSuccess)
      rc = set_err(ctx, AIDEEN_E_CUDA, "GEMM self-test launch failed");
    else if (presplit ? tc_split_error(true) : tc_gemm_error(true))
      rc = set_err(ctx, AIDEEN_E_TIMEOUT, "tensor-core GEMM pipeline wait timed out");
    if (getenv("AIDEEN_SELFTEST_DUMP")) {
      float a[8], b2[8];
      cudaMemcpy(a, C1, 32, cudaMemcpyDeviceToHost);
      cudaMemcpy(b2, C2, 32, cudaMemcpyDeviceToHost);
      for (int i = 0; i < 8; ++i) fprintf(stderr, "selftest C[%d] tc=%g fp32=%g\n", i, a[i], b2[i]);
      fprintf(stderr, "tc err flag %u\n", tc_gemm_error(false));
    }
    if (rel_err) *rel_err = (float)std::sqrt(h[0] / (h[1] > 0 ? h[1] : 1.0));
    if (ms_tc) *ms_tc = t1 / reps;
    if (ms_simt) *ms_simt = t2;
  }
  cudaFree(A); cudaFree(B); cudaFree(C1); cudaFree(C2); cudaFree(acc);
  if (presplit) { cudaFree(Ahi); cudaFree(Alo); cudaFree(Bhi); cudaFree(Blo); }
  return rc;
}

int aideen_comm_unique_id(char out[AIDEEN_UNIQUE_ID_BYTES]) {
  static_assert(sizeof(ncclUniqueId) == AIDEEN_UNIQUE_ID_BYTES, "ncclUniqueId size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return AIDEEN_E_NCCL;
  std::memcpy(out, &id, sizeof(id));
  return AIDEEN_OK;
}

int aideen_comm_init(aideen_ctx *ctx, const char id_bytes[AIDEEN_UNIQUE_ID_BYTES], int nranks, int rank) {
  if (!ctx || nranks < 1 || rank < 0 || rank >= nranks) return AIDEEN_E_INVALID;
  if (nranks == 1) return AIDEEN_OK;
  ncclUniqueId id;
  std::memcpy(&id, id_bytes, sizeof(id));
  CU(cudaSetDevice(ctx->device));
  ncclResult_t r = ncclCommInitRank(&ctx->comm, nranks, id, rank);
  if (r != ncclSuccess) return set_err(ctx, AIDEEN_E_NCCL, std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
  ctx->nranks = nranks;
  ctx->rank = rank;
  return AIDEEN_OK;
}

int aideen_allreduce_grads(aideen_ctx *ctx, int timeout_ms) {
  if (!ctx) return AIDEEN_E_INVALID;
  return run_allreduce(ctx, timeout_ms);
}

}  // extern "C"
