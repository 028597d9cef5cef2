// Kernel argument blocks and launchers shared between the .cu files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "layout.h"

namespace aideen {

// Strided batched fp32 GEMM on CUDA cores:
//   C[b] = alpha * opA(A[b]) * opB(B[b]) + beta * C[b]   (row-major)
// opA(m,k) = transA ? A[k*lda+m] : A[m*lda+k], plus abias[stored column]
// when abias != nullptr (the stored column is m when transA, else k).
// opB(k,n) = transB ? B[n*ldb+k] : B[k*ldb+n].
struct GemmArgs {
  int M, N, K, batch;
  const float *A; long lda, strideA; bool transA;
  const float *B; long ldb, strideB; bool transB;
  float *C; long ldc, strideC;
  float alpha, beta;
  const float *abias; long strideAbias;
  // tensor-core kernel only: one TF32 product per term (operands rounded to
  // tf32, fp32 accumulation) instead of the fp32-accurate 3xTF32 split
  bool tf32;
  // col_group > 0: C's columns come in groups of col_group that live
  // group_stride floats apart (column n is stored at
  // (n / col_group) * group_stride + n % col_group of the row), e.g. the
  // Q, K and V blocks of one 96-column product
  int col_group; long group_stride;
};
cudaError_t gemm_f32(const GemmArgs &g, cudaStream_t s);
// Same contract on tcgen05 tensor cores (3xTF32, fp32-accurate, or single TF32
// with g.tf32); no abias; g.col_group needs the split-K workspace.
bool tc_gemm_supported(const GemmArgs &g);
// ws: optional workspace for split-K partial sums (ws_floats capacity).
cudaError_t tc_gemm(const GemmArgs &g, cudaStream_t s, float *ws = nullptr, size_t ws_floats = 0);
unsigned int tc_gemm_error(bool reset);
// Kernels a GEMM call launched beyond its main one (split-K reductions) since
// the last call of tc_take_extra_launches, on this host thread.
extern thread_local unsigned tc_extra_launches;
unsigned tc_take_extra_launches();
// Persistent tcgen05 GEMM on pre-split operands (tcgemm_split.cu): g.A / g.B
// hold the tf32-exact high parts, A_lo / B_lo the remainders (same strides);
// beta must be 0 or 1.
bool tc_split_supported(const GemmArgs &g, const float *A_lo, const float *B_lo);
// row_stats (with row_bias): per-(row, 256-column tile) softmax statistics of
// C + bias in base 2, (max, sum exp2(z - max)), [M][ceil(N / 256)] (batch 1).
cudaError_t tc_gemm_split(const GemmArgs &g, const float *A_lo, const float *B_lo, cudaStream_t s,
                          float *ws = nullptr, size_t ws_floats = 0, int max_ctas = 0,
                          const float *row_bias = nullptr, float2 *row_stats = nullptr);
unsigned int tc_split_error(bool reset);
cudaError_t picard_error_async(unsigned int *host_flag, cudaStream_t st);
unsigned int *picard_error_dev();   // device address of the Picard error word
// x -> (hi, lo) with hi exact in tf32 and lo = x - hi (n % 4 == 0).
cudaError_t launch_split_hilo(const float *x, float *hi, float *lo, size_t n, cudaStream_t st);
// out[c][r] = split(x[r][c]): transposed hi / lo copies (row stride ldt).
cudaError_t launch_transpose_split(const float *x, int R, int C, long ldx, float *hiT, float *loT, long ldt,
                                   cudaStream_t st);

struct AttnArgs {
  int h, d;
  const float *W;
  size_t off_qb, off_kb, off_anchor;
  const float *Qh, *Kh, *Vh;      // [N][h] rows of 32 projections without bias, row stride qkv_ld
  int qkv_ld;                     // floats between consecutive (token, slot) rows of Qh / Kh / Vh
  float *alpha, *nmix, *rmix;     // [N][h][h], [N][h][32], [N][h]
  const float *signal, *amat;     // [N][h][d]
  float *A, *scale, *rho, *Rsrc;  // [N][h][d], [N][h] x3
};

struct PicardArgs {
  int B, T, h, d, max_iters, slot_coord;
  int t0, t1;      // token range of this launch (state carried in hstar / mstate)
  int n_resident;  // FPM matrices staged in shared memory (set by the launcher)
  int use_tmem;    // 1: rank-32 matrices in tensor memory (d = 512): 3..5, or 2..5 with push
  int push;        // 1: memory rows / read keys pushed into every peer's inbox by bulk copy
  int anderson_m;  // forward Anderson residuals mixed: 0 (plain Picard), 2 or 3
  float eps, blend, alpha_m, tau, gate_min;
  const float *W;
  size_t off_ns, off_anchor, off_hscale, off_hbias, off_wkm, off_wqm, off_bread, off_wgate,
      off_bwrite, off_wkw, off_wvw, off_bdelta, off_wup, off_wdown, off_bret, off_alog, off_wx;
  const float *signal, *A;
  float *hstar, *pre, *hist, *fpmctx, *mstate;
  int32_t *iters;
  // associative branch of the upper h/2 slots (with FPM; see picard_kernel)
  int assoc;
  size_t off_alpha_assoc;
  const float *s_in;               // [N][d] token-major S_in rows
  float *assoc_v, *assoc_p;        // [B][h][d] bank value, previous source (carried)
  float *assoc_u;                  // [B][h] bank usage (carried)
  float *sig_store;                // [N][h][d] stored signal: the payload on the upper slots
  float *assoc_read;               // [N][h][d] bank value each token read (upper slots' rows)
};

struct AdjointArgs {
  int N, h, d, iters, anderson_m;
  float beta;
  const float *pre_a, *pre_b;  // pre = pre_a (+ pre_b)
  const float *rhs_tok;        // [N][d] or null (scaled 1/h per slot)
  const float *rhs_slot;       // [N][h][d] or null
  const float *NS;
  float *v;                    // [h][v_ld][d] (rows n of slot s at (s * v_ld + n) * d)
  int v_ld;                    // rows per slot block of v (0: N)
  int max_ctas;                // SMs to use (0: every SM), at full occupancy each
  float *gpre;                 // [N][h][d]
  float *nsg;                  // [N][d] per-token NormScale-gradient partials or null
  float *nsg_cta;              // [grid][d] per-CTA NormScale-gradient partials or null
  uint32_t spin_limit;         // bound of each stage wait (set by launch_adjoint)
};
// Reads and clears the adjoint's timeout flag (stream-ordered copy into host_flag).
cudaError_t adjoint_error_async(unsigned int *host_flag, cudaStream_t st);
unsigned int *adjoint_error_dev();  // device address of the adjoint error word
// Dynamic shared memory of one adjoint CTA for these inputs (h*d floats per
// staged tensor, double-buffered; plus the Anderson ring where it is used).
size_t adjoint_smem_bytes(int h, int d, bool has_b, bool has_rs, bool has_tok, int anderson_m);

struct AttnBwdArgs {
  int h, d;
  const float *W;
  size_t off_qb, off_kb, off_anchor;
  const float *gpre, *amat, *scale, *rho, *Rsrc, *signal;
  float *da, *dRc;
  const float *dn, *nmix, *rmix, *alpha, *Qh, *Kh, *Vh;
  float *dQ, *dK, *dV;
  int qkv_ld;                     // row stride of Qh / Kh / Vh and of dQ / dK / dV
};

cudaError_t launch_embed(const int32_t *tok, const float *emb, float *S, int N, int d, int vocab,
                         cudaStream_t st);
cudaError_t launch_attn_softmax(const AttnArgs &a, int N, cudaStream_t st);
cudaError_t launch_attn_scale(const AttnArgs &a, int rows, cudaStream_t st);
cudaError_t launch_picard(const PicardArgs &a, bool fpm, cudaStream_t st);
cudaError_t launch_pool_rmsnorm(const float *hstar, const float *g, float *pooled, float *y,
                                float *lrms, int N, int h, int d, cudaStream_t st);
cudaError_t launch_solve_stats(const int32_t *iters, const float *hstar, int rows, int d,
                               int max_iters, unsigned long long *st4p, cudaStream_t st);

// grid_out (optional): CTAs launched, i.e. the rows of nsg_cta written.
cudaError_t launch_adjoint(const AdjointArgs &a, cudaStream_t st, int *grid_out = nullptr);
cudaError_t launch_source_grad(const float *gpre, float *out, int N, int h, int d, cudaStream_t st);
cudaError_t launch_attn_bwd_scale(const AttnBwdArgs &a, int rows, cudaStream_t st);
cudaError_t launch_attn_bwd_softmax(const AttnBwdArgs &a, int N, cudaStream_t st);
// dsig[n][s][:] -= g_pre[n][s][:] for the upper h/2 slots (the associative
// slots, whose branch does not hold their signal).
cudaError_t launch_sub_upper_slots(float *dsig, const float *gpre, int N, int h, int d, cudaStream_t st);
// The reference's alpha_assoc gradient (fused_fpm_retain_bwd.wgsl:1129-1160,
// 1281-1284), default flags: for every upper slot s,
//   G[s] = sigmoid'(alpha_s) * sum_n (v[s][n] . V[n][s]) / max(rms(V[n][s]), 0.1)
// with V the bank value token n read and v the adjoint ([h][N][d]); written, not added.
cudaError_t launch_assoc_alpha_grad(const float *v, const float *vread, const float *alpha_raw, int N, int h, int d,
                                    float *g_alpha, cudaStream_t st);
cudaError_t launch_dsig_init(const AttnBwdArgs &a, float *dsig, int rows, int slot_coord,
                             cudaStream_t st);
// out[map(c)] (+)= sum_r X[r*ld + c], c < ncols; map(c) = (c/seg)*ostride + c%seg.
// istride (0: seg) spaces the input columns the same way: input column of c
// is (c/seg)*istride + c%seg.
cudaError_t launch_colsum(const float *X, int rows, int ncols, long ld, float *out, int seg,
                          long ostride, bool accumulate, cudaStream_t st, long istride = 0);
// Wcat[s][j][0:32 | 32:64 | 64:96] = W_q / W_k / W_v[s][j][0:32]: the three
// head projections as one [d][96] operand per slot.
cudaError_t launch_pack_qkv(const float *W, size_t off_q, size_t off_k, size_t off_v, int h, int d, float *Wcat,
                            cudaStream_t st);
cudaError_t launch_add(float *dst, const float *a, const float *b, size_t n, cudaStream_t st);
// Row permutation between the caller's order (row b*T + t) and the library's
// token-major order (row t*B + b), for `blocks` consecutive sets of B*T rows of
// `len` 4-byte words each (to_internal: caller -> library).
cudaError_t launch_permute_rows(const void *src, void *dst, int B, int T, int blocks, size_t len,
                                bool to_internal, cudaStream_t st);
cudaError_t launch_add_rowbias(float *dst, const float *x, const float *bias, size_t rows, size_t len,
                               cudaStream_t st);

// optimizer / renorm
// Strided segments of a parameter vector (float offsets, rows of row4
// float4s, `stride` floats apart; start4 = prefix sums of rows * row4).
struct AdamSegs {
  unsigned long long off[8], start4[9];
  long stride[8];
  int rows[8], row4[8];
  int n;
};
cudaError_t launch_adam_segs(float *w, const float *g, float *m1, float *m2, const AdamSegs &sg, float lr,
                             float b1, float b2, float eps, float bc1, float bc2, float gs, cudaStream_t st);
cudaError_t launch_adam(float *w, const float *g, float *m1, float *m2, size_t n, float lr,
                        float b1, float b2, float eps, float bc1, float bc2, float gs,
                        cudaStream_t st);
cudaError_t launch_clipped_sgd(float *w, const float *g, size_t n, size_t main_len, float lr,
                               float wd, float gs, cudaStream_t st);
cudaError_t launch_spectral(float *W, int d, int h, const Layout &L, int n_iters, float attn,
                            float win, float fpm, float wv, float wo, float *sigmas,
                            cudaStream_t st);

// LM head helpers
cudaError_t launch_count_active(const int32_t *tg, int N, float *out, cudaStream_t st);
// dlogits replace the logits in place; with lo != nullptr the row is written
// pre-split: logits <- tf32-exact high part, lo <- remainder (same strides).
cudaError_t launch_softmax_ce(float *logits, const float *bias, const int32_t *tg,
                              const float *n_active, int N, int V, long ld, float *loss_rows, float *lo,
                              cudaStream_t st);
// Pre-split softmax-CE over blocks of rows that also writes per-block column
// sums of dlogits: colpart is [softmax_rows_blocks(N)][ld]; ld * 4 bytes must
// fit in one block's shared memory (vocab <= 58,000).
int softmax_rows_blocks(int N, int max_blocks = 0);
// max_blocks caps the grid (0: one block per SM); accumulate adds into colpart.
// stats: optional per-(row, 256-column tile) statistics from the logits GEMM
// ([N][ceil(V / 256)]); with them the row's max / sum need no read pass.
cudaError_t launch_softmax_ce_split(float *logits, const float *bias, const int32_t *tg,
                                    const float *n_active, int N, int V, long ld, float *loss_rows,
                                    float *lo, float *colpart, cudaStream_t st, int max_blocks = 0,
                                    bool accumulate = false, const float2 *stats = nullptr);
cudaError_t launch_rmsnorm_bwd(const float *dy, const float *P, const float *lrms,
                               const float *g, float *dl_dh, float *ggp, int N, int d,
                               cudaStream_t st);
cudaError_t launch_sum(const float *x, int n, float *out, cudaStream_t st);

// Sampled-softmax LM head and embedding update (lm_sampled.cu).
// S[cap] <- sampled vocabulary of the targets (K = *K entries used), *active <-
// valid target count (>= 1); err bit 1: candidate draws exhausted, bit 2: K > cap.
cudaError_t launch_sample_set(const int32_t *tg, int N, int V, int num_samples, int max_samples,
                              unsigned long long seed, uint32_t step, int32_t *S, int *K, float *active, int cap,
                              unsigned int *err, cudaStream_t st);
cudaError_t launch_gather_rows(const float *W, const int32_t *S, const int *K, int cap, int d, float *WS,
                               cudaStream_t st);
cudaError_t launch_softmax_sampled(float *logits, long ld, const float *b_lm, const int32_t *S, const int *K,
                                   const int32_t *tg, int V, const float *active, float *loss_rows, int N,
                                   cudaStream_t st);
cudaError_t launch_lm_sampled_adam(float *W, float *b, float *M1, float *M2, size_t off_b, const float *dW,
                                   const float *db, const int32_t *S, const int *K, int cap, int d, float *WS,
                                   float lr, float b1, float b2, float eps, float bc1, float bc2, cudaStream_t st);
int emb_csr_max_tokens();
cudaError_t launch_emb_csr(const int32_t *tok, int N, int V, int32_t *uniq, int32_t *off, int32_t *pos, int *U,
                           cudaStream_t st);
cudaError_t launch_emb_adam(float *emb, float *M1, float *M2, const float *grad, const int32_t *uniq,
                            const int32_t *off, const int32_t *pos, const int *U, int ucap, int d, float lr,
                            float b1, float b2, float eps, float bc1, float bc2, cudaStream_t st);

// Simple temporal carrier over a token chunk (temporal.cu): rows token-major
// (row t*B + b) [N][h][d]; mstate [B][h][d] in/out.
struct TemporalArgs {
  int B, T, h, d;
  const float *W;
  size_t off_alog, off_wx, off_wout;
  const float *hstar;
  float *hist, *mstate;
};
cudaError_t launch_temporal_scan(const TemporalArgs &a, cudaStream_t st);

// FPM memory backward (fpm_bwd.cu).  Row-major [N][h][d] buffers, N = B*T
// tokens in the library's token-major order (row t*B + b); v is the adjoint
// solution [h][N][d]; the chunk
// arrays cA, cU, gin are [B][h][nch][d] with nch = ceil(T / fpm_chunk_len(d)).
struct FpmBwdArgs {
  int B, T, h, d, nch;
  const float *W;
  size_t off_bdelta, off_bret, off_wgate, off_bwrite, off_alog, off_wx;
  const float *hstar, *hist, *c, *rpre, *dpre, *v;
  float *minner;        // [N][h][d] memory after the write, rebuilt as the reference does
  float *cA, *cU, *gin; // chunk composites and entry values
  float *dm, *gpre;     // [N][h][d] dL/dM[t] and the retain-gate pre-activation gradient
  float *carry;         // [B][h][d] TBPTT carry, in: dL/dM seed, out: dL/dM before the chunk
  float *part;          // [5][B*nch][h][d] per-chunk partial sums
  float *part_bw;       // [B*nch][h]
  float *slot_prm;      // [h][5][d] per-slot parameters (launch_fpm_slot_params)
  int ch0, ch1;         // composite: chunk range [ch0, ch1) (ch1 = 0: all chunks)
};
int fpm_chunk_len(int d);
size_t fpm_chunk_smem(int d, bool full);
cudaError_t launch_fpm_c(const float *hstar, const float *signal, float *c, size_t n, cudaStream_t st);
cudaError_t launch_fpm_slot_params(const FpmBwdArgs &a, cudaStream_t st);
cudaError_t launch_fpm_composite(const FpmBwdArgs &a, cudaStream_t st);
cudaError_t launch_fpm_carry(const FpmBwdArgs &a, cudaStream_t st);
cudaError_t launch_fpm_chunks(const FpmBwdArgs &a, cudaStream_t st);
cudaError_t launch_fpm_finalize(const FpmBwdArgs &a, float *G, cudaStream_t st);

}  // namespace aideen
