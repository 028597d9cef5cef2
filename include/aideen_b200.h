/*
 * aideen_b200 — C ABI of the B200-native AIDEEN DEQ training hot path.
 *
 * Drop-in boundary for the reference's `GpuDeqBackend`
 * (aideen-backbone/src/gpu_deq.rs:80-218) wrapping `RustDeqBridge`
 * (aideen-block/src/deq_bridge.rs:55-101).  Plain pointers and sizes only; no
 * torch and no CUDA types in the signatures (streams are passed as void*).
 *
 * Ownership: the context owns every device buffer, sized at create time from
 * the caps in `aideen_cfg` (the reference sizes its wgpu buffers from
 * `forward_seq_cap/forward_batch_cap`, gpu_deq.rs:82-83).  Caller memory is
 * only read or written during the call.  Pointers flagged AIDEEN_DEVICE are
 * device pointers on the context's device, ordered on the context's stream.
 *
 * Errors: every call returns an `aideen_status`; `aideen_last_error` gives the
 * message.  No call aborts the process.  A context is single-thread affine.
 *
 * Layouts (identical to the reference so its trainer needs no change):
 *   AllWeights   deq_bridge.rs:103-137 (+ HistParams gpu_deq.rs:260-422)
 *   S_in         [B*T][d]               token-major
 *   H* / HistCtx [B*T][h][d]            deq_slot_attn_unified_clean.wgsl:712
 *   MState       [B][h][d]
 *   dl_dh        [B*T][d]
 *   adjoint v    [h][B*T][d] slot-major staged_adjoint_picard_clean.wgsl:57-67
 */
#ifndef AIDEEN_B200_H
#define AIDEEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum aideen_status {
  AIDEEN_OK = 0,
  AIDEEN_E_INVALID = 1,   /* bad argument / size beyond caps */
  AIDEEN_E_CUDA = 2,      /* CUDA runtime failure */
  AIDEEN_E_NCCL = 3,      /* collective failure */
  AIDEEN_E_TIMEOUT = 4,   /* bounded wait ran out */
  AIDEEN_E_NONFINITE = 5, /* non-finite value detected in a checked buffer */
  AIDEEN_E_UNSUPPORTED = 6
} aideen_status;

enum { AIDEEN_HOST = 0, AIDEEN_DEVICE = 1 };

/* Construction caps + static architecture (ArchitectureConfig,
 * aideen-core/src/state.rs:7-58).  d_model in {128, 256, 512, 1024};
 * h_slots in [1, 16]. */
typedef struct aideen_cfg {
  uint32_t d_model;
  uint32_t h_slots;
  uint32_t max_batch;    /* forward_batch_cap */
  uint32_t max_seq_len;  /* forward_seq_cap */
  uint32_t vocab;        /* LM head / embedding rows; 0 = no LM head */
  uint32_t flags;        /* AIDEEN_CFG_* bits; 0 = none */
} aideen_cfg;
/* flags bit 0: with the FPM memory on, the upper h/2 slots run the reference's
 * default associative branch (deq_slot_attn_unified_clean.wgsl:554-556, on at
 * FPM stage 4) in place of the FPM write: a one-bank hard read added to the
 * memory context, a single bank write per empty bank, a 0.019 consolidation of
 * h* into the slot's memory, and the payload as the slot's stored signal (the
 * adjoint's branch and the FPM backward read it).  Of its own parameters,
 * alpha_assoc gets the reference's gradient (fused_fpm_retain_bwd.wgsl:1129-1160,
 * 1281-1284); under these default flags the reference's terms for the address,
 * value and event weights are exactly zero (one bank, event gate off), and so
 * are they here.  The bank state is carried across calls and cleared by
 * aideen_reset_state.  Needs h_slots >= 2. */
#define AIDEEN_CFG_ASSOC 1u

/* One forward dispatch (RunUniforms, deq_slot_attn_unified_clean.wgsl:1-21;
 * DeqComputeShape, deq_bridge.rs:4-25). */
typedef struct aideen_run {
  uint32_t batch;
  uint32_t seq_len;
  uint32_t max_iters;
  float epsilon;
  float damping;          /* Picard blend of the generic path; adjoint beta */
  uint32_t slot_coord;    /* 1 = iter-0 slot attention on (residual_alpha = -1) */
  uint32_t fpm;           /* 1 = FPM memory read/inject/write (Model A) */
  float fpm_alpha_m;
  float fpm_tau;
  float fpm_read_gate_min;
  /* Anderson acceleration of each (sequence, slot) Picard solve (no
   * counterpart in the reference forward): 0 or 1 = plain Picard; 2 or 3 =
   * type-II Anderson over the last 2 or 3 residuals f = G(h) - h of the slot's
   * d-vector, from the third iteration on (the residuals of iterations >= 1,
   * whose map is fixed within the token).  The stop rule is unchanged. */
  uint32_t anderson_m;
} aideen_run;

/* Forward convergence statistics (DebugLog[13..17] equivalents). */
typedef struct aideen_stats {
  uint64_t total_iters;   /* summed over (b, t, slot) */
  uint32_t max_iters_seen;
  uint32_t unconverged;   /* solves that ran to max_iters */
  uint32_t nonfinite;     /* (token, slot) rows of h* holding a non-finite value */
  uint32_t solves;        /* B*T*h */
} aideen_stats;

/* Adjoint call (run_staged_adjoint_picard_no_readback, gpu_deq.rs:4080). */
typedef struct aideen_adjoint_args {
  uint32_t batch;
  uint32_t seq_len;
  uint32_t iters;         /* fixed count, no early exit (gpu_deq.rs:4879) */
  float damping;
  uint32_t anderson_m;    /* 0 = off, else ring depth (<= 4) */
} aideen_adjoint_args;

/* Fused update (apply_fused_deq_update gpu_deq.rs:4980; apply_gradient_update :5509). */
enum { AIDEEN_RULE_ADAM = 0, AIDEEN_RULE_CLIPPED_SGD = 1 };
typedef struct aideen_update {
  uint32_t rule;
  float lr;
  float beta1, beta2, eps;   /* Adam (optimizer.rs:105-183) */
  float weight_decay;        /* clipped SGD main-weight decay */
  float grad_scale;          /* multiplies the gradient before the rule */
  uint32_t step;             /* Adam step t (>= 1) */
  uint32_t allreduce;        /* 1 = sum gradients over the communicator first */
  uint32_t update_lm_head;   /* 1 = also apply the rule to the LM head */
} aideen_update;

typedef struct aideen_ctx aideen_ctx;

/* ---- lifecycle (GpuDeqBackend::new_blocking, gpu_deq.rs:3122) ---------- */
aideen_ctx *aideen_create(const aideen_cfg *cfg, int device, int *status);
void aideen_destroy(aideen_ctx *ctx);
const char *aideen_last_error(const aideen_ctx *ctx);
int aideen_set_stream(aideen_ctx *ctx, void *cuda_stream);
/* Make the context stream wait for work the library deferred to its side
 * stream (the LM-head update of the last apply, which otherwise overlaps the
 * next forward).  Stream-ordered, no host wait; aideen_sync and every read
 * of LM-head state do it implicitly. */
int aideen_join(aideen_ctx *ctx);
int aideen_sync(aideen_ctx *ctx);
/* Number of this library's own kernel launches issued since create. */
uint64_t aideen_launch_count(const aideen_ctx *ctx);

/* Per-kernel-class device time (no counterpart in the reference; the
 * reference's AIDEEN_*_PROFILE timers, gpu_deq.rs:212-217, are host wall
 * clocks).  When enabled, every launch is bracketed by CUDA events on the
 * context's stream; aideen_profile_read synchronises and returns cumulative
 * milliseconds and launch counts per class. */
/* Classes: Picard solve; adjoint; GEMMs of the slot projections and weight
 * gradients (the per-slot source-gradient GEMMs of aideen_weight_grads count
 * as "everything else"); every kernel of the LM head (its GEMMs, softmax, reductions, and
 * the sampled head's Adam step); the optimizer sweeps; the FPM backward (its
 * GEMMs included); everything else. */
enum { AIDEEN_PROF_PICARD = 0, AIDEEN_PROF_ADJOINT = 1, AIDEEN_PROF_GEMM = 2,
       AIDEEN_PROF_LM_SOFTMAX = 3, AIDEEN_PROF_OPTIMIZER = 4, AIDEEN_PROF_OTHER = 5,
       AIDEEN_PROF_FPM_BWD = 6, AIDEEN_PROF_CLASSES = 7 };
int aideen_profile(aideen_ctx *ctx, int enable);
int aideen_profile_read(aideen_ctx *ctx, float *ms /*[AIDEEN_PROF_CLASSES]*/, uint64_t *launches /*[AIDEEN_PROF_CLASSES], nullable*/,
                        int reset);

/* Length of AllWeights for (d, h) (deq_bridge.rs:103-137). */
size_t aideen_all_weights_len(uint32_t d_model, uint32_t h_slots);

/* ---- weights (upload_weights gpu_deq.rs:3529; read_weights :5595) -------- */
int aideen_upload_weights(aideen_ctx *ctx, const float *all_weights, size_t n, int where);
int aideen_download_weights(aideen_ctx *ctx, float *out, size_t n);
int aideen_download_grads(aideen_ctx *ctx, float *out, size_t n);
/* LM head W_lm [vocab][d], b_lm [vocab], g_lm [d] (lm_train.wgsl bindings 2, 3, 10). */
int aideen_upload_lm_head(aideen_ctx *ctx, const float *w_lm, const float *b_lm,
                          const float *g_lm);
int aideen_download_lm_head(aideen_ctx *ctx, float *w_lm, float *b_lm, float *g_lm);
int aideen_upload_embedding(aideen_ctx *ctx, const float *emb /*[vocab][d]*/);
/* Embedding table back to the host (GpuEmbeddingTrainer's weights readback,
 * gpu_embedding.rs weights_buffer). */
int aideen_download_embedding(aideen_ctx *ctx, float *emb /*[vocab][d]*/);
/* Adam moments for checkpoints (the reference's Adam::save_state / load_state,
 * optimizer.rs:246-325): DEQ core in the packed AllWeights layout (n_core =
 * aideen_all_weights_len) and the LM head as [vocab*d + vocab + d]; NULL
 * skips a part.  After data-parallel train steps every rank holds current
 * moments only for its own shard of the core (the sharded update). */
int aideen_download_adam(aideen_ctx *ctx, float *m_core, float *v_core, size_t n_core, float *m_lm, float *v_lm);
int aideen_upload_adam(aideen_ctx *ctx, const float *m_core, const float *v_core, size_t n_core,
                       const float *m_lm, const float *v_lm);
/* Zero the carried FPM memory MState (reset_state gpu_deq.rs:3127). */
int aideen_reset_state(aideen_ctx *ctx);
/* Zero the Adam moments of the DEQ core and LM head. */
int aideen_reset_optimizer(aideen_ctx *ctx);

/* ---- forward (run_forward_deq_no_readback gpu_deq.rs:3855;
 *      run_forward_from_seq_buf :3918) ------------------------------------ */
int aideen_forward(aideen_ctx *ctx, const aideen_run *run, const float *s_in, int where,
                   aideen_stats *stats /*nullable*/);
/* Token ids -> S_in by embedding gather, then the forward
 * (GpuEmbeddingTrainer::gather_only_to_sbuf, trainer.rs:2823). */
int aideen_forward_tokens(aideen_ctx *ctx, const aideen_run *run, const int32_t *tokens,
                          int where, aideen_stats *stats);

/* ---- LM head: dense CE + RMSNorm backward -> dl_dh (lm_train.wgsl:79-395).
 * Also leaves the LM-head gradients for aideen_apply_update. */
int aideen_lm_head_loss(aideen_ctx *ctx, uint32_t batch, uint32_t seq_len,
                        const int32_t *targets, int where, float *loss_out /*host*/);

/* ---- adjoint (run_staged_adjoint_picard_no_readback gpu_deq.rs:4080) ----
 * dl_dh: [B*T][d] pooled upstream gradient; NULL = the LM head's last dl_dh.
 * rhs_slot: optional [B*T][h][d] per-slot RHS added to dl_dh/h.
 * Linearises around the state of the last aideen_forward. */
int aideen_adjoint(aideen_ctx *ctx, const aideen_adjoint_args *args, const float *dl_dh,
                   const float *rhs_slot, int where);
/* Adjoint on caller-provided fixed point (isolated adjoint benchmark): pre =
 * branch + hstar, both [B*T][h][d] (branch = signal + attn*scale + anchor). */
int aideen_adjoint_on(aideen_ctx *ctx, const aideen_adjoint_args *args, const float *hstar,
                      const float *branch, const float *dl_dh, const float *rhs_slot,
                      int where);
/* ---- simple temporal carrier (temporal_step, fixed_point_memory_reasoning.rs:1455-1486;
 *      hist_v2_temporal_main, hist_v2_temporal.wgsl:40-110) ----------------
 * Token by token over a chunk of fixed points h* ([B*T][h][d], caller order;
 * NULL = the last forward's), starting from the carried MState:
 *   M_t = (I + W_out^T)(a*M_{t-1} + (1-a)*(1 + 0.5 tanh(diag W_x))*h_t/rms(h_t)),
 *   a = sigmoid(-a_log[slot]).
 * Leaves every M_t in the HIST_CTX buffer and the last one in MState (the FPM
 * memory scan's buffers; this is the reference's non-default simpler carrier). */
int aideen_temporal_scan(aideen_ctx *ctx, uint32_t batch, uint32_t seq_len, const float *hstar, int where);

/* reduce_clean_adjoint_to_source_grad_no_readback (gpu_deq.rs:4922):
 * out[B*T][d] = sum_s beta*J_norm^T v. */
int aideen_source_grad(aideen_ctx *ctx, float *out, int where);

/* ---- gradients + update (apply_fused_deq_update gpu_deq.rs:4980) -------- */
int aideen_weight_grads(aideen_ctx *ctx);
int aideen_apply_update(aideen_ctx *ctx, const aideen_update *upd);

/* ---- spectral renorm (renormalize_spectral gpu_deq.rs:5568) -------------- */
int aideen_renormalize_spectral(aideen_ctx *ctx, uint32_t n_iters, float attn_threshold,
                                float win_threshold, float fpm_threshold,
                                float wv_threshold, float wo_threshold,
                                float *sigmas_out /*nullable, 5h+2 host floats*/);

/* ---- whole training step (Trainer::apply_training_update_from_gpu_buffers,
 *      trainer.rs:2640): gather -> forward -> LM head -> adjoint -> grads ->
 *      [allreduce] -> update -> [renorm]. ----------------------------------- */
typedef struct aideen_step_args {
  aideen_run run;
  uint32_t adj_iters;
  uint32_t anderson_m;
  aideen_update update;
  uint32_t renorm;           /* 1 = spectral renorm after the update (reference thresholds) */
  /* LM head: 0 = dense full-vocabulary CE, its gradients in the common update;
   * > 0 = the reference's sampled softmax with this num_samples (ArchitectureConfig
   * default 512, state.rs:54): the step's sampled vocabulary (distinct targets
   * plus deterministic candidates, up to min(max(num_samples, B*T), vocab, 2048),
   * gpu_lm_head.rs:244-281), softmax over it, and its own Adam step on the
   * sampled rows with dW, db clamped to +-0.1 before dL/dh is formed from the
   * updated rows (lm_train.wgsl:79-395; g_lm is not trained). */
  uint32_t lm_samples;
  /* Embedding rows of the step's tokens: 0 = frozen; 1 = Adam on the mean
   * dL/dpooled row of each distinct token (the reference trainer's default
   * source, trainer.rs:3285-3289; embedding_train.wgsl:100-147); 2 = the same
   * from the exact dL/dS_in. */
  uint32_t emb_update;
  float emb_lr;              /* embedding learning rate (0 = update.lr) */
  uint64_t sample_seed;      /* 0 = the reference's default seed 0xA1DEEE5A4D5EED5E */
} aideen_step_args;
int aideen_train_step(aideen_ctx *ctx, const aideen_step_args *args, const int32_t *tokens,
                      const int32_t *targets, int where, float *loss_out /*host, nullable*/,
                      aideen_stats *stats /*nullable*/);

/* ---- readbacks (read_hnext_seq gpu_deq.rs:5842, read_hpooled_seq :5886,
 *      read_adj_v_out :5821, ...) ----------------------------------------- */
enum aideen_buf {
  AIDEEN_BUF_HSTAR = 0,     /* [N][h][d] */
  AIDEEN_BUF_POOLED = 1,    /* [N][d] */
  AIDEEN_BUF_SIGNAL = 2,    /* [N][h][d] */
  AIDEEN_BUF_ATTN = 3,      /* [N][h][d] attention injection attn*scale */
  AIDEEN_BUF_ITERS = 4,     /* [N][h] int32 */
  AIDEEN_BUF_ADJ_V = 5,     /* [h][N][d] */
  AIDEEN_BUF_GPRE = 6,      /* [N][h][d] beta*J_norm^T v */
  AIDEEN_BUF_DL_DH = 7,     /* [N][d] */
  AIDEEN_BUF_HIST_CTX = 8,  /* [N][h][d] */
  AIDEEN_BUF_MSTATE = 9,    /* [B][h][d] */
  AIDEEN_BUF_FPM_CTX = 10,  /* [N][h][d] */
  AIDEEN_BUF_ALPHA = 11,    /* [N][h][h] */
  AIDEEN_BUF_S_IN = 12,     /* [N][d] */
  AIDEEN_BUF_DS_IN = 13,    /* [N][d] exact dL/dS_in */
  AIDEEN_BUF_LM_GRADS = 14, /* [vocab*d + vocab + d] */
  AIDEEN_BUF_PRE = 15,      /* [N][h][d] pre = branch + h* of the adjoint */
  AIDEEN_BUF_FPM_DM = 16,   /* [N][h][d] dL/dM[t] of the last FPM backward (fpm_dm_buf) */
  AIDEEN_BUF_FPM_CARRY = 17, /* [max_batch][h][d] FPM TBPTT carry (tbptt_carry_buf) */
  AIDEEN_BUF_LM_SAMPLES = 18  /* int32 sampled vocabulary of the last sampled LM head, ascending
                               * (last_sampled_indices, gpu_lm_head.rs:2604); with it the
                               * LM_GRADS buffer holds the sampled rows' dW [K][d] and, at
                               * offset vocab*d, db [K] */
};
/* Copies the first n_elems elements (4 bytes each) of a buffer to host dst,
 * token rows in the caller's order (row b*T + t). */
int aideen_read(aideen_ctx *ctx, int which, void *dst, size_t n_elems);
/* Device pointer of a buffer (zero-copy consumers); NULL if absent.  After a
 * forward the token rows of activation buffers are in the library's
 * token-major order (row t*B + b), not the caller's. */
void *aideen_device_ptr(aideen_ctx *ctx, int which);

/* ---- allocation-free adjoint (no counterpart in the reference) -------------
 * For callers that cannot allocate device memory (allocators that forbid
 * cudaMalloc once start-up is over, embedders that own every byte of the
 * device, host code that must not take the allocator's lock on its latency
 * path): the same fused clean adjoint as aideen_adjoint_on, with no context
 * and no allocation.  All pointers are device pointers on the current device
 * and must be 16-byte aligned (AIDEEN_E_INVALID otherwise); layouts as
 * aideen_adjoint_on (hstar, branch, rhs_slot [N][h][d]; dl_dh [N][d] or NULL;
 * norm_scale [d]; v_out [h][N][d]; gpre_out [N][h][d]).  One CTA
 * double-buffers the staged inputs of a token in shared memory, so
 * 8 * h_slots * d_model * (2 + (rhs_slot != NULL)) bytes must fit in one
 * block's shared memory (227 KB on B200: h_slots * d_model <= 9600 with
 * rhs_slot, <= 14400 without, less with the anderson_m = 4 ring); larger
 * shapes return AIDEEN_E_INVALID.
 * ns_grad_out (nullable, [d]) receives sum over tokens and slots of
 * beta*v*pre/rms(pre), the NormScale gradient.  Its per-token partials live in
 * a fixed device array of 2^22 floats (16 MiB) that every GPU loading the
 * library holds until exit, so n_tokens * d_model must be <= 4194304 when
 * ns_grad_out is given (AIDEEN_E_INVALID otherwise).  The first call on a
 * device looks up that array's address; make that first call before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * (different streams, or several threads on one device) race.  Nothing in it
 * needs zeroing.  The call waits for its work on `stream` and returns
 * AIDEEN_E_TIMEOUT if a bounded wait of the kernel ran out (outputs invalid). */
int aideen_adjoint_noalloc(const float *hstar, const float *branch, const float *dl_dh,
                           const float *rhs_slot, const float *norm_scale, uint32_t n_tokens,
                           uint32_t h_slots, uint32_t d_model, uint32_t iters, float damping,
                           uint32_t anderson_m, float *v_out, float *gpre_out, float *ns_grad_out,
                           void *stream);

/* ---- diagnostics (no counterpart in the reference) --------------------------
 * Runs a tcgen05 3xTF32 GEMM and the CUDA-core fp32 GEMM on the same seeded
 * device operands (C = op(A) op(B), row-major, `batch` independent problems)
 * and reports the relative L2 difference and both kernel times (the tensor-core
 * time averaged over 10 back-to-back calls).  flags bit 0
 * selects the persistent kernel on pre-split (hi/lo) operands instead of the
 * in-kernel-split one.  Allocates its own temporaries. */
#define AIDEEN_SELFTEST_PRESPLIT 1
/* flags bit 1: single TF32 products (operands rounded to tf32) instead of 3xTF32 */
#define AIDEEN_SELFTEST_TF32 2
int aideen_gemm_selftest(aideen_ctx *ctx, int M, int N, int K, int batch, int trans_a, int trans_b,
                         int flags, float *rel_err, float *ms_tc, float *ms_simt);

/* ---- multi-GPU (one process per GPU; NCCL over NVLink) ----------------- */
#define AIDEEN_UNIQUE_ID_BYTES 128
int aideen_comm_unique_id(char out[AIDEEN_UNIQUE_ID_BYTES]);
int aideen_comm_init(aideen_ctx *ctx, const char id[AIDEEN_UNIQUE_ID_BYTES], int nranks,
                     int rank);
/* Sum-allreduce of the gradient buffers (DEQ core and LM head) over the
 * communicator; waits at most timeout_ms, then aborts the communicator and
 * returns AIDEEN_E_TIMEOUT. */
int aideen_allreduce_grads(aideen_ctx *ctx, int timeout_ms);

#ifdef __cplusplus
}
#endif
#endif /* AIDEEN_B200_H */
