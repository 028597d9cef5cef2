"""Whole training steps through `aideen_train_step` against the oracle at the
shapes BASELINE.json names: configs[0] exactly, the per-GPU shard of
configs[2] that bench.py times (pipelined schedule, vocab 50257, Zipf ids,
Anderson adjoint), and a d_model 1024 / 16-slot step at configs[4]'s width.

Bar: 1e-3 relative L2 on loss, h*, pooled state, dL/dh, the adjoint v and every
gradient block, identical Picard iteration counts (see parity_util for the
split check of the Adam update).
"""
import os

import numpy as np
import pytest

from oracle import deq_oracle as O
from aideen_b200.backend import GpuDeqBackend, RunConfig
from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head, zipf_tokens
from parity_util import assert_step, rel, step_errors

pytestmark = pytest.mark.gpu


def _run(d, h, B, T, V, tok, tg, max_iters, adj_iters, anderson_m, fpm=True, seed=0, fwd_m=0):
    W = init_all_weights(d, h, seed=seed)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V)
    be.upload_weights(W)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rc = RunConfig(max_iters=max_iters, fpm=fpm, anderson_m=fwd_m)
    loss = be.train_step(tok, tg, B, T, rc, adj_iters=adj_iters, anderson_m=anderson_m, lr=1e-3, step=1)
    cfg = O.Cfg(d=d, h=h, fpm=fpm, max_iters=max_iters, adj_iters=adj_iters, anderson_m=anderson_m,
                fwd_anderson_m=fwd_m)
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    e = step_errors(be, r, W, lm, B, T)
    be.close()
    print({k: f"{v:.2e}" for k, v in e.items()})
    return loss, r, e


def test_configs0_tiny_char_lm_step():
    """vocab 65, d_r 128, h 4, ctx 64, batch 1, uniform ids, Picard
    max 12 / tol 1e-4, adjoint 12 iterations, one Adam step (lr 1e-3)."""
    V, B, T = 65, 1, 64
    rng = np.random.default_rng(0)
    ids = rng.integers(0, V, (B, T + 1)).astype(np.int32)
    loss, r, e = _run(128, 4, B, T, V, ids[:, :-1].copy(), ids[:, 1:].copy(), 12, 12, 0)
    assert_step(e, loss, r)


def test_configs1_single_sequence_anderson_forward_step():
    """vocab 50257, d_r 512, h 8, ctx 256, batch 1, Zipf(1.1) ids,
    Anderson-accelerated Picard forward (max 20 iterations, tol 1e-4), Picard
    adjoint (Anderson m=4, 12 iterations), Adam."""
    V, B, T = 50257, 1, 256
    ids = zipf_tokens(B * (T + 1), V, seed=5).reshape(B, T + 1)
    loss, r, e = _run(512, 8, B, T, V, ids[:, :-1].copy(), ids[:, 1:].copy(), 20, 12, 4, fwd_m=3)
    assert_step(e, loss, r)


def test_bench_shard_pipelined_step():
    """The per-GPU shard bench.py times (configs[2] at 8 GPUs): d 512, h 8,
    8 sequences x 256 tokens, vocab 50257, Zipf(1.1) ids, Picard max 20,
    12 adjoint iterations with Anderson m=4, through the pipelined schedule
    (three Picard token chunks on 16-token boundaries, the LM head and adjoint
    of finished chunks overlapped)."""
    assert "AIDEEN_NO_PIPELINE" not in os.environ
    V, B, T = 50257, 8, 256
    ids = zipf_tokens(B * (T + 1), V, seed=3).reshape(B, T + 1)
    loss, r, e = _run(512, 8, B, T, V, ids[:, :-1].copy(), ids[:, 1:].copy(), 20, 12, 4)
    assert_step(e, loss, r)


def test_d1024_h16_step():
    """configs[4]'s width (d_r 1024, 16 slots) on a short context: memory path
    at d 1024, Anderson adjoint over 16 slots."""
    V, B, T = 257, 2, 12
    ids = zipf_tokens(B * (T + 1), V, seed=4).reshape(B, T + 1)
    loss, r, e = _run(1024, 16, B, T, V, ids[:, :-1].copy(), ids[:, 1:].copy(), 30, 30, 4)
    assert_step(e, loss, r)


def _reference_step(d, h, B, T, V, ns, fwd_m=0, max_iters=20, adj=12, am=4, emb_src=1, step=1, assoc=False):
    """The reference's full step: sampled-softmax LM head with its own Adam step,
    DEQ core Adam, embedding rows updated from dL/dpooled (emb_src 1) or the
    exact dL/dS_in (emb_src 2); assoc: the associative branch on the upper slots
    (the reference's default runtime, as bench.py runs it)."""
    ids = zipf_tokens(B * (T + 1), V, seed=11).reshape(B, T + 1)
    tok, tg = ids[:, :-1].copy(), ids[:, 1:].copy()
    tg[0, 1] = -1                                    # an ignored target
    W = init_all_weights(d, h, seed=0)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V, assoc=assoc)
    be.upload_weights(W)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rc = RunConfig(max_iters=max_iters, fpm=True, anderson_m=fwd_m)
    loss = be.train_step(tok, tg, B, T, rc, adj_iters=adj, anderson_m=am, lr=1e-3, step=step,
                         lm_samples=ns, emb_update=emb_src)
    cfg = O.Cfg(d=d, h=h, fpm=True, max_iters=max_iters, adj_iters=adj, anderson_m=am, fwd_anderson_m=fwd_m,
                assoc=assoc)
    r = O.train_step(emb[tok], tg, W, lm, cfg, step=step, lm_samples=ns, tokens=tok, emb=emb,
                     emb_grad="dl_dh" if emb_src == 1 else "ds_in")
    N = B * T
    e = {}
    S = r["sampled"]
    K = len(S)
    e["S_equal"] = float(np.array_equal(be.read("lm_samples", (K,), np.int32), S))
    e["loss"] = abs(loss - r["loss"]) / abs(r["loss"])
    e["hstar"] = rel(be.read_hnext_seq(), r["fwd"].hstar)
    e["iters_mismatch"] = float((be.read("iters", (B, T, h), np.int32) != r["fwd"].iters).mean())
    dl = be.read("dl_dh", (N, d))
    e["dl_dh"] = rel(dl, r["dP"])
    e["v"] = rel(np.transpose(be.read_adj_v_out(), (1, 0, 2)), r["v"])
    Gg = be.read_grads()
    e["core_grads"] = rel(Gg, r["grads"])
    lg = be.read("lm_grads", (V * d + V + d,))
    dW_s, db_s = r["lm_grads"]
    e["dW_sampled"] = rel(lg[:K * d].reshape(K, d), dW_s)
    e["db_sampled"] = rel(lg[V * d:V * d + K], db_s)
    # the sampled-row Adam kernel on the GPU's own gradients (fp32 rounding only)
    lw, lb, _ = be.read_lm_head()
    w0 = np.asarray(lm[0], np.float64)
    gk = np.clip(lg[:K * d].reshape(K, d).astype(np.float64), -0.1, 0.1)
    wk = w0[S] - 1e-3 * gk / (np.abs(gk) + 1e-8)
    e["lm_adam_kernel"] = rel(lw[S].astype(np.float64) - w0[S], wk.astype(np.float32).astype(np.float64) - w0[S])
    untouched = np.setdiff1d(np.arange(V), S)
    e["lm_untouched"] = float(np.abs(lw[untouched] - lm[0][untouched]).max())
    # embedding: the Adam kernel on the GPU's gradient rows, and those rows
    em = be.read_embedding()
    src = dl if emb_src == 1 else be.read("ds_in", (N, d))
    st = dict(m=np.zeros((V, d)), v=np.zeros((V, d)))
    ek = O.embedding_update(emb, tok.reshape(N), src, st, step, lr=1e-3)
    e["emb_adam_kernel"] = rel(em.astype(np.float64) - emb, ek.astype(np.float32).astype(np.float64) - emb)
    be.close()
    print({k: f"{v:.2e}" for k, v in e.items()})
    return e


@pytest.mark.parametrize("shape,assoc", [((128, 4, 2, 16, 97, 32), False), ((512, 8, 8, 256, 50257, 512), False),
                                         ((512, 8, 8, 256, 50257, 512), True)],
                         ids=["small", "bench_shard", "bench_shard_assoc"])
def test_reference_full_step_sampled_lm_and_embedding(shape, assoc):
    e = _reference_step(*shape, assoc=assoc)
    assert e["S_equal"] == 1.0 and e["iters_mismatch"] == 0.0 and e["lm_untouched"] == 0.0
    for k in ("loss", "hstar", "dl_dh", "v", "core_grads", "dW_sampled", "db_sampled"):
        assert e[k] < 1e-3, (k, e)
    assert e["lm_adam_kernel"] < 1e-4 and e["emb_adam_kernel"] < 1e-4, e


def test_reference_step_exact_embedding_gradient():
    e = _reference_step(128, 4, 2, 16, 97, 32, emb_src=2)
    assert e["emb_adam_kernel"] < 1e-4 and e["core_grads"] < 1e-3, e
