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
from parity_util import assert_step, step_errors

pytestmark = pytest.mark.gpu


def _run(d, h, B, T, V, tok, tg, max_iters, adj_iters, anderson_m, fpm=True, seed=0):
    W = init_all_weights(d, h, seed=seed)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V)
    be.upload_weights(W)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rc = RunConfig(max_iters=max_iters, fpm=fpm)
    loss = be.train_step(tok, tg, B, T, rc, adj_iters=adj_iters, anderson_m=anderson_m, lr=1e-3, step=1)
    cfg = O.Cfg(d=d, h=h, fpm=fpm, max_iters=max_iters, adj_iters=adj_iters, anderson_m=anderson_m)
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
