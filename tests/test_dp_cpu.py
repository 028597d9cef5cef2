"""Data-parallel decomposition on CPU ranks (gloo, world size 2).

Each rank takes its own sequences, computes the oracle's gradients, sums them
with an allreduce and scales by 1/world (what `aideen_apply_update` does with
grad_scale = 1/world after `aideen_allreduce_grads`); the result must equal the
single-process gradient of the whole batch.  A rank that never joins must
surface as a host-side timeout, not a hang.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import deq_oracle as O
from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head

D, H, T, V = 16, 3, 4, 13


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case():
    W = init_all_weights(D, H, seed=11)
    lm = init_lm_head(D, V, seed=12)
    emb = init_embedding(D, V, seed=13)
    rng = np.random.default_rng(14)
    tok = rng.integers(0, V, (2, T))
    tg = rng.integers(0, V, (2, T))
    return W, lm, emb, tok, tg


def _rank(rank, world, port, out, assoc=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    W, lm, emb, tok, tg = _case()
    cfg = O.Cfg(d=D, h=H, max_iters=12, adj_iters=30, fpm=True, assoc=assoc)
    r = O.train_step(emb[tok[rank:rank + 1]], tg[rank:rank + 1], W, lm, cfg)
    g = torch.from_numpy(np.concatenate([r["grads"], r["lm_grads"]]))
    dist.all_reduce(g)
    g /= world
    if rank == 0:
        out.put(g.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("assoc", [False, True], ids=["fpm", "fpm_assoc"])
def test_allreduced_shard_gradients_equal_full_batch_gradient(assoc):
    """assoc: the associative branch of the upper slots keeps per-sequence state
    only (banks, previous source), so it shards like the FPM memory."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, assoc)) for r in range(2)]
    for p in ps:
        p.start()
    g_dp = q.get(timeout=240)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    W, lm, emb, tok, tg = _case()
    # full batch: mean over both sequences' tokens.  With per-sequence FPM memory
    # and equal shard sizes, the mean of the shard means is the global mean.
    cfg = O.Cfg(d=D, h=H, max_iters=12, adj_iters=30, fpm=True, assoc=assoc)
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    g_full = np.concatenate([r["grads"], r["lm_grads"]])
    err = np.linalg.norm(g_dp - g_full) / np.linalg.norm(g_full)
    assert err < 1e-9, err


def _lonely_rank(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # the missing peer shows up as an error on the host
        q.put(type(e).__name__)


def test_rank_that_never_joins_times_out_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=30)
    assert res != "joined"
