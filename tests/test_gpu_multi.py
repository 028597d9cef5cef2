"""Two-GPU data parallelism through the C ABI: each rank computes its own
gradients, `aideen_allreduce_grads` sums them over NCCL, and every rank must
hold g_rank0 + g_rank1 afterwards.  Skipped when fewer than two GPUs are visible."""
import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

D, H, B, T, V = 128, 4, 2, 8, 61


def _rank(rank, uid, q):
    from aideen_b200.backend import GpuDeqBackend, RunConfig
    from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
    be = GpuDeqBackend(D, H, max_batch=B, max_seq_len=T, vocab=V, device=rank)
    be.upload_weights(init_all_weights(D, H, seed=5))
    be.upload_lm_head(*init_lm_head(D, V))
    be.upload_embedding(init_embedding(D, V))
    be.comm_init(uid, 2, rank)
    rng = np.random.default_rng(100 + rank)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    be.run_forward_tokens(tok, B, T, RunConfig(fpm=True))
    be.lm_head_loss(tg)
    be.run_staged_adjoint_picard_no_readback(0.85, 12)
    be.weight_grads()
    local = be.read_grads()
    be.allreduce_grads(timeout_ms=60000)
    summed = be.read_grads()
    q.put((rank, local, summed))
    be.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_gradient_allreduce_two_gpus():
    from aideen_b200.backend import GpuDeqBackend
    uid = GpuDeqBackend.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, uid, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict((r, (l, s)) for r, l, s in (q.get(timeout=300) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = out[0][0].astype(np.float64) + out[1][0]
    for r in range(2):
        got = out[r][1]
        assert np.linalg.norm(got - expect) / np.linalg.norm(expect) < 1e-6
    assert np.linalg.norm(out[0][0] - out[1][0]) > 0   # the ranks really saw different data


DP, HP, BP, TP = 128, 4, 4, 16   # the pipelined step's shape in the parity tests


def _rank_step(rank, uid, uid2, q):
    """One data-parallel training step per rank, through the pipelined path
    (where the LM-head gradients are summed on their own stream)."""
    from aideen_b200.backend import GpuDeqBackend, RunConfig
    from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
    rng = np.random.default_rng(200 + rank)
    tok = rng.integers(0, V, (BP, TP)).astype(np.int32)
    tg = rng.integers(0, V, (BP, TP)).astype(np.int32)
    import os
    res = {}
    for dp in (False, True, "sharded"):
        # the gradient sum is read back from the plain allreduce; the default
        # sharded update must give the same weights
        if dp is True:
            os.environ["AIDEEN_NO_SHARDED_UPDATE"] = "1"
        else:
            os.environ.pop("AIDEEN_NO_SHARDED_UPDATE", None)
        be = GpuDeqBackend(DP, HP, max_batch=BP, max_seq_len=TP, vocab=V, device=rank)
        be.upload_weights(init_all_weights(DP, HP, seed=6))
        be.upload_lm_head(*init_lm_head(DP, V))
        be.upload_embedding(init_embedding(DP, V))
        if dp:
            be.comm_init(uid if dp is True else uid2, 2, rank)
        be.train_step(tok, tg, BP, TP, RunConfig(fpm=True), adj_iters=12, lr=1e-3, step=1,
                      allreduce=bool(dp), grad_scale=0.5 if dp else 1.0)
        res[dp] = (be.read("lm_grads", (V * DP + V + DP,)), be.read_grads(), be.read_weights())
        be.close()
    q.put((rank, res[False][0], res[False][1], res[True], res["sharded"][2]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_pipelined_train_step_two_gpus_sums_all_gradients():
    from aideen_b200.backend import GpuDeqBackend
    uid, uid2 = GpuDeqBackend.comm_unique_id(), GpuDeqBackend.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_step, args=(r, uid, uid2, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {r: rest for r, *rest in (q.get(timeout=300) for _ in range(2))}
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    lm_sum = out[0][0].astype(np.float64) + out[1][0]
    g_sum = out[0][1].astype(np.float64) + out[1][1]
    for r in range(2):
        lm, g, w = out[r][2]
        assert np.linalg.norm(lm - lm_sum) / np.linalg.norm(lm_sum) < 1e-6
        assert np.linalg.norm(g - g_sum) / np.linalg.norm(g_sum) < 1e-6
    assert np.array_equal(out[0][2][2], out[1][2][2])   # identical update on both ranks
    # the sharded update (reduce-scatter, Adam per shard, all-gather) gives the same weights
    for r in range(2):
        np.testing.assert_allclose(out[r][3], out[r][2][2], rtol=0, atol=1e-6)


DR, HR, BR, TR, VR, NSR = 128, 4, 2, 16, 97, 24   # the reference-step case


def _rank_ref_step(rank, uid, q):
    """The reference's full step (sampled LM head, embedding update) on two ranks:
    the sampled set comes from both ranks' targets, the sampled-row and core
    gradients are summed, the embedding rows use both ranks' positions."""
    from aideen_b200.backend import GpuDeqBackend, RunConfig
    from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
    rng = np.random.default_rng(300 + rank)
    tok = rng.integers(0, VR, (BR, TR)).astype(np.int32)
    tg = rng.integers(0, VR, (BR, TR)).astype(np.int32)
    be = GpuDeqBackend(DR, HR, max_batch=BR, max_seq_len=TR, vocab=VR, device=rank)
    be.upload_weights(init_all_weights(DR, HR, seed=7))
    be.upload_lm_head(*init_lm_head(DR, VR))
    be.upload_embedding(init_embedding(DR, VR))
    import os
    os.environ["AIDEEN_NO_SHARDED_UPDATE"] = "1"   # the summed gradients stay readable
    be.comm_init(uid, 2, rank)
    loss = be.train_step(tok, tg, BR, TR, RunConfig(fpm=True), adj_iters=12, lr=1e-3, step=1,
                         allreduce=True, grad_scale=1.0, lm_samples=NSR, emb_update=1)
    os.environ.pop("AIDEEN_NO_SHARDED_UPDATE")
    out = dict(tok=tok, tg=tg, loss=loss, grads=be.read_grads(), W=be.read_weights(),
               lm=be.read_lm_head(), emb=be.read_embedding(), dl=be.read("dl_dh", (BR * TR, DR)),
               lmg=be.read("lm_grads", (VR * DR + VR + DR,)))
    q.put((rank, out))
    be.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_reference_step_two_gpus_matches_the_union_batch():
    from aideen_b200.backend import GpuDeqBackend
    from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
    from oracle import deq_oracle as O
    uid = GpuDeqBackend.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_ref_step, args=(r, uid, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = out[0], out[1]
    # every rank applies the same update
    assert np.array_equal(a["W"], b["W"])
    assert all(np.array_equal(x, y) for x, y in zip(a["lm"], b["lm"]))
    assert np.array_equal(a["emb"], b["emb"])
    # and it is the single-process step on the union batch
    W = init_all_weights(DR, HR, seed=7)
    lm, emb = init_lm_head(DR, VR), init_embedding(DR, VR)
    tok = np.concatenate([a["tok"], b["tok"]])
    tg = np.concatenate([a["tg"], b["tg"]])
    cfg = O.Cfg(d=DR, h=HR, fpm=True, max_iters=12, adj_iters=12)
    r = O.train_step(emb[tok], tg, W, lm, cfg, lm_samples=NSR, tokens=tok, emb=emb)
    rel = lambda x, y: np.linalg.norm(np.asarray(x, np.float64) - y) / np.linalg.norm(y)
    assert rel(a["grads"], r["grads"]) < 1e-3
    K = len(r["sampled"])
    assert rel(a["lmg"][:K * DR].reshape(K, DR), r["lm_grads"][0]) < 1e-3
    dl = np.concatenate([a["dl"], b["dl"]])
    assert rel(dl, r["dP"]) < 1e-3
    # the Adam kernels on the GPU's own (summed) gradients
    Wk, _, _ = O.adam(W, a["grads"].astype(np.float64), np.zeros_like(W, np.float64), np.zeros_like(W, np.float64), 1)
    assert rel(a["W"].astype(np.float64) - W, Wk.astype(np.float32).astype(np.float64) - W) < 1e-4
    st = dict(m=np.zeros((VR, DR)), v=np.zeros((VR, DR)))
    ek = O.embedding_update(emb, tok.reshape(-1), dl, st, 1)
    assert rel(a["emb"].astype(np.float64) - emb, ek.astype(np.float32).astype(np.float64) - emb) < 1e-4


def _rank_leaver(rank, uid, q, gone):
    """Rank 1 takes part in one gradient sum, then leaves between steps (its
    context and communicator are destroyed, no collective in flight).  Rank 0's
    next sum must come back as AIDEEN_E_TIMEOUT from the host-side deadline,
    with the communicator aborted and the context still usable."""
    import os
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from aideen_b200.backend import AideenError, GpuDeqBackend, RunConfig
    from aideen_b200.weights import init_all_weights
    be = GpuDeqBackend(D, H, max_batch=B, max_seq_len=T, device=rank)
    be.upload_weights(init_all_weights(D, H, seed=5))
    be.comm_init(uid, 2, rank)
    S = np.random.default_rng(rank).uniform(-1, 1, (B, T, D)).astype(np.float32)
    be.run_forward_deq_no_readback(S, B, T, RunConfig())
    be.run_staged_adjoint_picard_no_readback(0.85, 4, dl_dh=np.ones((B * T, D), np.float32))
    be.weight_grads()
    be.allreduce_grads(timeout_ms=60000)      # both ranks: a normal step
    be.sync()
    if rank == 1:
        be.close()
        gone.set()
        q.put((rank, "left"))
        return
    gone.wait(timeout=120)
    status = None
    try:
        be.allreduce_grads(timeout_ms=2000)
    except AideenError as e:
        status = str(e)
    # the context survives without its communicator: a local forward still runs
    be.run_forward_deq_no_readback(S, B, T, RunConfig())
    hs = be.read_hnext_seq()
    q.put((rank, (status, bool(np.isfinite(hs).all()))))
    be.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_rank_that_leaves_times_out_the_next_gradient_sum():
    from aideen_b200.backend import GpuDeqBackend
    uid = GpuDeqBackend.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gone = ctx.Event()
    ps = [ctx.Process(target=_rank_leaver, args=(r, uid, q, gone)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    status, finite = out[0]
    assert status is not None and "status 4" in status, status
    assert finite
