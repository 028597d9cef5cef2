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


def _rank_step(rank, uid, q):
    """One data-parallel training step per rank, through the pipelined path
    (where the LM-head gradients are summed on their own stream)."""
    from aideen_b200.backend import GpuDeqBackend, RunConfig
    from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
    rng = np.random.default_rng(200 + rank)
    tok = rng.integers(0, V, (BP, TP)).astype(np.int32)
    tg = rng.integers(0, V, (BP, TP)).astype(np.int32)
    res = {}
    for dp in (False, True):
        be = GpuDeqBackend(DP, HP, max_batch=BP, max_seq_len=TP, vocab=V, device=rank)
        be.upload_weights(init_all_weights(DP, HP, seed=6))
        be.upload_lm_head(*init_lm_head(DP, V))
        be.upload_embedding(init_embedding(DP, V))
        if dp:
            be.comm_init(uid, 2, rank)
        be.train_step(tok, tg, BP, TP, RunConfig(fpm=True), adj_iters=12, lr=1e-3, step=1,
                      allreduce=dp, grad_scale=0.5 if dp else 1.0)
        res[dp] = (be.read("lm_grads", (V * DP + V + DP,)), be.read_grads(), be.read_weights())
        be.close()
    q.put((rank, res[False][0], res[False][1], res[True]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_pipelined_train_step_two_gpus_sums_all_gradients():
    from aideen_b200.backend import GpuDeqBackend
    uid = GpuDeqBackend.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_step, args=(r, uid, q)) for r in range(2)]
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
