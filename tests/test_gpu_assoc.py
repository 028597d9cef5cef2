"""The associative branch of the upper slots (AIDEEN_CFG_ASSOC) against the
oracle's restatement (oracle/deq_oracle.py: assoc_read, assoc_write), through
the C ABI: the forward over two calls (the bank state carried from the first
to the second, where the bank is occupied and no longer written) and whole
training steps.  Tolerance 1e-3 relative L2, iteration counts equal.
"""
import numpy as np
import pytest

from oracle import deq_oracle as O
from aideen_b200.backend import GpuDeqBackend, RunConfig
from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head
from parity_util import TOL, assert_step, rel, step_errors

pytestmark = pytest.mark.gpu

CASES = [dict(d=128, h=4, B=2, T=8), dict(d=512, h=8, B=2, T=6), dict(d=256, h=3, B=1, T=7)]


@pytest.mark.parametrize("c", CASES, ids=lambda c: f"d{c['d']}h{c['h']}")
def test_assoc_forward_parity_over_two_calls(c):
    d, h, B, T = c["d"], c["h"], c["B"], c["T"]
    W = init_all_weights(d, h, seed=5)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, assoc=True)
    be.upload_weights(W)
    rng = np.random.default_rng(11)
    S1 = rng.uniform(-1, 1, (B, T, d)).astype(np.float32)
    S2 = rng.uniform(-1, 1, (B, T, d)).astype(np.float32)
    rc = RunConfig(max_iters=12, fpm=True)
    cfg = O.Cfg(d=d, h=h, max_iters=12, fpm=True, assoc=True)
    ref = None
    for S in (S1, S2):
        st = be.run_forward_deq_no_readback(S, B, T, rc, stats=True)
        ref = O.forward(S, W, cfg, mstate=None if ref is None else ref.mstate,
                        assoc_state=None if ref is None else ref.assoc_state)
        it = be.read("iters", (B, T, h), np.int32)
        assert (it != ref.iters).mean() == 0.0
        assert rel(be.read_hnext_seq(), ref.hstar) < TOL
        assert rel(be.read("hist_ctx", (B, T, h, d)), ref.hist_ctx) < TOL
        assert rel(be.read("fpm_ctx", (B, T, h, d)), ref.fpm_ctx) < TOL
        assert rel(be.read("mstate", (B, h, d)), ref.mstate) < TOL
        pre = ref.hstar + O.branch_of(ref, W, cfg)
        assert rel(be.read("pre", (B, T, h, d)), pre) < TOL
        assert st.total_iters == int(ref.iters.sum()) and st.nonfinite == 0
    # the branch acted: the upper slots' memory is the consolidation only
    up = slice(h // 2, h)
    assert np.abs(ref.hist_ctx[:, :, up]).max() > 0
    # a state reset clears the banks: the first call's result comes back
    be.reset_state()
    be.run_forward_deq_no_readback(S1, B, T, rc)
    ref1 = O.forward(S1, W, cfg)
    assert rel(be.read_hnext_seq(), ref1.hstar) < TOL
    assert rel(be.read("hist_ctx", (B, T, h, d)), ref1.hist_ctx) < TOL
    be.close()


@pytest.mark.parametrize("c", [dict(d=128, h=4, B=2, T=8), dict(d=512, h=8, B=4, T=8)],
                         ids=["d128h4", "d512h8B4"])
def test_assoc_train_step_parity(c):
    """A whole step with the dense LM head: the adjoint linearises the payload
    branch of the upper slots, W_in and S_in receive their direct term from the
    lower slots only, the FPM backward reads the stored signal, and alpha_assoc
    gets the reference's gradient."""
    d, h, B, T, V = c["d"], c["h"], c["B"], c["T"], 61
    W = init_all_weights(d, h, seed=6)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V, assoc=True)
    be.upload_weights(W)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rng = np.random.default_rng(12)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    rc = RunConfig(max_iters=12, fpm=True)
    loss = be.train_step(tok, tg, B, T, rc, adj_iters=12, lr=1e-3, step=1)
    cfg = O.Cfg(d=d, h=h, max_iters=12, fpm=True, assoc=True, adj_iters=12)
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    assert_step(step_errors(be, r, W, lm, B, T), loss, r)
    # the reference's alpha_assoc gradient (upper slots; zero below)
    L = O.Offsets(d, h)
    ga = be.read_grads()[L.alpha_assoc:L.alpha_assoc + h]
    assert rel(ga, r["grads"][L.alpha_assoc:L.alpha_assoc + h]) < TOL and not ga[: h // 2].any()
    be.close()


def test_assoc_flag_needs_two_slots():
    from aideen_b200.backend import AideenError
    with pytest.raises(AideenError):
        GpuDeqBackend(128, 1, max_batch=1, max_seq_len=4, assoc=True)
