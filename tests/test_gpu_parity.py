"""CUDA path vs the CPU oracle, through the C ABI (include/aideen_b200.h).

Tolerance: 1e-3 relative L2 (the bar BASELINE.json's north star sets for
loss, h*, the adjoint and every weight gradient); iteration counts equal.
"""
import numpy as np
import pytest

from oracle import deq_oracle as O
from aideen_b200.backend import GpuDeqBackend, RunConfig, RULE_ADAM, RULE_CLIPPED_SGD, AideenError
from aideen_b200.weights import init_all_weights, init_lm_head, init_embedding
from parity_util import assert_step, step_errors

pytestmark = pytest.mark.gpu
TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (nb if nb > 0 else 1.0)


CASES = [
    dict(d=128, h=4, B=2, T=16, fpm=False),
    dict(d=128, h=4, B=2, T=16, fpm=True),
    dict(d=256, h=3, B=1, T=9, fpm=True),
    dict(d=512, h=8, B=2, T=8, fpm=True),
    dict(d=512, h=8, B=1, T=8, fpm=False),
]


def _setup(c, vocab=0, seed=0):
    d, h, B, T = c["d"], c["h"], c["B"], c["T"]
    W = init_all_weights(d, h, seed=seed)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=vocab)
    be.upload_weights(W)
    S = np.random.default_rng(seed + 10).uniform(-1, 1, (B, T, d)).astype(np.float32)
    rc = RunConfig(max_iters=12, fpm=c["fpm"])
    cfg = O.Cfg(d=d, h=h, max_iters=12, fpm=c["fpm"])
    return W, be, S, rc, cfg


@pytest.mark.parametrize("c", CASES, ids=lambda c: f"d{c['d']}h{c['h']}fpm{int(c['fpm'])}")
def test_forward_parity(c):
    W, be, S, rc, cfg = _setup(c)
    B, T, h, d = c["B"], c["T"], c["h"], c["d"]
    st = be.run_forward_deq_no_readback(S, B, T, rc, stats=True)
    ref = O.forward(S, W, cfg)
    hs = be.read_hnext_seq()
    it = be.read("iters", (B, T, h), np.int32)
    assert rel(be.read("signal", (B, T, h, d)), ref.signal) < 1e-5
    assert rel(be.read("attn", (B, T, h, d)), ref.A) < 1e-4
    assert rel(hs, ref.hstar) < TOL
    mismatch = (it != ref.iters).mean()
    assert mismatch == 0.0, f"iteration counts differ on {mismatch:.3%} of solves"
    assert rel(be.read_hpooled_seq(), ref.pooled) < TOL
    if c["fpm"]:
        assert rel(be.read("hist_ctx", (B, T, h, d)), ref.hist_ctx) < TOL
        assert rel(be.read("mstate", (B, h, d)), ref.mstate) < TOL
        assert rel(be.read("fpm_ctx", (B, T, h, d)), ref.fpm_ctx) < TOL
    assert st.solves == B * T * h and st.nonfinite == 0
    assert st.total_iters == int(ref.iters.sum())
    be.close()


@pytest.mark.parametrize("m", [2, 3])
@pytest.mark.parametrize("c", [CASES[1], CASES[3], CASES[4]], ids=["d128fpm", "d512fpm", "d512"])
def test_forward_anderson_parity(c, m):
    """Anderson-accelerated forward (residual mixing per slot): same h*, same
    iteration counts as the oracle's restatement."""
    W, be, S, rc, cfg = _setup(c)
    B, T, h, d = c["B"], c["T"], c["h"], c["d"]
    rc.max_iters = cfg.max_iters = 20
    rc.anderson_m = cfg.fwd_anderson_m = m
    st = be.run_forward_deq_no_readback(S, B, T, rc, stats=True)
    ref = O.forward(S, W, cfg)
    it = be.read("iters", (B, T, h), np.int32)
    assert (it != ref.iters).mean() == 0.0
    assert rel(be.read_hnext_seq(), ref.hstar) < TOL
    if c["fpm"]:
        assert rel(be.read("hist_ctx", (B, T, h, d)), ref.hist_ctx) < TOL
    assert st.total_iters == int(ref.iters.sum())
    be.close()


def test_fpm_state_carries_across_chunks():
    c = dict(d=128, h=4, B=1, T=8, fpm=True)
    W, be, S, rc, cfg = _setup(c)
    be.run_forward_deq_no_readback(S, 1, 8, rc)
    ref1 = O.forward(S, W, cfg)
    be.run_forward_deq_no_readback(S, 1, 8, rc)   # second chunk starts from MState
    ref2 = O.forward(S, W, cfg, mstate=ref1.mstate)
    assert rel(be.read_hnext_seq(), ref2.hstar) < TOL
    be.reset_state()
    be.run_forward_deq_no_readback(S, 1, 8, rc)
    assert rel(be.read_hnext_seq(), ref1.hstar) < TOL
    be.close()


@pytest.mark.parametrize("m", [0, 4])
@pytest.mark.parametrize("c", [CASES[1], CASES[3]], ids=["d128", "d512"])
def test_adjoint_parity(c, m):
    W, be, S, rc, cfg = _setup(c)
    B, T, h, d = c["B"], c["T"], c["h"], c["d"]
    N = B * T
    be.run_forward_deq_no_readback(S, B, T, rc)
    ref = O.forward(S, W, cfg)
    dl = np.random.default_rng(3).standard_normal((N, d)).astype(np.float32)
    be.run_staged_adjoint_picard_no_readback(0.85, 12, dl_dh=dl, anderson_m=m)
    cfg.adj_iters, cfg.anderson_m = 12, m
    # adjoint linearises around the GPU's own h* (identical within TOL to the oracle's)
    hs = be.read_hnext_seq().reshape(N, h, d)
    br = O.branch_of(ref, W, cfg).reshape(N, h, d)
    v, g, pre, r = O.adjoint(hs, br, dl, O.View(W, d, h).NS, cfg)
    vg = be.read_adj_v_out()                      # [h][N][d]
    assert rel(np.transpose(vg, (1, 0, 2)), v) < TOL
    assert rel(be.read("gpre", (N, h, d)), g) < TOL
    assert rel(be.reduce_clean_adjoint_to_source_grad(), O.source_grad(g)) < TOL
    be.close()


def test_adjoint_on_per_slot_rhs():
    """Isolated adjoint on a given fixed point with a per-slot RHS (adjoint micro-benchmark shape)."""
    d, h, N = 512, 8, 64
    W = init_all_weights(d, h, seed=1)
    be = GpuDeqBackend(d, h, max_batch=1, max_seq_len=N)
    be.upload_weights(W)
    rng = np.random.default_rng(4)
    hs = rng.standard_normal((N, h, d)).astype(np.float32)
    br = rng.standard_normal((N, h, d)).astype(np.float32)
    rs = rng.standard_normal((N, h, d)).astype(np.float32)
    be.run_adjoint_on(hs, br, 1, N, 0.85, 20, rhs_slot=rs)
    cfg = O.Cfg(d=d, h=h, adj_iters=20)
    v, g, _, _ = O.adjoint(hs, br, None, O.View(W, d, h).NS, cfg, rhs_slot=rs)
    assert rel(np.transpose(be.read_adj_v_out(), (1, 0, 2)), v) < TOL
    be.close()


@pytest.mark.parametrize("c", [CASES[1], CASES[3], CASES[4]], ids=["d128fpm", "d512fpm", "d512"])
def test_full_step_gradients_and_update(c):
    d, h, B, T = c["d"], c["h"], c["B"], c["T"]
    V = 97
    W, be, S, rc, cfg = _setup(c, vocab=V)
    lm = init_lm_head(d, V)
    emb = init_embedding(d, V)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rng = np.random.default_rng(5)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    tg[0, 1] = -1                                   # ignored target
    N = B * T
    be.run_forward_tokens(tok, B, T, rc)
    loss = be.lm_head_loss(tg)
    be.run_staged_adjoint_picard_no_readback(0.85, 12)
    be.weight_grads()
    Gg = be.read_grads()
    cfg.adj_iters = 12
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    assert abs(loss - r["loss"]) / abs(r["loss"]) < TOL
    assert rel(be.read("dl_dh", (N, d)), r["dP"]) < TOL
    G = r["grads"]
    L = O.Offsets(d, h)
    blocks = dict(wq=(L.wq, L.q_bias), qb=(L.q_bias, L.wk), wk=(L.wk, L.k_bias), kb=(L.k_bias, L.wv),
                  wv=(L.wv, L.wo), wo=(L.wo, L.win), win=(L.win, L.wx), ns=(L.nscale, L.hist),
                  anchor=(L.slot_anchor, L.w_k_write))
    if c["fpm"]:
        blocks.update(wup=(L.w_retain_up, L.w_retain_down), wdown=(L.w_retain_down, L.b_retain),
                      bret=(L.b_retain, L.w_q_mem), bdelta=(L.b_delta, L.flags),
                      wgate=(L.w_write_gate, L.b_write_mem), bwrite=(L.b_write_mem, L.hhist_gamma),
                      alog=(L.alog, L.nscale), wout=(L.wout, L.alog), wx=(L.wx, L.wout))
        assert np.abs(G[L.w_retain_down:L.b_retain]).max() > 0 and np.abs(G[L.b_retain:L.w_q_mem]).max() > 0
    for name, (a, b) in blocks.items():
        assert rel(Gg[a:b], G[a:b]) < TOL, name
    assert rel(be.read("ds_in", (N, d)), r["dS"]) < TOL
    assert rel(be.read("lm_grads", (r["lm_grads"].size,)), r["lm_grads"]) < TOL
    # Adam step on both parameter sets: the kernel against the oracle's Adam on
    # the GPU's own gradients (fp32 rounding only); the gradients feeding it
    # were compared at 1e-3 above (parity_util.step_errors says why the update
    # W_new - W is not itself a 1e-3 quantity)
    be.apply_update(rule=RULE_ADAM, lr=1e-3, step=1, lm_head=True)
    e = step_errors(be, r, W, lm, B, T)
    assert e["adam_kernel"] < 1e-4 and e["lm_adam_kernel"] < 1e-4, e
    be.close()


def test_clipped_sgd_update():
    d, h = 128, 2
    W = init_all_weights(d, h, seed=2)
    be = GpuDeqBackend(d, h, max_batch=1, max_seq_len=4)
    be.upload_weights(W)
    S = np.random.default_rng(0).uniform(-1, 1, (1, 4, d)).astype(np.float32)
    be.run_forward_deq_no_readback(S, 1, 4, RunConfig())
    be.run_staged_adjoint_picard_no_readback(0.85, 4, dl_dh=np.ones((4, d), np.float32))
    be.weight_grads()
    G = be.read_grads()
    be.apply_update(rule=RULE_CLIPPED_SGD, lr=0.5, weight_decay=0.1)
    ref = O.clipped_sgd(W, G, 0.5, 0.1, O.Offsets(d, h).hist)
    assert np.abs(be.read_weights() - ref).max() < 1e-5
    be.close()


@pytest.mark.parametrize("d,h", [(128, 4), (256, 2), (512, 8), (1024, 16)])
def test_spectral_renorm_parity(d, h):
    W = init_all_weights(d, h, seed=9, attn_sigma=0.9, win_sigma=0.9)
    be = GpuDeqBackend(d, h, max_batch=1, max_seq_len=1)
    be.upload_weights(W)
    sig = be.renormalize_spectral(n_iters=12)
    Wr, sr = O.spectral_renorm(W, d, h, n_iters=12)
    assert rel(sig, sr) < 1e-4
    assert rel(be.read_weights(), Wr) < 1e-5
    be.close()


def test_train_step_api_matches_oracle():
    c = dict(d=128, h=4, B=2, T=8, fpm=True)
    d, h, B, T, V = 128, 4, 2, 8, 50
    W, be, S, rc, cfg = _setup(c, vocab=V)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rng = np.random.default_rng(8)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    loss = be.train_step(tok, tg, B, T, rc, adj_iters=12, lr=1e-3, step=1)
    cfg.adj_iters = 12
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    assert_step(step_errors(be, r, W, lm, B, T), loss, r)
    be.close()


def test_adam_skips_only_entries_no_gradient_reaches(monkeypatch):
    """The update that sweeps only the entries a gradient can reach (W_q/W_k/W_v
    columns 0..31, W_o rows 0..31, everything else whole) leaves weights and
    moments bitwise equal to the full sweep, over three steps; moments uploaded
    with non-zero entries there switch it back to the full sweep."""
    d, h, B, T, V = 128, 4, 2, 8, 50
    rng = np.random.default_rng(3)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    out = []
    for full in (False, True):
        if full:
            monkeypatch.setenv("AIDEEN_ADAM_FULL", "1")
        else:
            monkeypatch.delenv("AIDEEN_ADAM_FULL", raising=False)
        W, be, S, rc, cfg = _setup(dict(d=d, h=h, B=B, T=T, fpm=True), vocab=V)
        be.upload_lm_head(*init_lm_head(d, V))
        be.upload_embedding(init_embedding(d, V))
        for k in range(3):
            be.train_step(tok, tg, B, T, rc, adj_iters=12, lr=1e-3, step=k + 1)
        mc, vc, _, _ = be.read_adam()
        out.append((be.read_weights(), mc, vc))
        be.close()
    for a, b in zip(out[0], out[1]):
        assert np.array_equal(a, b)
    # non-zero moments where no gradient reaches: the full sweep again
    monkeypatch.delenv("AIDEEN_ADAM_FULL", raising=False)
    W, be, S, rc, cfg = _setup(dict(d=d, h=h, B=B, T=T, fpm=True), vocab=V)
    be.upload_lm_head(*init_lm_head(d, V))
    be.upload_embedding(init_embedding(d, V))
    L = be.layout
    m = np.zeros(L.total, np.float32)
    m[L.wq + d - 1] = 1e-3                        # row 0, column d-1 of slot 0's W_q
    be.upload_adam(m, np.full(L.total, 1e-6, np.float32))
    w0 = be.read_weights()
    be.train_step(tok, tg, B, T, rc, adj_iters=12, lr=1e-3, step=2)
    assert be.read_weights()[L.wq + d - 1] != w0[L.wq + d - 1]
    be.close()


def test_rejects_sizes_beyond_caps():
    be = GpuDeqBackend(128, 2, max_batch=1, max_seq_len=4)
    be.upload_weights(init_all_weights(128, 2))
    with pytest.raises(AideenError):
        be.run_forward_deq_no_readback(np.zeros((1, 8, 128), np.float32), 1, 8, RunConfig())
    with pytest.raises(AideenError):
        be.upload_weights(np.zeros(10, np.float32))
    be.close()


def _fpm_chunk(be, W, lm, emb, tok, tg, rc, cfg, carry, mstate):
    B, T = tok.shape
    d, h = cfg.d, cfg.h
    be.run_forward_tokens(tok, B, T, rc)
    be.lm_head_loss(tg)
    be.run_staged_adjoint_picard_no_readback(0.85, 12)
    be.weight_grads()
    r = O.train_step(emb[tok], tg, W, lm, cfg, mstate=mstate, fpm_carry=carry)
    return r


def test_fpm_backward_tbptt_carry_across_chunks():
    """Two consecutive chunks of the same sequences: the FPM memory and the
    TBPTT carry both flow into the second chunk's gradients; reset_state clears both."""
    d, h, B, T, V = 128, 4, 2, 8, 61
    c = dict(d=d, h=h, B=B, T=T, fpm=True)
    W, be, S, rc, cfg = _setup(c, vocab=V)
    cfg.adj_iters = 12
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    be.upload_lm_head(*lm)
    be.upload_embedding(emb)
    rng = np.random.default_rng(21)
    toks = [rng.integers(0, V, (B, T)).astype(np.int32) for _ in range(2)]
    tgs = [rng.integers(0, V, (B, T)).astype(np.int32) for _ in range(2)]
    r1 = _fpm_chunk(be, W, lm, emb, toks[0], tgs[0], rc, cfg, None, None)
    N = B * T
    assert rel(be.read("fpm_dm", (B, T, h, d)), r1["fpm"]["dm"]) < TOL
    assert rel(be.read("fpm_carry", (B, h, d)), r1["fpm"]["carry"]) < TOL
    r2 = _fpm_chunk(be, W, lm, emb, toks[1], tgs[1], rc, cfg, r1["fpm"]["carry"], r1["fwd"].mstate)
    L = O.Offsets(d, h)
    Gg = be.read_grads()
    G = r2["grads"]
    for name, (a, b) in dict(wup=(L.w_retain_up, L.w_retain_down), wdown=(L.w_retain_down, L.b_retain),
                             bret=(L.b_retain, L.w_q_mem), alog=(L.alog, L.nscale),
                             wout=(L.wout, L.alog), wgate=(L.w_write_gate, L.b_write_mem)).items():
        assert rel(Gg[a:b], G[a:b]) < TOL, name
    assert rel(be.read("fpm_carry", (B, h, d)), r2["fpm"]["carry"]) < TOL
    be.reset_state()
    assert np.abs(be.read("fpm_carry", (B, h, d))).max() == 0.0
    be.close()


def test_pipelined_train_step_matches_sequential_and_oracle():
    """The chunked training step (Picard token chunks overlapped with the LM head
    and adjoint) gives the sequential step's loss, gradients and update."""
    import os
    d, h, B, T, V = 128, 4, 4, 16, 61
    c = dict(d=d, h=h, B=B, T=T, fpm=True)
    W, _, _, rc, cfg = _setup(c, vocab=V)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    rng = np.random.default_rng(31)
    tok = rng.integers(0, V, (B, T)).astype(np.int32)
    tg = rng.integers(0, V, (B, T)).astype(np.int32)
    tg[1, 3] = -1
    out = {}
    for mode in ("seq", "pipe"):
        if mode == "seq":
            os.environ["AIDEEN_NO_PIPELINE"] = "1"
        else:
            os.environ.pop("AIDEEN_NO_PIPELINE", None)
        be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V)
        be.upload_weights(W)
        be.upload_lm_head(*lm)
        be.upload_embedding(emb)
        loss = be.train_step(tok, tg, B, T, rc, adj_iters=12, lr=1e-3, step=1)
        out[mode] = (loss, be.read_grads(), be.read("lm_grads", (V * d + V + d,)), be.read_weights(),
                     be.read("iters", (B, T, h), np.int32))
        be.close()
    os.environ.pop("AIDEEN_NO_PIPELINE", None)
    ls, gs, lgs, ws, its = out["seq"]
    lp, gp, lgp, wp, itp = out["pipe"]
    assert np.array_equal(its, itp)
    assert abs(lp - ls) <= 1e-6 * abs(ls)
    assert rel(gp, gs) < 1e-5 and rel(lgp, lgs) < 1e-5
    cfg.adj_iters = 12
    r = O.train_step(emb[tok], tg, W, lm, cfg)
    assert abs(lp - r["loss"]) / r["loss"] < TOL
    assert rel(gp, r["grads"]) < TOL and rel(lgp, r["lm_grads"]) < TOL
    W_kernel, _, _ = O.adam(W, gp, np.zeros_like(W, np.float64), np.zeros_like(W, np.float64), 1, lr=1e-3)
    assert rel(wp.astype(np.float64) - W, W_kernel.astype(np.float32).astype(np.float64) - W) < 1e-4


@pytest.mark.parametrize("d,h", [(128, 4), (512, 8), (1024, 16)])
def test_temporal_carrier_scan(d, h):
    """The simple temporal carrier over two consecutive chunks of fixed points
    (the carried MState links them) against the oracle's `temporal_scan`."""
    B, T = 2, 6
    W = init_all_weights(d, h, seed=4)
    rng = np.random.default_rng(6)
    L = O.Offsets(d, h)
    W[L.wout:L.wout + d * d] = (0.02 * rng.standard_normal(d * d)).astype(np.float32)
    W[L.wx:L.wx + d * d] = (0.5 * rng.standard_normal(d * d)).astype(np.float32)
    be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T)
    be.upload_weights(W)
    m = None
    for chunk in range(2):
        hs = rng.standard_normal((B, T, h, d)).astype(np.float32)
        be.temporal_scan(B, T, hs)
        hist, m = O.temporal_scan(hs, W, d, h, mstate=m)
        assert rel(be.read("hist_ctx", (B, T, h, d)), hist) < 1e-5
        assert rel(be.read("mstate", (B, h, d)), m) < 1e-5
    be.close()


def test_checkpoint_resume_continues_identically(tmp_path):
    """Save the weights (.aidn) and Adam state (.opt) after two steps, load them
    into a fresh context: the third step (from a reset memory state) is the
    same on both."""
    from aideen_b200 import checkpoint as ck
    d, h, B, T, V = 128, 4, 2, 8, 61
    W = init_all_weights(d, h, seed=3)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    rng = np.random.default_rng(4)
    toks = [rng.integers(0, V, (B, T)).astype(np.int32) for _ in range(3)]
    rc = RunConfig(fpm=True)

    def fresh():
        be = GpuDeqBackend(d, h, max_batch=B, max_seq_len=T, vocab=V)
        return be

    a = fresh()
    a.upload_weights(W)
    a.upload_lm_head(*lm)
    a.upload_embedding(emb)
    for k in range(2):
        a.train_step(toks[k], toks[k], B, T, rc, adj_iters=8, step=k + 1)
    ck.full_model(a.read_weights(), d, h, a.read_lm_head(), a.read_embedding()).save(str(tmp_path / "m.aidn"))
    ck.save_opt(str(tmp_path / "m.opt"), 2, ck.adam_tensors(*a.read_adam()[:2], d, h, *a.read_adam()[2:]))
    b = fresh()
    w, lmb, e = ck.unpack_full_model(ck.AidenModel.load(str(tmp_path / "m.aidn")))
    b.upload_weights(w)
    b.upload_lm_head(*lmb)
    b.upload_embedding(e)
    step, t = ck.load_opt(str(tmp_path / "m.opt"))
    b.upload_adam(*ck.adam_from_tensors(t, d, h))
    # the carried FPM memory and TBPTT carry are run state, not checkpointed:
    # both contexts start the next step from zero
    a.reset_state()
    b.reset_state()
    la = a.train_step(toks[2], toks[2], B, T, rc, adj_iters=8, step=3)
    lb = b.train_step(toks[2], toks[2], B, T, rc, adj_iters=8, step=step + 1)
    assert la == lb
    assert np.array_equal(a.read_weights(), b.read_weights())
    assert all(np.array_equal(x, y) for x, y in zip(a.read_lm_head(), b.read_lm_head()))
    a.close()
    b.close()
