"""CPU oracle for the AIDEEN DEQ training hot path.  TEST INFRASTRUCTURE ONLY.

This module is the parity checker.  Only `tests/`, `__graft_entry__.smoke()`
and the CPU-baseline leg of `bench.py` may import it; the product path
(`aideen_b200`) never calls it.

It restates, in float64 numpy, the reference's live GPU semantics:

* input projection          `deq_slot_attn_unified_clean.wgsl:762-804`
* iter-0 slot attention      `deq_slot_attn_unified_clean.wgsl:281-495`
* Picard solve + stop rule   `deq_slot_attn_unified_clean.wgsl:900-943, 960-1806`
* FPM read (Model A inject)  `deq_slot_attn_unified_clean.wgsl:855-883, 1006-1200`
* FPM write (memory scan)    `deq_slot_attn_unified_clean.wgsl:1965-2140, 2290-2300`
* slot pooling               `aideen-block/src/shaders/deq_forward_pool.wgsl:32-65`
* LM-head CE + RMSNorm bwd   `aideen-backbone/src/shaders/lm_train.wgsl:79-130, 327-395`
* clean adjoint init/step    `staged_adjoint_picard_clean.wgsl:143-248`
* Anderson store/mix         `staged_adjoint_picard_clean.wgsl:1011-1135`
* source-grad reduce         `staged_adjoint_picard_clean.wgsl:250-327`
* Adam                       `aideen-training-lab/src/optimizer.rs:105-183`
* clipped SGD apply          `aideen-backbone/src/shaders/fused_deq_update.wgsl:809-823`
* spectral renorm            `aideen-block/src/shaders/spectral_renorm.wgsl:83-196`
* FPM backward (TBPTT scan)  `aideen-backbone/src/shaders/fused_fpm_retain_bwd.wgsl:364-2095`
* FPM W_out / W_x grads      `aideen-backbone/src/shaders/fused_fpm_shared_update.wgsl:129-256`
* temporal carrier (simple)  `aideen-backbone/src/fixed_point_memory_reasoning.rs:1455-1486`
* sampled-softmax LM head    `aideen-backbone/src/shaders/lm_train.wgsl:79-395`, `gpu_lm_head.rs:213-281`
* embedding-row Adam         `aideen-backbone/src/shaders/embedding_train.wgsl:100-147`
* associative branch (upper h/2 slots, default flags; Cfg.assoc)
                             `deq_slot_attn_unified_clean.wgsl:554-556, 1216-1563, 1970-1971, 2293-2948`

Weight gradients are derived analytically (implicit-function theorem through
the map the clean adjoint linearises); the reference's own stage-4 shaders
read a stale scratch layout and are not used as a source.  The gradients are
pinned by central finite differences in `tests/test_oracle_cpu.py`.

PARITY PIN STATUS: partially pinned.  The reference is Rust + WGSL and cannot
run here (no cargo, no wgpu adapter); its tests hold no golden vectors for
this path.  What pins the oracle: the reference's spectral-norm known answers
(`spectral_norm.rs:102-149`), the reference's numeric-adjoint test case
(`aideen-backbone/tests/picard_pipeline_test.rs:1859-1935`, cosine > 0.80),
and finite-difference checks of every gradient.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

RANK = 32
HOMEO_MIN_ITERS = 4           # FPM_HOMEO_MIN_ITERS
HOMEO_ALPHA_ERR_SCALE = 0.15  # FPM_HOMEO_ALPHA_ERR_SCALE
HOMEO_PLATEAU_TOL = 0.10      # FPM_HOMEO_PLATEAU_TOL
FPM_ALPHA_H = 0.2
FPM_GATE_BIAS = -1.5
FPM_RESIDUAL_SCALE = 0.1
# associative branch, default flags (deq_slot_attn_unified_clean.wgsl:79-96, deq_bridge.rs:176-350)
ASSOC_WRITE_CAP = 0.95
ASSOC_OCCUPIED_THRESHOLD = 1e-4
ASSOC_USAGE_DECAY = 0.999
ASSOC_TO_FPM_SCALE = 0.02
ASSOC_SUPPRESS_COS = 0.85        # ENABLE_ASSOC_SUPPRESS_VALUE_SOURCE threshold (`:2755`)


def es(spec, *ops):
    return np.einsum(spec, *ops, optimize=True)


class Offsets:
    """AllWeights offsets, restated independently of the package
    (`deq_slot_attn_unified_clean.wgsl:189-237`, `gpu_deq.rs:260-422`)."""

    def __init__(self, d: int, h: int):
        r = RANK
        self.d, self.h = d, h
        dd = d * d
        self.wq = 0
        self.q_bias = h * dd
        self.wk = h * dd + h * d
        self.k_bias = self.wk + h * dd
        self.wv = self.wk + h * dd + h * d
        self.wo = self.wv + h * dd
        self.win = self.wo + h * dd
        self.wx = self.win + h * dd
        self.wout = self.wx + dd
        self.alog = self.wout + dd
        self.nscale = self.alog + h * d
        self.hist = self.nscale + d
        o = self.hist + dd                 # after hist_mat
        self.hist_scale = o; o += h * d
        self.hist_bias = o; o += h * d
        self.hist_gate = o; o += h
        self.slot_anchor = o; o += h * d
        self.w_k_write = o; o += h * d * r
        self.w_v_write = o; o += h * r * d
        self.b_delta = o; o += h * d
        self.flags = o; o += 21
        self.signal_zero = self.flags + 9
        self.signal_scale = self.flags + 16
        self.hist_gate_query = o; o += h * d
        self.w_write_gate = o; o += h * d
        self.b_write_mem = o; o += h
        self.hhist_gamma = o; o += h
        self.w_retain_up = o; o += h * d * r
        self.w_retain_down = o; o += h * r * d
        self.b_retain = o; o += h * d
        self.w_q_mem = o; o += h * d * r
        self.w_k_mem = o; o += h * d * r
        self.b_read_mem = o; o += h
        self.w_k_assoc = o; o += h * d * r    # associative block (`:232-237`)
        self.w_v_assoc = o; o += h * d * r
        self.w_q_assoc = o; o += h * d * r
        self.alpha_assoc = o; o += h
        self.w_event_assoc = o; o += h * d
        self.b_event_assoc = o; o += h
        self.total = o


class View:
    """Named float64 views of an AllWeights vector."""

    def __init__(self, w: np.ndarray, d: int, h: int):
        L = Offsets(d, h)
        self.L = L
        w = np.asarray(w, dtype=np.float64)
        dd, r = d * d, RANK
        self.hd = min(d, 32)
        self.Wq = w[L.wq:L.wq + h * dd].reshape(h, d, d)       # [s][j][o]
        self.qb = w[L.q_bias:L.q_bias + h * d].reshape(h, d)
        self.Wk = w[L.wk:L.wk + h * dd].reshape(h, d, d)
        self.kb = w[L.k_bias:L.k_bias + h * d].reshape(h, d)
        self.Wv = w[L.wv:L.wv + h * dd].reshape(h, d, d)
        self.Wo = w[L.wo:L.wo + h * dd].reshape(h, d, d)       # [s][k][o]
        self.Win = w[L.win:L.win + h * dd].reshape(h, d, d)
        self.Wx = w[L.wx:L.wx + dd].reshape(d, d)
        self.Wout = w[L.wout:L.wout + dd].reshape(d, d)
        self.Alog = w[L.alog:L.alog + h * d].reshape(h, d)
        self.NS = w[L.nscale:L.nscale + d]
        self.anchor = w[L.slot_anchor:L.slot_anchor + h * d].reshape(h, d)
        self.hscale = w[L.hist_scale:L.hist_scale + h * d].reshape(h, d)
        self.hbias = w[L.hist_bias:L.hist_bias + h * d].reshape(h, d)
        self.Wkw = w[L.w_k_write:L.w_k_write + h * d * r].reshape(h, d, r)
        self.Wvw = w[L.w_v_write:L.w_v_write + h * r * d].reshape(h, r, d)
        self.bdelta = w[L.b_delta:L.b_delta + h * d].reshape(h, d)
        self.signal_zero = w[L.signal_zero] > 0.5
        self.sig_scale = float(w[L.signal_scale])
        self.wgate = w[L.w_write_gate:L.w_write_gate + h * d].reshape(h, d)
        self.bwrite = w[L.b_write_mem:L.b_write_mem + h]
        self.Wup = w[L.w_retain_up:L.w_retain_up + h * d * r].reshape(h, d, r)
        self.Wdown = w[L.w_retain_down:L.w_retain_down + h * r * d].reshape(h, r, d)
        self.bret = w[L.b_retain:L.b_retain + h * d].reshape(h, d)
        self.Wqm = w[L.w_q_mem:L.w_q_mem + h * d * r].reshape(h, d, r)
        self.Wkm = w[L.w_k_mem:L.w_k_mem + h * d * r].reshape(h, d, r)
        self.bread = w[L.b_read_mem:L.b_read_mem + h]
        self.alpha_assoc = w[L.alpha_assoc:L.alpha_assoc + h]


@dataclass
class Cfg:
    d: int
    h: int
    max_iters: int = 12
    eps: float = 1e-4
    damping: float = 0.85          # forward blend (generic path) and adjoint beta
    slot_coord: bool = True        # residual_alpha in (-1.5, -0.9]: attention branch on
    fpm: bool = False              # Model-A memory read/inject/write
    fpm_alpha_m: float = 0.01
    fpm_tau: float = 0.5
    fpm_read_gate_min: float = 0.0
    adj_iters: int = 12
    anderson_m: int = 0            # adjoint Anderson depth (0 = off)
    fwd_anderson_m: int = 0        # forward Anderson depth (0 = plain Picard)
    assoc: bool = False            # associative branch of the upper h/2 slots (needs fpm)


def rms(x, axis=-1, eps=1e-6):
    return np.sqrt(np.mean(x * x, axis=axis) + eps)


# ---------------------------------------------------------------------------
# forward
# ---------------------------------------------------------------------------

def project_signal(S, V: View):
    """signal[n,s,o] = sigma * sum_j Win[s][j][o] S[n,j]  (`:762-804`)."""
    S = np.asarray(S, np.float64)
    sig = es('nj,sjo->nso', S, V.Win) * V.sig_scale
    if V.signal_zero:
        sig = np.zeros_like(sig)
    return sig


def slot_attention(signal, V: View):
    """Iter-0 slot attention per token (`compute_slot_coord`, `:281-495`).

    signal: [N,h,d].  Returns A = attn*scale [N,h,d] and a cache dict.
    """
    N, h, d = signal.shape
    hd = V.hd
    src = signal + V.anchor[None]
    R = rms(src)                                         # slot_coord_prev, [N,h]
    K = es('nkj,kjc->nkc', src, V.Wk[:, :, :hd]) + V.kb[None, :, :hd]
    Vv = es('nkj,kjc->nkc', src, V.Wv[:, :, :hd])
    Q = es('nsj,sjc->nsc', src, V.Wq[:, :, :hd]) + V.qb[None, :, :hd]
    logits = es('nsc,nkc->nsk', Q, K) * (2.0 / math.sqrt(max(1, hd)))
    if h > 1:
        idx = np.arange(h)
        logits[:, idx, idx] = -1e30
    mx = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - mx)
    ssum = np.maximum(e.sum(-1, keepdims=True), 1e-12)
    alpha = e / ssum                                      # [N,s,k]
    mix = es('nsk,nkc->nsc', alpha, Vv) - Vv.mean(axis=1, keepdims=True)
    r = np.sqrt(np.mean(mix * mix, -1) + 1e-6)            # [N,s]
    nmix = mix / r[..., None]
    a = es('nsc,sco->nso', nmix, V.Wo[:, :hd, :])
    rho = rms(a)
    scale = np.maximum(R, 1e-3) / np.maximum(rho, 1e-6)
    A = a * scale[..., None]
    cache = dict(src=src, R=R, K=K, V=Vv, Q=Q, alpha=alpha, mix=mix, r=r, n=nmix,
                 a=a, rho=rho, scale=scale)
    return A, cache


def _converged(err, prev, it, eps):
    band = max(eps, HOMEO_ALPHA_ERR_SCALE * FPM_ALPHA_H)
    plateau = np.abs(err - prev) / np.maximum(prev, eps)
    strict = err < eps
    homeo = (it + 1 >= HOMEO_MIN_ITERS) & (err <= band) & (plateau <= HOMEO_PLATEAU_TOL)
    return strict | homeo


def fpm_keys(m_prev, V: View):
    """k_mem[b,ms,r] = sum_j Wkm[ms][j][r] (m + scale*tanh(m) + bias)  (`:855-883`)."""
    keyed = m_prev + V.hscale[None] * np.tanh(m_prev) + V.hbias[None]
    return es('bmj,mjr->bmr', keyed, V.Wkm)


def fpm_read(h_cur, sig_t, keys, m_prev, V: View, cfg: Cfg):
    """Memory context from the first structured state (`:1031-1200`).

    h_cur: [B,h,d] (state after iteration 0), sig_t: [B,h,d].
    """
    B, h, d = h_cur.shape
    hq = h_cur / np.sqrt(np.maximum((h_cur * h_cur).sum(-1, keepdims=True), 1e-6))
    q = es('bsj,sjr->bsr', hq, V.Wqm)
    score = es('bsr,bmr->bsm', q, keys) + V.bread[None, None, :]
    score = score / math.sqrt(RANK) / max(cfg.fpm_tau, 1e-3)
    mx = score.max(-1, keepdims=True)
    e = np.exp(score - mx)
    w = e / np.maximum(e.sum(-1, keepdims=True), 1e-12)
    peak = w.max(-1)
    uni = 1.0 / max(1, h)
    conf = np.clip((peak - uni) / max(1e-6, 1.0 - uni), 0.0, 1.0)
    gate = np.maximum(np.sqrt(conf), cfg.fpm_read_gate_min)
    mem_raw = es('bsm,bmd->bsd', w, m_prev)
    mu = np.tanh(mem_raw)
    mu_norm = np.sqrt(np.maximum((mu * mu).sum(-1), 1e-6))
    sig_norm = np.sqrt(np.maximum((sig_t * sig_t).sum(-1), 1e-6))
    alpha_m = max(cfg.fpm_alpha_m, 0.001)
    coef = sig_norm * alpha_m / np.maximum(mu_norm, 1e-6) * gate
    return mu * coef[..., None]


def fpm_write(h_star, sig_t, m_prev, V: View, Wx_diag):
    """Post-solve memory update (`:1965-2140`); returns m_inner [B,h,d]."""
    B, h, d = h_star.shape
    c = 0.5 * (h_star + sig_t)
    h_rms = np.sqrt(np.maximum((h_star * h_star).sum(-1) / d, 1e-6))
    hu = h_star / h_rms[..., None]
    gate_in = (c * V.wgate[None]).sum(-1) / math.sqrt(d) + V.bwrite[None] + FPM_GATE_BIAS
    z = np.clip(1.0 / (1.0 + np.exp(-gate_in)), 0.0, 1.0)
    bott = es('bsj,sjr->bsr', c, V.Wkw)
    prop = np.tanh(V.bdelta[None] + es('bsr,sro->bso', bott, V.Wvw))
    prev_norm = np.sqrt(np.maximum((m_prev * m_prev).sum(-1), 1e-6))
    diff = prop - m_prev
    diff_norm = np.sqrt(np.maximum((diff * diff).sum(-1), 1e-6))
    novelty = diff_norm / (diff_norm + prev_norm + 1e-6)
    up = es('bsj,sjr->bsr', c, V.Wup)
    retain_raw = 1.0 / (1.0 + np.exp(-(V.bret[None] + es('bsr,sro->bso', up, V.Wdown))))
    retain = 1.0 - novelty[..., None] * (1.0 - retain_raw)
    write = z[..., None] * (FPM_RESIDUAL_SCALE * prop)
    wx = 0.5 * np.tanh(Wx_diag)[None, None, :]
    x = np.sqrt(np.maximum(z, 1e-6))[..., None] * hu + wx * hu + write
    a = 1.0 / (1.0 + np.exp(V.Alog))[None]
    base = a * m_prev + (1.0 - a) * x
    return retain * m_prev + (1.0 - retain) * base


def _rms_floor(x):
    """sqrt(mean(x^2) + 1e-6) floored at 1e-6 (the shader's max(rms, 1e-6))."""
    return np.maximum(np.sqrt((x * x).mean(-1) + 1e-6), 1e-6)


def assoc_read(bank_v, sig_t, V: View, cfg: Cfg):
    """Associative read of one token, default flags (`deq_slot_attn_unified_clean.wgsl:1216-1563`):
    one bank and a hard read, so the bank is selected whatever its address score, and the
    read returns its value.  Injected into the memory context:
    sigmoid(alpha_assoc[s]) * bank_v * |signal| * alpha_m / max(|bank_v|, 1e-3).
    bank_v, sig_t: [B,h,d]; returns [B,h,d] for every slot (the caller keeps the upper half)."""
    sig_norm = np.sqrt(np.maximum((sig_t * sig_t).sum(-1), 1e-6))
    v_norm = np.sqrt(np.maximum((bank_v * bank_v).sum(-1), 1e-6))
    alpha = 1.0 / (1.0 + np.exp(-V.alpha_assoc))[None, :]
    scale = sig_norm * max(cfg.fpm_alpha_m, 0.001) / np.maximum(v_norm, 1e-6)
    return (alpha * scale)[..., None] * bank_v


def assoc_write(x_t, state, m, h_star, t):
    """Associative write of one token, default flags (`:2293-2948`): returns the
    memory after the consolidation, the unnormalised payload the stored signal is
    replaced with, and updates `state` (bank value V, usage u, previous source P;
    each [B,h,...]) in place.

    value   = x / rms(x), renormalised by its own rms   (x = this token's S_in row)
    payload = value + P / rms(P), then / rms(payload)    (ASSOC_REL_VALUE_MIX = 1)
    mass    = [t > 0] * [bank empty: usage < 1e-4] * [cos(V, P / rms(P)) <= 0.85]
    V <- (1 - mass) V + mass payload;  usage <- clamp(max(0.999 usage, mass), 0, 1)
    m <- (1 - c) m + c h*/rms(h*),  c = 0.02 * min(1, 0.95) * mass  (no FPM write on
         these slots, so the write-gate factor keeps its initial 1.0, `:1970`)
    P <- value.
    x_t: [B,d]; m, h_star: [B,h,d]."""
    Vb, u, P = state["V"], state["u"], state["P"]
    x = np.broadcast_to(np.asarray(x_t, np.float64)[:, None, :], P.shape)
    val0 = x / _rms_floor(x)[..., None]
    val = val0 / _rms_floor(val0)[..., None]
    Pn = P / _rms_floor(P)[..., None]
    pay_raw = val + Pn
    pay = pay_raw / _rms_floor(pay_raw)[..., None]
    u_c = np.clip(np.where(np.isfinite(u), u, 0.0), 0.0, 1.0)
    empty = u_c < ASSOC_OCCUPIED_THRESHOLD
    vv = (Vb * Vb).sum(-1)
    pp = (Pn * Pn).sum(-1)
    cos = (Vb * Pn).sum(-1) / np.sqrt(np.maximum(vv * pp, 1e-12))
    cos = np.where(np.isfinite(cos), cos, -1.0)
    allow = empty & ~(cos > ASSOC_SUPPRESS_COS)
    mass = (1.0 if t > 0 else 0.0) * allow.astype(np.float64)
    state["V"] = (1.0 - mass)[..., None] * Vb + mass[..., None] * pay
    c = ASSOC_TO_FPM_SCALE * min(1.0, ASSOC_WRITE_CAP) * mass
    hu = h_star / _rms_floor(h_star)[..., None]
    m_new = (1.0 - c)[..., None] * m + c[..., None] * hu
    state["u"] = np.clip(np.maximum(ASSOC_USAGE_DECAY * u_c, mass), 0.0, 1.0)
    state["P"] = val
    return m_new, pay_raw


def assoc_alpha_grad(assoc_read, v, W, d, h):
    """The reference's alpha_assoc gradient, default flags (`fused_fpm_retain_bwd.wgsl:
    1129-1160, 1281-1284`): one bank, read confidence and slot prior 1, so per
    upper slot s
        G[s] = sigmoid'(alpha_s) * sum_{b,t} (v[b,t,s] . V[b,t,s]) / max(rms(V[b,t,s]), 0.1)
    with V the bank value token t read and v the clean adjoint (non-finite entries
    as 0).  Like the rest of that backward it is the reference's formula, not the
    exact derivative of the forward's injection (which scales V to
    sigmoid(alpha) |signal| alpha_m / |V|).  assoc_read [B,T,h,d]; v [B*T,h,d]."""
    V = View(W, d, h)
    vr = np.asarray(assoc_read, np.float64).reshape(-1, h, d)
    vv = np.asarray(v, np.float64)
    vv = np.where(np.isfinite(vv), vv, 0.0)
    rms_v = np.sqrt((vr * vr).sum(-1) / d)
    tot = ((vv * vr).sum(-1) / np.maximum(rms_v, 0.1)).sum(0)        # [h]
    a = 1.0 / (1.0 + np.exp(-V.alpha_assoc))
    g = a * (1.0 - a) * tot
    g[: h // 2] = 0.0
    return g


def assoc_state_zeros(B, h, d):
    """The reset state (reset_state, gpu_deq.rs:3141-3160: AssocBuf and PrevHStarBuf zeroed)."""
    return dict(V=np.zeros((B, h, d)), u=np.zeros((B, h)), P=np.zeros((B, h, d)))


def temporal_step(m_prev, h_star, V: View):
    """The simple temporal carrier `temporal_step` (fixed_point_memory_reasoning.rs:1455-1486;
    GPU form hist_v2_temporal.wgsl:60-108): per slot,
    M' = (I + W_out^T)(a * M + (1 - a) * (1 + 0.5 tanh(diag W_x)) * h / rms(h)),
    a = sigmoid(-a_log[slot]), W_out read as [j][d_out] like the shader.
    m_prev, h_star: [B,h,d]."""
    hr = np.sqrt((h_star * h_star).mean(-1) + 1e-6)
    hu = h_star / np.maximum(hr, 1e-6)[..., None]
    a = 1.0 / (1.0 + np.exp(V.Alog))[None]
    x = hu + 0.5 * np.tanh(np.diag(V.Wx))[None, None, :] * hu
    mn = a * m_prev + (1.0 - a) * x
    return mn + es('bsj,jo->bso', mn, V.Wout)


def temporal_scan(hstar, W, d, h, mstate=None):
    """The carrier over a [B,T,h,d] chunk of fixed points, token by token:
    returns the memory after every token [B,T,h,d] and the carried state [B,h,d]."""
    V = View(W, d, h)
    hs = np.asarray(hstar, np.float64)
    B, T = hs.shape[:2]
    m = np.zeros((B, h, d)) if mstate is None else np.asarray(mstate, np.float64).copy()
    out = np.zeros_like(hs)
    for t in range(T):
        m = temporal_step(m, hs[:, t], V)
        out[:, t] = m
    return out, m


@dataclass
class ForwardOut:
    signal: np.ndarray        # [B,T,h,d]
    A: np.ndarray             # [B,T,h,d] attention injection (attn*scale)
    hstar: np.ndarray         # [B,T,h,d]
    iters: np.ndarray         # [B,T,h] int
    pooled: np.ndarray        # [B,T,d]
    hist_ctx: np.ndarray      # [B,T,h,d] (FPM memory per token; zeros without FPM)
    mstate: np.ndarray        # [B,h,d]
    fpm_ctx: np.ndarray       # [B,T,h,d]
    attn_cache: dict = field(default_factory=dict)   # flattened [B*T, ...]
    # the signal the adjoint's branch is built from: the projection, except on the
    # associative slots, where the write replaced it with the payload (`:2497`)
    branch_signal: np.ndarray = None
    assoc_state: dict = None  # bank value V, usage u, previous source P after the chunk
    assoc_read: np.ndarray = None  # [B,T,h,d] bank value each token read (before its write)


def forward(S_in, W, cfg: Cfg, mstate=None, assoc_state=None) -> ForwardOut:
    """Forward DEQ solve over a [B,T,d] chunk (token carry on, `:900`).

    With cfg.fpm and cfg.assoc the upper h/2 slots run the reference's default
    associative branch instead of the FPM write (`:554-556, 1971`): `assoc_read`
    at the memory read, `assoc_write` after the solve; `assoc_state` carries its
    state across chunks (zeros: the reset state)."""
    d, h = cfg.d, cfg.h
    V = View(W, d, h)
    S = np.asarray(S_in, np.float64)
    B, T, _ = S.shape
    signal = project_signal(S.reshape(B * T, d), V).reshape(B, T, h, d)
    if cfg.slot_coord:
        A, cache = slot_attention(signal.reshape(B * T, h, d), V)
        A = A.reshape(B, T, h, d)
    else:
        A, cache = np.zeros_like(signal), {}
    NS = V.NS[None, None, :]
    anchor = V.anchor[None]
    blend = FPM_ALPHA_H if cfg.fpm else cfg.damping
    Wx_diag = np.diag(V.Wx)
    m = np.zeros((B, h, d)) if mstate is None else np.asarray(mstate, np.float64).copy()
    hstar = np.zeros((B, T, h, d))
    iters = np.zeros((B, T, h), np.int64)
    hist = np.zeros((B, T, h, d))
    ctx_all = np.zeros((B, T, h, d))
    hcur = None
    am = cfg.fwd_anderson_m
    assoc = cfg.fpm and cfg.assoc
    upper = (np.arange(h) >= h // 2)[None, :, None]
    ast = None
    if assoc:
        ast = assoc_state_zeros(B, h, d) if assoc_state is None else {
            k: np.asarray(x, np.float64).copy() for k, x in assoc_state.items()}
    branch_sig = signal.copy()
    vread = np.zeros((B, T, h, d)) if assoc else None
    for t in range(T):
        sig = signal[:, t]
        if t == 0:
            hcur = sig / np.maximum(rms(sig), 1e-6)[..., None]
        ctx = np.zeros((B, h, d))
        keys = fpm_keys(m, V) if cfg.fpm else None
        active = np.ones((B, h), bool)
        prev = np.ones((B, h))
        it_count = np.zeros((B, h), np.int64)
        # Anderson ring: Picard outputs g and residuals f of the last two iterations
        g1 = g2 = f1 = f2 = None
        for it in range(cfg.max_iters):
            if not active.any():
                break
            if cfg.fpm and it == 1:
                ctx_new = fpm_read(hcur, sig, keys, m, V, cfg)
                if assoc:
                    ctx_new = ctx_new + np.where(upper, assoc_read(ast["V"], sig, V, cfg), 0.0)
                ctx = np.where(active[..., None], ctx_new, ctx)
            dep = sig + hcur + anchor + (A[:, t] if it == 0 else 0.0)
            pre = dep + (ctx if (cfg.fpm and it >= 1) else 0.0)
            r = rms(dep)
            f = NS * pre / r[..., None]
            hn = blend * f + (1.0 - blend) * hcur
            dh = hn - hcur
            err = np.sqrt(np.mean(dh * dh, -1) + 1e-12) / np.maximum(r, 1e-6)
            conv = _converged(err, prev, it, cfg.eps)
            hnext = hn
            f0 = hn - hcur
            if am >= 2 and it >= 2:
                # Anderson (type II) over the residuals f = g(x) - x of the
                # iterations >= 1, whose map is fixed within the token
                n_res = min(it, am)
                D = [f0 - f1] + ([f1 - f2] if n_res == 3 else [])
                DtD = np.zeros((B, h, 2, 2))
                Dtf = np.zeros((B, h, 2))
                for i in range(n_res - 1):
                    Dtf[..., i] = (D[i] * f0).sum(-1)
                    for j in range(i, n_res - 1):
                        DtD[..., i, j] = DtD[..., j, i] = (D[i] * D[j]).sum(-1)
                gam, ok = anderson_fwd_gamma(DtD, Dtf, n_res - 1)
                mixed = hn - gam[..., 0, None] * (hn - g1)
                if n_res == 3:
                    mixed = mixed - gam[..., 1, None] * (g1 - g2)
                hnext = np.where((conv | ~ok)[..., None], hn, mixed)
            f2, f1 = f1, f0
            g2, g1 = g1, hn
            hcur = np.where(active[..., None], hnext, hcur)
            prev = np.where(active, err, prev)
            it_count = it_count + active
            active = active & ~conv
        hstar[:, t] = hcur
        iters[:, t] = it_count
        ctx_all[:, t] = ctx
        if cfg.fpm:
            m_w = fpm_write(hcur, sig, m, V, Wx_diag)
            if assoc:
                vread[:, t] = np.where(upper, ast["V"], 0.0)
                old = {k: x.copy() for k, x in ast.items()}
                m_a, pay_raw = assoc_write(S[:, t], ast, m, hcur, t)
                for k in ast:  # the lower slots hold no associative state
                    msk = upper if ast[k].ndim == 3 else upper[..., 0]
                    ast[k] = np.where(msk, ast[k], old[k])
                m_w = np.where(upper, m_a, m_w)
                branch_sig[:, t] = np.where(upper, pay_raw, sig)
            m = m_w
            hist[:, t] = m
    pooled = hstar.mean(axis=2)
    return ForwardOut(signal=signal, A=A, hstar=hstar, iters=iters, pooled=pooled,
                      hist_ctx=hist, mstate=m, fpm_ctx=ctx_all, attn_cache=cache,
                      branch_signal=branch_sig, assoc_state=ast, assoc_read=vread)


# ---------------------------------------------------------------------------
# LM head (producer of the adjoint RHS)
# ---------------------------------------------------------------------------

def lm_head(pooled, targets, w_lm, b_lm, g_lm):
    """Dense full-vocab CE through RMSNorm (`lm_train.wgsl:79-130, 327-395`).

    pooled: [N,d], targets: [N] (negative = ignored).  Returns loss (mean over
    active tokens), dL/dpooled [N,d], and grads of (w_lm, b_lm, g_lm).
    """
    P = np.asarray(pooled, np.float64)
    W = np.asarray(w_lm, np.float64)
    g_lm = np.asarray(g_lm, np.float64)
    N, d = P.shape
    r = np.sqrt(np.mean(P * P, -1) + 1e-5)
    xhat = P / r[:, None]
    y = xhat * g_lm[None]
    logits = y @ W.T + np.asarray(b_lm, np.float64)[None]
    mx = logits.max(-1, keepdims=True)
    e = np.exp(logits - mx)
    Z = e.sum(-1, keepdims=True)
    p = e / Z
    tg = np.asarray(targets).astype(np.int64)
    act = tg >= 0
    n_act = max(1, int(act.sum()))
    rows = np.nonzero(act)[0]
    loss = float(-(logits[rows, tg[rows]] - mx[rows, 0] - np.log(Z[rows, 0])).sum()) / n_act
    dlog = p.copy()
    dlog[rows, tg[rows]] -= 1.0
    dlog[~act] = 0.0
    dlog /= n_act
    dy = dlog @ W
    gW = dlog.T @ y
    gb = dlog.sum(0)
    gg = (dy * xhat).sum(0)
    dyg = dy * g_lm[None]
    dot = (dyg * P).sum(-1)
    dP = dyg / r[:, None] - P * (dot / (d * r ** 3))[:, None]
    return loss, dP, gW, gb, gg


LM_SAMPLE_SEED = 0xA1DEEE5A4D5EED5E   # gpu_lm_head.rs:1492-1494 default
LM_MAX_SAMPLES = 2048                 # MAX_SHADER_SAMPLES, gpu_lm_head.rs:247
_M64 = (1 << 64) - 1


def sample_candidate(seed, step_t, draw, vocab):
    """`deterministic_sample_candidate` (gpu_lm_head.rs:213-223): the seed mixed
    with the step and the draw index, then the splitmix64 finaliser."""
    x = (seed ^ ((step_t * 0x9E3779B97F4A7C15) & _M64) ^ ((draw * 0xD1B54A32D192ED03) & _M64)) & _M64
    x ^= x >> 30
    x = (x * 0xBF58476D1CE4E5B9) & _M64
    x ^= x >> 27
    x = (x * 0x94D049BB133111EB) & _M64
    x ^= x >> 31
    return x % vocab


def sampled_indices(targets, step_t, vocab, num_samples=512, seed=LM_SAMPLE_SEED):
    """`build_sampled_indices` (gpu_lm_head.rs:244-281): the distinct valid
    targets, filled with deterministic candidates in draw order (skipping ones
    already present) up to min(max(num_samples, len(targets)), vocab, 2048),
    sorted ascending.  (The reference's buffer capacity, at least 1024 x batch,
    never binds at these sizes.)"""
    tg = [int(t) for t in np.asarray(targets).ravel()]
    desired = min(max(num_samples, len(tg)), vocab, LM_MAX_SAMPLES)
    S = sorted({t for t in tg if 0 <= t < vocab})
    seen = set(S)
    draw = 0
    while len(S) < desired:
        c = sample_candidate(seed, step_t, draw, vocab)
        draw += 1
        if c not in seen:
            seen.add(c)
            S.append(c)
    return np.array(sorted(S), np.int64)


def lm_head_sampled(pooled, targets, w_lm, b_lm, g_lm, S, state, step, lr=1e-3, b1=0.9, b2=0.999,
                    eps=1e-8):
    """Sampled-softmax LM head with its fused Adam step, in the reference's
    order (`lm_train.wgsl`): lm_probs_main (:79-217) -> lm_update_main (:224-290,
    dW and db clamped to +-0.1 after the 1/active scaling, Adam on the sampled
    rows only) -> lm_backprop_h_t_main (:327-395, dL/dh from the *updated*
    rows, through the RMSNorm).  g_lm is not trained here.

    state: dict of Adam moments mW, vW [V,d], mb, vb [V] (updated in place).
    Returns loss (mean over valid targets), dL/dpooled [N,d], new W_lm, new
    b_lm, and the unclamped sampled-row gradients dW [K,d], db [K].
    """
    P = np.asarray(pooled, np.float64)
    W = np.asarray(w_lm, np.float64).copy()
    b = np.asarray(b_lm, np.float64).copy()
    g = np.asarray(g_lm, np.float64)
    N, d = P.shape
    V = W.shape[0]
    tg = np.asarray(targets).astype(np.int64).ravel()
    valid = (tg >= 0) & (tg < V)
    active = max(1, int(valid.sum()))
    r = np.sqrt(np.mean(P * P, -1) + 1e-5)
    y = P / r[:, None] * g[None]
    logits = y @ W[S].T + b[S][None]
    mx = logits.max(-1, keepdims=True)
    e = np.exp(logits - mx)
    p = e / np.maximum(e.sum(-1, keepdims=True), 1e-10)
    onehot = (S[None, :] == tg[:, None]).astype(np.float64)
    pt = (p * onehot).sum(-1)
    loss = float(-(np.log(np.maximum(pt[valid], 1e-10))).sum()) / active
    coef = (p - onehot) * valid[:, None] / active
    dW_raw, db_raw = coef.T @ y, coef.sum(0)
    dW = np.clip(dW_raw, -0.1, 0.1)
    db = np.clip(db_raw, -0.1, 0.1)
    t = max(1, step)
    bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
    for (w_arr, m_key, v_key, gr) in ((W, "mW", "vW", dW), (b, "mb", "vb", db)):
        m = state[m_key][S] * b1 + (1 - b1) * gr
        v = state[v_key][S] * b2 + (1 - b2) * gr * gr
        state[m_key][S] = m
        state[v_key][S] = v
        w_arr[S] -= lr * (m / bc1) / (np.sqrt(v / bc2) + eps)
    dldy = coef @ W[S]
    dot = (dldy * g[None] * P).sum(-1)
    dP = dldy * g[None] / r[:, None] - P * (dot / (d * r ** 3))[:, None]
    return loss, dP, W, b, dW_raw, db_raw


def embedding_update(emb, tokens, grad_rows, state, step, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8):
    """`apply_embedding_update_from_buffer` (gpu_embedding.rs:775-857) with
    `embedding_adamw_update` (embedding_train.wgsl:100-147): per distinct token
    (ids clamped to vocab - 1, `build_unique_token_csr` gpu_embedding.rs:47-70)
    the mean of its positions' gradient rows, then Adam on that row only.
    state: dict with m, v [V,d] (updated in place).  Returns the new table."""
    E = np.asarray(emb, np.float64).copy()
    V = E.shape[0]
    tok = np.minimum(np.asarray(tokens).astype(np.int64).ravel(), V - 1)
    G = np.asarray(grad_rows, np.float64)
    uniq, inv = np.unique(tok, return_inverse=True)
    sums = np.zeros((len(uniq), E.shape[1]))
    np.add.at(sums, inv, G)
    cnt = np.bincount(inv, minlength=len(uniq)).astype(np.float64)
    gr = sums / cnt[:, None]
    t = max(1, step)
    m = state["m"][uniq] * b1 + (1 - b1) * gr
    v = state["v"][uniq] * b2 + (1 - b2) * gr * gr
    state["m"][uniq] = m
    state["v"][uniq] = v
    E[uniq] -= lr * (m / (1 - b1 ** t)) / (np.sqrt(v / (1 - b2 ** t)) + eps)
    return E


# ---------------------------------------------------------------------------
# adjoint
# ---------------------------------------------------------------------------

def adjoint(hstar, branch, rhs_tok, NS, cfg: Cfg, rhs_slot=None):
    """Clean Picard adjoint (`staged_adjoint_picard_clean.wgsl:143-248`) with
    optional Anderson mixing (`:1011-1135`).

    hstar, branch: [N,h,d] (branch = signal + attn*scale + anchor),
    rhs_tok: [N,d] (pooled dL/dH, scaled 1/h per slot) or None,
    rhs_slot: optional [N,h,d] added to the per-slot RHS.
    Returns v [N,h,d], g_pre = beta*J_norm^T v [N,h,d], pre, rms(pre).
    """
    N, h, d = hstar.shape
    beta = cfg.damping
    pre = np.asarray(branch, np.float64) + np.asarray(hstar, np.float64)
    r = np.sqrt(np.mean(pre * pre, -1) + 1e-6)
    inv = 1.0 / np.maximum(r, 1e-6)
    den = np.maximum(d * r ** 3, 1e-6)
    rhs = np.zeros((N, h, d))
    if rhs_tok is not None:
        rhs = rhs + (np.asarray(rhs_tok, np.float64) / max(1, h))[:, None, :]
    if rhs_slot is not None:
        rhs = rhs + np.asarray(rhs_slot, np.float64)
    NSb = np.asarray(NS, np.float64)[None, None, :]

    def norm_grad(v):
        up = beta * v
        coeff = (up * NSb * pre).sum(-1)
        return NSb * inv[..., None] * up - pre * (coeff / den)[..., None]

    v = rhs.copy()
    m = cfg.anderson_m
    hist = [np.zeros_like(v) for _ in range(m)] if m > 0 else []
    for k in range(cfg.adj_iters):
        v = rhs + (norm_grad(v) + (1.0 - beta) * v)
        if m > 0:
            hist[k % m] = v.copy()
            n_res = min(k, m - 1)
            if k >= 2 and n_res >= 2:
                v = _anderson_mix(hist, k, m, n_res)
    return v, norm_grad(v), pre, r


def anderson_fwd_gamma(A, rhs, n):
    """Forward Anderson step (no counterpart in the reference forward).

    Type-II Anderson acceleration in the difference form of Walker & Ni
    (SIAM J. Numer. Anal. 49(4), 2011): with residuals f_i = g(x_i) - x_i of
    the last n + 1 iterations and differences D_i = f_i - f_{i+1}, gamma
    minimises |f_0 - sum_i gamma_i D_i| (normal equations A gamma = rhs,
    A = D^T D [..., 2, 2], rhs = D^T f_0 [..., 2], n = 1 or 2), regularised with
    1e-3 * trace(A) on the diagonal; the next iterate is
    g_0 - sum_i gamma_i (g_i - g_{i+1}).  Returns (gamma [..., 2], ok): ok is
    False (plain Picard step) for a zero trace or any |gamma_i| > 20.
    """
    if n == 1:
        tr = A[..., 0, 0]
        ok = tr > 0
        a = A[..., 0, 0] + 1e-3 * tr
        gam = np.zeros(A.shape[:-2] + (2,))
        gam[..., 0] = rhs[..., 0] / np.where(ok, a, 1.0)
    else:
        tr = A[..., 0, 0] + A[..., 1, 1]
        ok = tr > 0
        lam = 1e-3 * tr
        a, b, c = A[..., 0, 0] + lam, A[..., 0, 1], A[..., 1, 1] + lam
        det = a * c - b * b
        ok &= det > 0
        idet = 1.0 / np.where(ok, det, 1.0)
        gam = np.stack([(c * rhs[..., 0] - b * rhs[..., 1]) * idet,
                        (a * rhs[..., 1] - b * rhs[..., 0]) * idet], -1)
    ok &= np.abs(gam).max(-1) <= 20.0
    return gam, ok


def _anderson_coefs(G, n_res):
    """Mixing weights from the Gram matrix of pseudo-residuals G [..., 3, 3]:
    Tikhonov term 1e-4*trace, Cramer solve with a floored determinant, clamp
    to [-2, 3], renormalise to sum 1 with a most-recent fallback
    (`staged_adjoint_picard_clean.wgsl:1075-1124`).  Returns [..., 3]."""
    beta = np.zeros(G.shape[:-2] + (3,))
    if n_res == 2:
        g00, g01, g10, g11 = G[..., 0, 0], G[..., 0, 1], G[..., 1, 0], G[..., 1, 1]
        reg = np.maximum(1e-8, 1e-4 * (np.abs(g00) + np.abs(g11)))
        g00 = g00 + reg
        g11 = g11 + reg
        det = g00 * g11 - g01 * g10
        sdet = np.where(det < 0, np.minimum(det, -1e-10), np.maximum(det, 1e-10))
        beta[..., 0] = (g11 - g01) / sdet
        beta[..., 1] = (g00 - g10) / sdet
    else:
        g = G.copy()
        reg = np.maximum(1e-8, 1e-4 * (np.abs(g[..., 0, 0]) + np.abs(g[..., 1, 1]) + np.abs(g[..., 2, 2])))
        for i in range(3):
            g[..., i, i] += reg
        g00, g01, g02 = g[..., 0, 0], g[..., 0, 1], g[..., 0, 2]
        g10, g11, g12 = g[..., 1, 0], g[..., 1, 1], g[..., 1, 2]
        g20, g21, g22 = g[..., 2, 0], g[..., 2, 1], g[..., 2, 2]
        det = (g00 * (g11 * g22 - g12 * g21) - g01 * (g10 * g22 - g12 * g20)
               + g02 * (g10 * g21 - g11 * g20))
        sdet = np.where(det < 0, np.minimum(det, -1e-8), np.maximum(det, 1e-8))
        beta[..., 0] = ((g11 * g22 - g12 * g21) - g01 * (g22 - g12) + g02 * (g21 - g11)) / sdet
        beta[..., 1] = (g00 * (g22 - g12) - (g10 * g22 - g12 * g20) + g02 * (g10 - g20)) / sdet
        beta[..., 2] = (g00 * (g11 - g21) - g01 * (g10 - g20) + (g10 * g21 - g11 * g20)) / sdet
    beta[..., :n_res] = np.clip(beta[..., :n_res], -2.0, 3.0)
    beta[..., n_res:] = 0.0
    ssum = beta.sum(-1)
    small = np.abs(ssum) < 1e-6
    beta = np.where(small[..., None], 0.0, beta / np.where(small, 1.0, ssum)[..., None])
    beta[small, 0] = 1.0
    return beta


def _anderson_mix(hist, k, m, n_res):
    """Adjoint mixing: per-token Gram over all h*d of the token (`:1049-1074`)."""
    N = hist[0].shape[0]
    deltas = [hist[(k + m - i) % m] - hist[(k + m - i - 1) % m] for i in range(n_res)]
    G = np.zeros((N, 3, 3))
    for i in range(n_res):
        for j in range(i, n_res):
            dot = (deltas[i] * deltas[j]).sum(axis=(1, 2))
            G[:, i, j] = dot
            G[:, j, i] = dot
    beta = _anderson_coefs(G, n_res)
    out = np.zeros_like(hist[0])
    for i in range(n_res):
        out += beta[:, i][:, None, None] * hist[(k + m - i) % m]
    return out


def source_grad(g_pre):
    """dL/dsignal pooled over slots (`picard_source_grad_reduce_main`, `:250-327`)."""
    return g_pre.sum(axis=1)


# ---------------------------------------------------------------------------
# weight gradients (analytic)
# ---------------------------------------------------------------------------

def weight_grads(S_flat, signal, A, cache, v, g_pre, pre, r_pre, W, cfg: Cfg):
    """dL/dtheta for every DEQ-core parameter, in the AllWeights layout.

    S_flat [N,d]; signal, A, v, g_pre, pre [N,h,d]; r_pre [N,h]; cache from
    `slot_attention` on the same N tokens.  Returns (G, dS_in).
    """
    d, h = cfg.d, cfg.h
    V = View(W, d, h)
    L = V.L
    hd = V.hd
    G = np.zeros(L.total)
    beta = cfg.damping
    gNS = (beta * v * pre / np.maximum(r_pre, 1e-6)[..., None]).sum(axis=(0, 1))
    G[L.nscale:L.nscale + d] = gNS
    dsig = g_pre.copy()                 # dL/dsignal
    if cfg.slot_coord:
        c = cache
        gA = g_pre
        a, rho, R, scale = c['a'], c['rho'], c['R'], c['scale']
        rhoc = np.maximum(rho, 1e-6)
        dscale = (gA * a).sum(-1)
        da = gA * scale[..., None]
        drho = np.where(rho > 1e-6, -dscale * scale / rhoc, 0.0)
        da += (drho / (d * rho))[..., None] * a
        dR = np.where(R > 1e-3, dscale / rhoc, 0.0)
        src = c['src']
        dsrc = (dR / (d * R))[..., None] * src
        n = c['n']
        dn = es('sco,nso->nsc', V.Wo[:, :hd, :], da)
        gWo = es('nsc,nso->sco', n, da)
        rr = c['r']
        dmix = (dn - n * ((n * dn).sum(-1) / hd)[..., None]) / rr[..., None]
        alpha, K, Vv, Q = c['alpha'], c['K'], c['V'], c['Q']
        dalpha = es('nsc,nkc->nsk', dmix, Vv)
        dV = es('nsk,nsc->nkc', alpha, dmix) - dmix.sum(1, keepdims=True) / h
        dlog = alpha * (dalpha - (alpha * dalpha).sum(-1, keepdims=True))
        gain = 2.0 / math.sqrt(max(1, hd))
        dQ = es('nsk,nkc->nsc', dlog, K) * gain
        dK = es('nsk,nsc->nkc', dlog, Q) * gain
        gWq = es('nsj,nsc->sjc', src, dQ)
        gWk = es('nsj,nsc->sjc', src, dK)
        gWv = es('nsj,nsc->sjc', src, dV)
        dsrc += (es('sjc,nsc->nsj', V.Wq[:, :, :hd], dQ)
                 + es('sjc,nsc->nsj', V.Wk[:, :, :hd], dK)
                 + es('sjc,nsc->nsj', V.Wv[:, :, :hd], dV))
        G[L.wq:L.wq + h * d * d].reshape(h, d, d)[:, :, :hd] = gWq
        G[L.wk:L.wk + h * d * d].reshape(h, d, d)[:, :, :hd] = gWk
        G[L.wv:L.wv + h * d * d].reshape(h, d, d)[:, :, :hd] = gWv
        G[L.wo:L.wo + h * d * d].reshape(h, d, d)[:, :hd, :] = gWo
        G[L.q_bias:L.q_bias + h * d].reshape(h, d)[:, :hd] = dQ.sum(0)
        G[L.k_bias:L.k_bias + h * d].reshape(h, d)[:, :hd] = dK.sum(0)
        dsig += dsrc
        G[L.slot_anchor:L.slot_anchor + h * d] = dsig.sum(0).ravel()
    if cfg.fpm and cfg.assoc:
        # the associative slots' branch holds the payload, not their signal
        # (`:2497`), so the direct term reaches W_in and S_in from the lower slots only
        dsig = dsig - np.where((np.arange(h) >= h // 2)[None, :, None], g_pre, 0.0)
    if not V.signal_zero:
        G[L.win:L.win + h * d * d] = (es('nj,nso->sjo', S_flat, dsig) * V.sig_scale).ravel()
        dS = es('sjo,nso->nj', V.Win, dsig) * V.sig_scale
    else:
        dS = np.zeros_like(S_flat)
    return G, dS


# ---------------------------------------------------------------------------
# FPM memory backward (reverse scan over the write recurrence)
# ---------------------------------------------------------------------------

FPM_READ_GRAD_SCALE = 0.5


def fpm_backward(hstar, signal, hist, v, W, d, h, carry=None):
    """Reverse-time backward of the FPM memory write, as the reference computes it
    (`aideen-backbone/src/shaders/fused_fpm_retain_bwd.wgsl:364-2095`), followed
    by the shared W_out / diag W_x gradients (`fused_fpm_shared_update.wgsl:
    129-158, 225-256`, the entry points bound at `gpu_deq.rs:1811,1820`).

    hstar, signal, hist: [B,T,h,d] (hist[t] = memory after the write of token t);
    v: adjoint solution [B*T,h,d]; carry: dL/dM seed [B,h,d] from the following
    chunk (TBPTT carry, zero after a state reset).

    The reference's formulas are kept as they are, including where they are not
    the exact derivative of `fpm_write`: x_proj is rebuilt as
    h_unit + wx*h_unit + write (no sqrt(z) factor) for m_inner and the a_log term,
    the novelty gradient is applied per dimension, W_x's carrier gradient omits
    the (1 - retain) factor, the read path contributes 0.5 * v[t] to dL/dM[t-1],
    and m_prev is zero at t = 0 of the chunk.  The W_k_write / W_v_write updates
    (compiled out: ENABLE_FPM_WRITE_BWD = false, FPM_DIRECT_WRITE_SCALE = 0)
    contribute nothing.  With the associative branch on, `signal` is the stored
    signal the reference reads here (`:399`), the payload on the associative
    slots.  Of the branch's own parameter gradients (`:475-1290`) only alpha_assoc
    is nonzero under the default flags (`assoc_alpha_grad`, added by
    `train_step`): with one bank the read's score gradient p * (g - p g) is 0,
    so the address weights get nothing (`:976, 1266`), the event-gate factor
    gate * (1 - gate) is 0 with the gate off (`:964`), and the value gradient
    reaches no parameter.

    Gradients are returned as raw sums over all sequences and tokens, in the
    AllWeights layout; the reference's per-family divisors (B*T for the slot
    parameters, B*T*h for W_out and W_x) are learning-rate factors left to the
    update's grad_scale.  Returns dict(G, carry, dm, minner, hunit, gx).
    """
    V = View(W, d, h)
    L = V.L
    hstar = np.asarray(hstar, np.float64)
    signal = np.asarray(signal, np.float64)
    hist = np.asarray(hist, np.float64)
    B, T = hstar.shape[:2]
    v = np.asarray(v, np.float64).reshape(B, T, h, d)
    v = np.where(np.isfinite(v), v, 0.0)
    g = np.zeros((B, h, d)) if carry is None else np.asarray(carry, np.float64).copy()
    inv_sqrt_d = 1.0 / math.sqrt(max(1, d))
    wx = 0.5 * np.tanh(np.diag(V.Wx))[None, None, :]
    a = 1.0 / (1.0 + np.exp(V.Alog))[None]                      # [1,h,d]
    gWup = np.zeros((h, d, RANK)); gWdown = np.zeros((h, RANK, d))
    gbret = np.zeros((h, d)); gbd = np.zeros((h, d)); gwf = np.zeros((h, d))
    gbw = np.zeros(h); galog = np.zeros((h, d))
    dm_all = np.zeros((B, T, h, d)); minner_all = np.zeros_like(dm_all)
    hunit_all = np.zeros_like(dm_all); gx_all = np.zeros_like(dm_all)
    for t in range(T - 1, -1, -1):
        c = 0.5 * (hstar[:, t] + signal[:, t])
        m_prev = hist[:, t - 1] if t > 0 else np.zeros((B, h, d))
        up = es('bsj,sjr->bsr', c, V.Wup)
        retain = 1.0 / (1.0 + np.exp(-(V.bret[None] + es('bsr,srd->bsd', up, V.Wdown))))
        kw = es('bsj,sjr->bsr', c, V.Wkw)
        prop = np.tanh(V.bdelta[None] + es('bsr,srd->bsd', kw, V.Wvw))
        raw_z = 1.0 / (1.0 + np.exp(-((c * V.wgate[None]).sum(-1) * inv_sqrt_d + V.bwrite[None] + FPM_GATE_BIAS)))
        prev_norm = np.sqrt(np.maximum((m_prev * m_prev).sum(-1), 1e-6))
        diff = prop - m_prev
        diff_norm = np.sqrt(np.maximum((diff * diff).sum(-1), 1e-6))
        denom = diff_norm + prev_norm + 1e-6
        nov = (diff_norm / denom)[..., None]
        z = np.clip(raw_z, 0.0, 1.0)[..., None]
        dnov_ddiff = (prev_norm / denom ** 2)[..., None]
        dnov_dprev = (-diff_norm / denom ** 2)[..., None]
        h_rms = np.sqrt(np.maximum((hstar[:, t] ** 2).sum(-1) / max(1, d), 1e-6))
        hu = hstar[:, t] / h_rms[..., None]
        ret_eff = 1.0 - nov * (1.0 - retain)
        x_proj = hu + wx * hu + z * FPM_RESIDUAL_SCALE * prop
        base = a * m_prev + (1.0 - a) * x_proj
        m_inner = ret_eff * m_prev + (1.0 - ret_eff) * base
        g_x = (1.0 - a) * (1.0 - ret_eff) * g
        g_prev = ret_eff * g + (1.0 - ret_eff) * a * g
        q = nov * retain * (1.0 - retain)
        g_pre = (m_prev - base) * g * q
        g_z = (g_x * (FPM_RESIDUAL_SCALE * prop + 0.5 * hu / np.sqrt(np.maximum(z, 1e-6)))).sum(-1)
        g_raw_z = g_z * raw_z * (1.0 - raw_z)
        dm_all[:, t], minner_all[:, t], hunit_all[:, t] = g, m_inner, hu
        gx_all[:, t] = (1.0 - a) * g
        g_re = g_pre / np.maximum(q, 1e-6)
        g_nov = -g_re * (1.0 - retain)
        g_dn = g_nov * dnov_ddiff
        g_pn = g_nov * dnov_dprev
        unit_diff = diff / np.maximum(diff_norm, 1e-6)[..., None]
        g_prop = g_x * z * FPM_RESIDUAL_SCALE + g_dn * unit_diff
        g_prev = g_prev + g_pn * m_prev / np.maximum(prev_norm, 1e-6)[..., None] - g_dn * unit_diff
        g_a = (1.0 - ret_eff) * (m_prev - x_proj) * g
        galog += (-a * (1.0 - a) * g_a).sum(0)
        gbd += (g_prop * (1.0 - prop * prop)).sum(0)
        gbret += g_pre.sum(0)
        dup = es('bsd,srd->bsr', g_pre, V.Wdown)
        gWdown += es('bsr,bsd->srd', up, g_pre)
        gWup += es('bsd,bsr->sdr', c, dup)
        gwf += (g_raw_z[..., None] * c).sum(0) * inv_sqrt_d
        gbw += g_raw_z.sum(0)
        g = g_prev + FPM_READ_GRAD_SCALE * v[:, t]
    G = np.zeros(L.total)
    G[L.w_retain_up:L.w_retain_up + h * d * RANK] = gWup.ravel()
    G[L.w_retain_down:L.w_retain_down + h * RANK * d] = gWdown.ravel()
    G[L.b_retain:L.b_retain + h * d] = gbret.ravel()
    G[L.b_delta:L.b_delta + h * d] = gbd.ravel()
    G[L.w_write_gate:L.w_write_gate + h * d] = gwf.ravel()
    G[L.b_write_mem:L.b_write_mem + h] = gbw
    G[L.alog:L.alog + h * d] = galog.ravel()
    gwout = es('btsr,btsc->rc', dm_all, minner_all)
    G[L.wout:L.wout + d * d] = gwout.ravel()
    wraw = np.diag(V.Wx)
    gwx = (gx_all * hunit_all).sum((0, 1, 2)) * 0.5 * (1.0 - np.tanh(wraw) ** 2)
    G[L.wx + np.arange(d) * (d + 1)] = gwx
    return dict(G=G, carry=g, dm=dm_all, minner=minner_all, hunit=hunit_all, gx=gx_all)


# ---------------------------------------------------------------------------
# optimizers and spectral renorm
# ---------------------------------------------------------------------------

def adam(w, g, m, v, t, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, grad_scale=1.0):
    """`Adam::step_matrix_scaled_inplace` (`optimizer.rs:105-183`)."""
    w = np.asarray(w, np.float64).copy()
    g = np.asarray(g, np.float64) * grad_scale
    m = b1 * np.asarray(m, np.float64) + (1 - b1) * g
    v = b2 * np.asarray(v, np.float64) + (1 - b2) * g * g
    tt = max(1, t)
    bc1 = 1 - b1 ** tt
    bc2 = 1 - b2 ** tt
    w -= lr * (m / bc1) / (np.sqrt(v / bc2) + eps)
    return w, m, v


def clipped_sgd(w, g, lr, wd, main_len, grad_scale=1.0):
    """`apply_grad_update_main` (`fused_deq_update.wgsl:809-823`) with the
    lr*grad_scale product of the stage kernels (`:402-410`)."""
    w = np.asarray(w, np.float64).copy()
    step = lr * np.asarray(g, np.float64) * grad_scale
    mult = np.ones_like(w)
    mult[:main_len] = 1.0 - lr * wd
    return w * mult - np.clip(step, -0.5, 0.5)


def spectral_renorm(W, d, h, n_iters=12, attn=0.10, win=0.30, fpm=0.70, wv=0.50, wo=0.50):
    """`spectral_renorm_main` for every matrix index (`spectral_renorm.wgsl:83-196`).

    Row-major view A[r][c] = flat[r*d + c]; v = A^T u / |.|, u = A v,
    sigma = sqrt(|u|^2 + 1e-12).  Returns the new weights and the sigmas.
    """
    W = np.asarray(W, np.float64).copy()
    L = Offsets(d, h)
    mats = []
    for base, thr in ((L.wq, attn), (L.wk, attn), (L.wv, wv), (L.wo, wo), (L.win, win)):
        for s in range(h):
            mats.append((base + s * d * d, thr))
    mats.append((L.wx, fpm))
    mats.append((L.wout, fpm))
    sigmas = []
    for off, thr in mats:
        A = W[off:off + d * d].reshape(d, d)
        u = np.full(d, 1.0 / math.sqrt(d))
        sigma = 1.0
        for _ in range(n_iters):
            vv = A.T @ u
            vv = vv / math.sqrt((vv * vv).sum() + 1e-12)
            uu = A @ vv
            sigma = math.sqrt((uu * uu).sum() + 1e-12)
            u = uu / sigma
        sigmas.append(sigma)
        if sigma > thr:
            W[off:off + d * d] = (A * (thr / sigma)).ravel()
    return W, np.array(sigmas)


# ---------------------------------------------------------------------------
# one full training step
# ---------------------------------------------------------------------------

def branch_of(fwd: ForwardOut, W, cfg: Cfg):
    V = View(W, cfg.d, cfg.h)
    sig = fwd.signal if fwd.branch_signal is None else fwd.branch_signal
    if cfg.slot_coord:
        return sig + fwd.A + V.anchor[None, None]
    return sig.copy()


def train_step(S_in, targets, W, lm, cfg: Cfg, adam_state=None, step=1, lr=1e-3,
               mstate=None, fpm_carry=None, lm_samples=0, sample_seed=LM_SAMPLE_SEED,
               lm_state=None, tokens=None, emb=None, emb_state=None, emb_grad="dl_dh", assoc_state=None):
    """Forward -> LM head -> adjoint -> weight grads -> Adam (DEQ core and LM head).

    lm_samples = 0: dense full-vocabulary CE; the LM-head gradients join the
    common Adam step.  lm_samples > 0: the reference's sampled-softmax head with
    its own fused Adam step inside the LM stage (`lm_head_sampled`, sampled set
    from `sampled_indices`).  With `emb` and `tokens`, the embedding rows of the
    step's tokens get the reference's Adam update (`embedding_update`) from
    the LM head's dL/dpooled rows (emb_grad="dl_dh", trainer.rs:3285-3289
    default) or the exact dL/dS_in (emb_grad="ds_in").

    Returns a dict with every intermediate the GPU path is compared on.
    """
    B, T, d = S_in.shape
    h = cfg.h
    N = B * T
    fwd = forward(S_in, W, cfg, mstate, assoc_state)
    w_lm, b_lm, g_lm = lm
    tg = np.asarray(targets).reshape(N)
    sampled = None
    if lm_samples > 0:
        V = np.asarray(w_lm).shape[0]
        if lm_state is None:
            lm_state = dict(mW=np.zeros((V, d)), vW=np.zeros((V, d)), mb=np.zeros(V), vb=np.zeros(V))
        sampled = sampled_indices(tg, step, V, lm_samples, sample_seed)
        loss, dP, w_new, b_new, dW_s, db_s = lm_head_sampled(fwd.pooled.reshape(N, d), tg, w_lm, b_lm, g_lm,
                                                             sampled, lm_state, step, lr=lr)
        lm_new = np.concatenate([w_new.ravel(), b_new, np.asarray(g_lm, np.float64)])
        lm_g = (dW_s, db_s)
    else:
        loss, dP, gW_lm, gb_lm, gg_lm = lm_head(fwd.pooled.reshape(N, d), tg, w_lm, b_lm, g_lm)
    br = branch_of(fwd, W, cfg).reshape(N, h, d)
    V_ = View(W, d, h)
    v, g_pre, pre, r_pre = adjoint(fwd.hstar.reshape(N, h, d), br, dP, V_.NS, cfg)
    G, dS = weight_grads(np.asarray(S_in, np.float64).reshape(N, d),
                         fwd.signal.reshape(N, h, d), fwd.A.reshape(N, h, d), fwd.attn_cache,
                         v, g_pre, pre, r_pre, W, cfg)
    fpm_out = None
    if cfg.fpm:
        # the reference's FPM backward reads the stored signal (fused_fpm_retain_bwd.wgsl:399),
        # the payload on associative slots
        fpm_out = fpm_backward(fwd.hstar, fwd.branch_signal, fwd.hist_ctx, v, W, d, h, carry=fpm_carry)
        G = G + fpm_out["G"]
        if cfg.assoc:
            L_ = Offsets(d, h)
            G[L_.alpha_assoc:L_.alpha_assoc + h] += assoc_alpha_grad(fwd.assoc_read, v, W, d, h)
    if adam_state is None:
        adam_state = (np.zeros_like(G), np.zeros_like(G))
    Wn, m1, m2 = adam(W, G, adam_state[0], adam_state[1], step, lr=lr)
    if lm_samples <= 0:
        lm_flat = np.concatenate([np.ravel(w_lm), np.ravel(b_lm), np.ravel(g_lm)]).astype(np.float64)
        lm_g = np.concatenate([gW_lm.ravel(), gb_lm, gg_lm])
        lm_new, _, _ = adam(lm_flat, lm_g, np.zeros_like(lm_g), np.zeros_like(lm_g), step, lr=lr)
    emb_new = None
    if emb is not None and tokens is not None:
        if emb_state is None:
            emb_state = dict(m=np.zeros(np.shape(emb)), v=np.zeros(np.shape(emb)))
        rows = dP if emb_grad == "dl_dh" else dS
        emb_new = embedding_update(emb, np.asarray(tokens).reshape(N), rows, emb_state, step, lr=lr)
    return dict(fwd=fwd, loss=loss, dP=dP, v=v, g_pre=g_pre, grads=G, dS=dS, W_new=Wn,
                adam=(m1, m2), lm_grads=lm_g, lm_new=lm_new, fpm=fpm_out, sampled=sampled,
                emb_new=emb_new)
