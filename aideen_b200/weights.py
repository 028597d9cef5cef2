"""Seeded weight initialisation in the AllWeights layout.

Distributions follow `FixedPointMemoryReasoning::new_with_rng`
(`aideen-backbone/src/fixed_point_memory_reasoning.rs:249-462`) and the
per-slot replication of `*_gpu_flat` (`:476-574`):

* W_q, W_k, W_v, W_o, W_in: Xavier-uniform U(+-sqrt(3/d)), then scaled down to
  sigma <= threshold by 20 power iterations (`spectral_norm.rs:25-82`); one
  matrix replicated to every slot.
* W_x, W_out: U(+-0.01) (identity scale 0, `:283-284`).
* A_log: logit(a) with a spread over [0.80, 0.999] across slots (`:371-381`).
* NormScale = 1, slot anchor U(+-1) (`:225-232`), q/k bias = shared sin/cos
  slot code + U(+-0.005) (`:429-456`).
* FPM write/retain/read parameters as in `:290-424`.

The random stream is numpy's PCG64 seeded with `seed`; it does NOT reproduce
Rust's StdRng (ChaCha12) bit for bit, only the same distributions.
"""
from __future__ import annotations

import math

import numpy as np

from .layout import FLAG_DEFAULTS, RANK, Layout


def power_sigma(w: np.ndarray, n_iter: int = 20) -> float:
    """sigma_max of a square matrix by the reference's power iteration.

    `spectral_norm.rs:25-63`: u0 = 1/sqrt(rows); v = W^T u / |W^T u|;
    u = W v / |W v|; sigma = u^T W v.  Computed in float64.
    """
    w = np.asarray(w, dtype=np.float64)
    rows = w.shape[0]
    u = np.full(rows, 1.0 / math.sqrt(rows))
    sigma = 1.0
    for _ in range(n_iter):
        wtu = w.T @ u
        n = np.linalg.norm(wtu)
        if n < 1e-12:
            return 0.0
        v = wtu / n
        wv = w @ v
        n2 = np.linalg.norm(wv)
        if n2 < 1e-12:
            return 0.0
        u = wv / n2
        sigma = float(u @ w @ v)
    return max(abs(sigma), 1e-12)


def normalize_if_needed(w: np.ndarray, threshold: float, n_iter: int = 20) -> np.ndarray:
    """`spectral_norm.rs:76-82`."""
    s = power_sigma(w, n_iter)
    if s > threshold:
        w = w * (threshold / s)
    return w


def init_all_weights(d: int, h: int, seed: int = 0, *, attn_sigma: float = 0.85,
                     win_sigma: float = 0.85, signal_scale: float = 1.0) -> np.ndarray:
    """Build one AllWeights vector (float32) for (d, h)."""
    L = Layout(d, h)
    rng = np.random.default_rng(seed)
    w = np.zeros(L.total, dtype=np.float64)
    xr = math.sqrt(3.0 / d)

    def xavier():
        return rng.uniform(-xr, xr, size=(d, d))

    wq = normalize_if_needed(xavier(), attn_sigma)
    wk = normalize_if_needed(xavier(), attn_sigma)
    wv = normalize_if_needed(xavier(), attn_sigma)
    wo = normalize_if_needed(xavier(), attn_sigma)
    win = normalize_if_needed(xavier(), win_sigma)
    dd = d * d
    for s in range(h):
        w[L.wq + s * dd: L.wq + (s + 1) * dd] = wq.ravel()
        w[L.wk + s * dd: L.wk + (s + 1) * dd] = wk.ravel()
        w[L.wv + s * dd: L.wv + (s + 1) * dd] = wv.ravel()
        w[L.wo + s * dd: L.wo + (s + 1) * dd] = wo.ravel()
        w[L.win + s * dd: L.win + (s + 1) * dd] = win.ravel()

    dims = np.arange(d)
    for s in range(h):
        theta = 2.0 * math.pi * s / max(h, 1)
        code = 0.08 * np.sin(theta + 0.047 * dims) + 0.08 * np.cos(theta + 0.089 * dims)
        w[L.q_bias + s * d: L.q_bias + (s + 1) * d] = code + rng.uniform(-0.005, 0.005, d)
        w[L.k_bias + s * d: L.k_bias + (s + 1) * d] = code + rng.uniform(-0.005, 0.005, d)

    w[L.wx: L.wx + dd] = rng.uniform(-0.01, 0.01, dd)
    w[L.wout: L.wout + dd] = rng.uniform(-0.01, 0.01, dd)
    for s in range(h):
        frac = 0.5 if h <= 1 else s / (h - 1)
        a = 0.80 + frac * (0.999 - 0.80)
        w[L.alog + s * d: L.alog + (s + 1) * d] = math.log(a / (1.0 - a))
    w[L.nscale: L.nscale + d] = 1.0

    w[L.hist_mat: L.hist_mat + dd] = (0.15 * np.eye(d) + rng.uniform(-0.01, 0.01, (d, d))).ravel()
    cen = np.arange(h) - (h - 1) * 0.5
    w[L.hist_scale: L.hist_scale + h * d] = (cen[:, None] * 5e-5 + rng.uniform(-1e-4, 1e-4, (h, d))).ravel()
    w[L.hist_bias: L.hist_bias + h * d] = (cen[:, None] * 2.5e-3 + rng.uniform(-5e-4, 5e-4, (h, d))).ravel()
    w[L.hist_gate: L.hist_gate + h] = -1.204 + cen * 0.02
    w[L.slot_anchor: L.slot_anchor + h * d] = rng.uniform(-1.0, 1.0, h * d)
    w[L.w_k_write: L.w_k_write + h * d * RANK] = rng.uniform(-0.01, 0.01, h * d * RANK)
    w[L.w_v_write: L.w_v_write + h * RANK * d] = rng.uniform(-0.01, 0.01, h * RANK * d)
    w[L.flags: L.flags + len(FLAG_DEFAULTS)] = FLAG_DEFAULTS
    w[L.signal_scale] = signal_scale
    w[L.b_write_mem: L.b_write_mem + h] = cen * 0.02
    w[L.hhist_gamma: L.hhist_gamma + h] = -2.0
    w[L.w_retain_up: L.w_retain_up + h * d * RANK] = rng.uniform(-0.01, 0.01, h * d * RANK)
    mr = math.sqrt(3.0 / max(d, 1))
    qmem = rng.uniform(-mr, mr, (h, d * RANK))
    w[L.w_q_mem: L.w_q_mem + h * d * RANK] = qmem.ravel()
    w[L.w_k_mem: L.w_k_mem + h * d * RANK] = (qmem + rng.uniform(-0.1 * mr, 0.1 * mr, qmem.shape)).ravel()
    w[L.b_read_mem: L.b_read_mem + h] = cen * 0.02 + rng.uniform(-5e-4, 5e-4, h)
    kassoc = rng.uniform(-0.01, 0.01, h * d * RANK)
    w[L.w_k_assoc: L.w_k_assoc + h * d * RANK] = kassoc
    w[L.w_v_assoc: L.w_v_assoc + h * d * RANK] = rng.uniform(-0.01, 0.01, h * d * RANK)
    w[L.w_q_assoc: L.w_q_assoc + h * d * RANK] = kassoc
    w[L.alpha_assoc: L.alpha_assoc + h] = math.log(0.7 / 0.3)
    return w.astype(np.float32)


def init_lm_head(d: int, vocab: int, seed: int = 1):
    """LM head W_lm [vocab][d] (Xavier), bias 0, RMSNorm gain 1."""
    rng = np.random.default_rng(seed)
    xr = math.sqrt(3.0 / d)
    w_lm = rng.uniform(-xr, xr, (vocab, d)).astype(np.float32)
    return w_lm, np.zeros(vocab, np.float32), np.ones(d, np.float32)


def init_embedding(d: int, vocab: int, seed: int = 2) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.uniform(-1.0, 1.0, (vocab, d)).astype(np.float32)


def zipf_tokens(n: int, vocab: int, s: float = 1.1, seed: int = 3) -> np.ndarray:
    """Token ids from Zipf(s) over [0, vocab) by inverse-CDF sampling (rank-ordered ids)."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    cdf = np.cumsum(p)
    cdf /= cdf[-1]
    u = rng.random(n)
    return np.searchsorted(cdf, u).astype(np.int32).clip(0, vocab - 1)
