"""Loop-level restatements of the CPU maps in the reference's own pipeline test
(aideen-backbone/tests/picard_pipeline_test.rs), used to pin the oracle where
the two describe the same function.  Test infrastructure only."""
from __future__ import annotations

import numpy as np


def _rms(v):
    return np.sqrt(np.mean(v * v) + 1e-6)


def cpu_signal(s_in, w_in, d):
    """`cpu_signal` (picard_pipeline_test.rs:156-166): out[o] = sum_j w_in[j*d + o] s[j]."""
    return np.array([sum(w_in[j * d + o] * s_in[j] for j in range(d)) for o in range(d)])


def cpu_forward_map_no_fpm(h, s_in, w_q, w_k, w_v, w_o, w_in, norm, damping, h_slots, d):
    """`cpu_forward_map_no_fpm` (picard_pipeline_test.rs:168-261): one damped map
    with h-dependent full-width attention (shared W_q/W_k/W_v/W_o, scores scaled
    by 1/sqrt(d) and clamped to [-4, 4]), combined = attn + signal, RMS-normalised."""
    scale = 1.0 / max(np.sqrt(d), 1.0)
    sig = cpu_signal(s_in, w_in, d)
    W = lambda w: np.asarray(w, np.float64).reshape(d, d)   # [j][o]
    H = np.asarray(h, np.float64).reshape(h_slots, d)
    q, k, v = H @ W(w_q), H @ W(w_k), H @ W(w_v)
    out = np.zeros((h_slots, d))
    for qs in range(h_slots):
        sc = np.clip((k @ q[qs]) * scale, -4.0, 4.0)
        e = np.exp(sc - sc.max())
        aw = e / max(e.sum(), 1e-12)
        mix = aw @ v
        comb = mix @ W(w_o) + sig
        r = np.sqrt((comb * comb).sum() / d + 1e-6)
        out[qs] = damping * (np.asarray(norm) * comb / r) + (1 - damping) * H[qs]
    return out.ravel()


def cpu_hist_gated_forward_no_attn(s_in, w_in, w_hist, hist_slot_scale, hist_gate_logit, slot_anchor, w_x, w_out,
                                   a_log, norm, damping, h_slots, d):
    """`cpu_hist_gated_forward_no_attn` (picard_pipeline_test.rs:59-154, carrier =
    the previous memory): one damped step per token from a token-fixed history
    context, then the memory update x = a*m + (1-a)*(h_u + W_x^T h_u),
    m' = x + W_out^T x (full W_x; the shared a_log [d])."""
    T = len(s_in) // d
    h_curr = np.zeros(h_slots * d)
    m_prev = np.zeros(h_slots * d)
    h_out = np.zeros(T * h_slots * d)
    Wx = np.asarray(w_x, np.float64).reshape(d, d)
    Wo = np.asarray(w_out, np.float64).reshape(d, d)
    Wh = np.asarray(w_hist, np.float64).reshape(d, d)
    for t in range(T):
        inj = cpu_signal(s_in[t * d:(t + 1) * d], w_in, d)
        inj_rms = _rms(inj)
        hist = np.zeros(h_slots * d)
        for s in range(h_slots):
            off = s * d
            car = np.zeros(d) if t == 0 else m_prev[off:off + d]
            cr = _rms(car)
            u = np.asarray(hist_slot_scale[off:off + d]) * (car / cr) + Wh @ (car / cr)
            hs = min(inj_rms / max(_rms(u), 1e-6), 1.0)
            alpha = 0.08 + 0.20 / (1.0 + np.exp(-hist_gate_logit[s]))
            hist[off:off + d] = alpha * u * hs
        for s in range(h_slots):
            off = s * d
            comb = inj + hist[off:off + d] + np.asarray(slot_anchor[off:off + d])
            f = np.asarray(norm) * comb / _rms(comb)
            h_out[t * h_slots * d + off:t * h_slots * d + off + d] = damping * f + (1 - damping) * h_curr[off:off + d]
        h_curr = h_out[t * h_slots * d:(t + 1) * h_slots * d].copy()
        nm = np.zeros(h_slots * d)
        for s in range(h_slots):
            off = s * d
            hc = h_curr[off:off + d]
            hu = hc / _rms(hc)
            a = 1.0 / (1.0 + np.exp(np.asarray(a_log)))
            x = a * m_prev[off:off + d] + (1 - a) * (hu + Wx.T @ hu)
            nm[off:off + d] = x + Wo.T @ x
        m_prev = nm
    return h_out, m_prev
