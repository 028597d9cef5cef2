"""Shared comparison of one training step of the CUDA path with the oracle.

Used by the GPU parity tests; the oracle is only the checker here.
"""
from __future__ import annotations

import numpy as np

from oracle import deq_oracle as O

TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def grad_blocks(d, h, fpm):
    """Gradient segments of AllWeights compared one by one (name -> [a, b))."""
    L = O.Offsets(d, h)
    blocks = dict(wq=(L.wq, L.q_bias), qb=(L.q_bias, L.wk), wk=(L.wk, L.k_bias), kb=(L.k_bias, L.wv),
                  wv=(L.wv, L.wo), wo=(L.wo, L.win), win=(L.win, L.wx), ns=(L.nscale, L.hist),
                  anchor=(L.slot_anchor, L.w_k_write))
    if fpm:
        blocks.update(wup=(L.w_retain_up, L.w_retain_down), wdown=(L.w_retain_down, L.b_retain),
                      bret=(L.b_retain, L.w_q_mem), bdelta=(L.b_delta, L.flags),
                      wgate=(L.w_write_gate, L.b_write_mem), bwrite=(L.b_write_mem, L.hhist_gamma),
                      alog=(L.alog, L.nscale), wout=(L.wout, L.alog), wx=(L.wx, L.wout))
    return blocks


def step_errors(be, r, W, lm, B, T, lr=1e-3, step=1):
    """Relative L2 errors of everything one `aideen_train_step` leaves behind,
    against the oracle's `train_step` result `r` on the same inputs.

    The Adam update is checked in two parts: the kernel (the oracle's Adam
    applied to the GPU's own gradients, which must agree to fp32 rounding) and
    the gradients feeding it (1e-3 like every other quantity).  The update
    W_new - W itself is reported too: at step 1 it is lr*g/(|g| + eps), about
    lr*sign(g), so gradient entries whose magnitude is below the 1e-4-level
    agreement of the two gradients flip sign and dominate that difference.
    """
    d, h = be.d, be.h
    N = B * T
    fwd = r["fwd"]
    e = {}
    e["hstar"] = rel(be.read_hnext_seq(), fwd.hstar)
    e["pooled"] = rel(be.read_hpooled_seq(), fwd.pooled)
    its = be.read("iters", (B, T, h), np.int32)
    e["iters_mismatch"] = float((its != fwd.iters).mean())
    e["dl_dh"] = rel(be.read("dl_dh", (N, d)), r["dP"])
    e["v"] = rel(np.transpose(be.read_adj_v_out(), (1, 0, 2)), r["v"])
    Gg = be.read_grads()
    G = r["grads"]
    for name, (a, b) in grad_blocks(d, h, fwd.hist_ctx.any()).items():
        e["g_" + name] = rel(Gg[a:b], G[a:b])
    lm_g = be.read("lm_grads", (r["lm_grads"].size,))
    e["lm_grads"] = rel(lm_g, r["lm_grads"])
    Wn = be.read_weights()
    W_kernel, _, _ = O.adam(W, Gg, np.zeros_like(G), np.zeros_like(G), step, lr=lr)
    # both sides rounded to the fp32 weights the GPU stores
    e["adam_kernel"] = rel(Wn.astype(np.float64) - W, W_kernel.astype(np.float32).astype(np.float64) - W)
    e["update"] = rel(Wn.astype(np.float64) - W, r["W_new"] - W)
    lw, lb, lg = be.read_lm_head()
    lm_new = np.concatenate([lw.ravel(), lb, lg]).astype(np.float64)
    lm_old = np.concatenate([np.ravel(x) for x in lm]).astype(np.float64)
    lm_kernel, _, _ = O.adam(lm_old, lm_g, np.zeros_like(lm_old), np.zeros_like(lm_old), step, lr=lr)
    e["lm_adam_kernel"] = rel(lm_new - lm_old, lm_kernel.astype(np.float32).astype(np.float64) - lm_old)
    return e


def assert_step(e, loss, r, tol=TOL, iters_mismatch=0.0):
    assert abs(loss - r["loss"]) / abs(r["loss"]) < tol, (loss, r["loss"])
    assert e["iters_mismatch"] <= iters_mismatch, e
    bad = {k: v for k, v in e.items()
           if k not in ("iters_mismatch", "update", "adam_kernel", "lm_adam_kernel") and not v < tol}
    assert not bad, bad
    assert e["adam_kernel"] < 1e-4 and e["lm_adam_kernel"] < 1e-4, e
