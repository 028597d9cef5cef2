"""Checkpoint wire formats (.aidn bincode container, .opt Adam state) on the host."""
import struct

import numpy as np

from aideen_b200 import checkpoint as ck
from aideen_b200.layout import Layout
from aideen_b200.weights import init_all_weights, init_embedding, init_lm_head


def test_aidn_round_trip_and_byte_layout(tmp_path):
    d, h, V = 128, 4, 37
    W = init_all_weights(d, h, seed=1)
    lm, emb = init_lm_head(d, V), init_embedding(d, V)
    m = ck.full_model(W, d, h, lm, emb, config=dict(ctx_len=64), metadata=dict(note="x"))
    p = tmp_path / "m.aidn"
    m.save(str(p))
    raw = p.read_bytes()
    # bincode 1: the config's first field d_m = 1024 as u64 LE, d_r second
    assert struct.unpack_from("<QQ", raw, 0) == (1024, d)
    m2 = ck.AidenModel.load(str(p))
    assert m2.config["d_r"] == d and m2.config["h_slots"] == h and m2.config["ctx_len"] == 64
    assert m2.config["train_deq"] is True and abs(m2.config["deq_epsilon"] - 1e-4) < 1e-9
    w2, lm2, emb2 = ck.unpack_full_model(m2)
    assert np.array_equal(w2, W)
    assert np.array_equal(lm2[0], lm[0]) and np.array_equal(lm2[1], lm[1]) and np.array_equal(lm2[2], lm[2])
    assert np.array_equal(emb2, emb)
    assert m2.metadata["gpu_exact_checkpoint"] == "true" and m2.metadata["note"] == "x"
    # W_q carries q_bias, hist_params is the tail after NormScale
    L = Layout(d, h)
    assert m2.weights["reasoning.gpu_exact.w_q"].size == h * d * d + h * d
    assert m2.weights["reasoning.gpu_exact.hist_params"].size == L.total - L.hist
    # the embeddings are an nalgebra vocab x d matrix: column-major
    assert np.array_equal(m2.weights["tokenizer.embeddings"][:V], emb[:, 0])


def test_aidn_rejects_trailing_bytes(tmp_path):
    m = ck.AidenModel()
    raw = m.to_bytes() + b"\0"
    try:
        ck.AidenModel.from_bytes(raw)
    except ValueError:
        return
    raise AssertionError("trailing bytes accepted")


def test_opt_round_trip_and_truncation(tmp_path):
    d, h = 128, 2
    L = Layout(d, h)
    rng = np.random.default_rng(0)
    mc, vc = rng.standard_normal(L.total).astype(np.float32), rng.random(L.total).astype(np.float32)
    ml, vl = rng.standard_normal(50).astype(np.float32), rng.random(50).astype(np.float32)
    p = tmp_path / "a.opt"
    ck.save_opt(str(p), 17, ck.adam_tensors(mc, vc, d, h, ml, vl))
    raw = p.read_bytes()
    assert raw[:8] == b"AIDENOPT" and struct.unpack_from("<Q", raw, 8)[0] == 17
    step, t = ck.load_opt(str(p))
    mc2, vc2, ml2, vl2 = ck.adam_from_tensors(t, d, h)
    assert step == 17 and np.array_equal(mc2, mc) and np.array_equal(vc2, vc)
    assert np.array_equal(ml2, ml) and np.array_equal(vl2, vl)
    # like load_state, a cut-off last entry ends the read without an error
    p.write_bytes(raw[:-7])
    step, t2 = ck.load_opt(str(p))
    assert len(t2) == len(t) - 1
