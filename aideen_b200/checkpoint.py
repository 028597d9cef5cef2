"""Checkpoint files in the reference's wire formats.

* ``.aidn`` — `AidenModel` (aideen-core/src/model.rs:8-47) serialised with
  bincode 1's default encoding: little-endian fixed-width integers, ``usize``
  as u64, ``bool`` as one byte, strings and vectors prefixed by a u64 length,
  maps as a u64 count followed by key/value pairs, struct fields in
  declaration order.  ``ArchitectureConfig`` field order and types follow
  aideen-core/src/state.rs:7-35.  The weight names are the ones the reference
  trainer's `save_full` writes (aideen-training-lab/src/trainer.rs:6470-6530):
  the GPU-exact DEQ slices ``reasoning.gpu_exact.*`` of the AllWeights buffer
  (`deq_bridge.rs` read_weights: W_q and W_k carry their biases), the LM head
  ``head.w`` (row-major [vocab][d]), ``head.b``, ``head.g``, and the token
  embeddings ``tokenizer.embeddings`` (an nalgebra vocab x d matrix, i.e.
  column-major).
* ``.opt`` — `Adam::save_state` (aideen-training-lab/src/optimizer.rs:246-290):
  the magic ``AIDENOPT``, the step as u64, then per tensor a u32 key length,
  the UTF-8 key, a u32 element count and the f32 data (the writer emits no
  type byte, whatever its header comment says; the reader here follows the
  writer, like `load_state` :292-370).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from .layout import Layout

# ArchitectureConfig (state.rs:7-35): name, struct code
CONFIG_FIELDS = [
    ("d_m", "Q"), ("d_r", "Q"), ("d_c", "Q"), ("d_e", "Q"), ("d_sim", "Q"), ("h_slots", "Q"),
    ("vocab_size", "Q"), ("ctx_len", "Q"), ("max_deq_iters", "Q"), ("deq_epsilon", "f"),
    ("adj_iters", "Q"), ("train_deq", "?"), ("deq_grad_scale", "f"), ("renorm_every_steps", "Q"),
    ("num_samples", "Q"), ("weight_decay", "f"),
]
# ArchitectureConfig::default (state.rs:37-57)
CONFIG_DEFAULTS = dict(d_m=1024, d_r=512, d_c=256, d_e=256, d_sim=1024, h_slots=8, vocab_size=50257,
                       ctx_len=512, max_deq_iters=16, deq_epsilon=1e-4, adj_iters=2, train_deq=True,
                       deq_grad_scale=1.0, renorm_every_steps=4, num_samples=512, weight_decay=0.01)


class _W:
    def __init__(self):
        self.parts = []

    def pack(self, fmt, *v):
        self.parts.append(struct.pack("<" + fmt, *v))

    def string(self, s: str):
        b = s.encode("utf-8")
        self.pack("Q", len(b))
        self.parts.append(b)

    def f32s(self, a):
        a = np.ascontiguousarray(a, dtype="<f4").ravel()
        self.pack("Q", a.size)
        self.parts.append(a.tobytes())

    def bytes(self) -> bytes:
        return b"".join(self.parts)


class _R:
    def __init__(self, buf: bytes):
        self.b, self.o = buf, 0

    def unpack(self, fmt):
        v = struct.unpack_from("<" + fmt, self.b, self.o)
        self.o += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.unpack("Q")
        s = self.b[self.o:self.o + n].decode("utf-8")
        self.o += n
        return s

    def f32s(self) -> np.ndarray:
        n = self.unpack("Q")
        a = np.frombuffer(self.b, dtype="<f4", count=n, offset=self.o).astype(np.float32)
        self.o += 4 * n
        return a


@dataclass
class AidenModel:
    """The `.aidn` container: configuration, named f32 tensors, string metadata."""
    config: dict = field(default_factory=lambda: dict(CONFIG_DEFAULTS))
    weights: dict = field(default_factory=dict)
    metadata: dict = field(default_factory=dict)

    def to_bytes(self) -> bytes:
        w = _W()
        for name, code in CONFIG_FIELDS:
            w.pack(code, self.config[name])
        w.pack("Q", len(self.weights))
        for k, v in self.weights.items():
            w.string(k)
            w.f32s(v)
        w.pack("Q", len(self.metadata))
        for k, v in self.metadata.items():
            w.string(k)
            w.string(str(v))
        return w.bytes()

    @classmethod
    def from_bytes(cls, buf: bytes) -> "AidenModel":
        r = _R(buf)
        cfg = {name: r.unpack(code) for name, code in CONFIG_FIELDS}
        weights = {}
        for _ in range(r.unpack("Q")):
            k = r.string()
            weights[k] = r.f32s()
        meta = {}
        for _ in range(r.unpack("Q")):
            k = r.string()
            meta[k] = r.string()
        if r.o != len(buf):
            raise ValueError(f".aidn: {len(buf) - r.o} trailing bytes")
        return cls(cfg, weights, meta)

    def save(self, path: str):
        with open(path, "wb") as f:
            f.write(self.to_bytes())

    @classmethod
    def load(cls, path: str) -> "AidenModel":
        with open(path, "rb") as f:
            return cls.from_bytes(f.read())


# AllWeights slices the reference's read_weights returns (deq_bridge.rs:1805-1880),
# as (name, first segment, end segment) of the packed layout
_GPU_EXACT = [("w_q", "wq", "wk"), ("w_k", "wk", "wv"), ("w_v", "wv", "wo"), ("w_o", "wo", "win"),
              ("w_in", "win", "wx"), ("w_x", "wx", "wout"), ("w_out", "wout", "alog"),
              ("a_log", "alog", "nscale"), ("norm_scale", "nscale", "hist")]


def split_all_weights(all_weights: np.ndarray, d: int, h: int) -> dict:
    """Packed AllWeights -> the ``reasoning.gpu_exact.*`` tensors (hist_params = the rest)."""
    L = Layout(d, h)
    w = np.asarray(all_weights, np.float32)
    out = {f"reasoning.gpu_exact.{n}": w[getattr(L, a):getattr(L, b)].copy() for n, a, b in _GPU_EXACT}
    out["reasoning.gpu_exact.hist_params"] = w[L.hist:L.total].copy()
    return out


def join_all_weights(tensors: dict, d: int, h: int) -> np.ndarray:
    L = Layout(d, h)
    w = np.zeros(L.total, np.float32)
    for n, a, b in _GPU_EXACT:
        t = np.asarray(tensors[f"reasoning.gpu_exact.{n}"], np.float32)
        if t.size != getattr(L, b) - getattr(L, a):
            raise ValueError(f"reasoning.gpu_exact.{n}: {t.size} values for d={d}, h={h}")
        w[getattr(L, a):getattr(L, b)] = t
    hp = np.asarray(tensors["reasoning.gpu_exact.hist_params"], np.float32)
    if hp.size != L.total - L.hist:
        raise ValueError("reasoning.gpu_exact.hist_params: wrong length")
    w[L.hist:] = hp
    return w


def full_model(all_weights, d, h, lm=None, emb=None, config=None, metadata=None) -> AidenModel:
    """The reference trainer's full checkpoint of this state (trainer.rs:6470-6530)."""
    cfg = dict(CONFIG_DEFAULTS)
    cfg.update(d_r=d, h_slots=h)
    if emb is not None:
        cfg["vocab_size"] = int(np.shape(emb)[0])
    cfg.update(config or {})
    m = AidenModel(cfg, split_all_weights(all_weights, d, h),
                   {"gpu_exact_checkpoint": "true", "aideen_version": "0.1.0", "type": "FullModel"})
    if lm is not None:
        w_lm, b_lm, g_lm = lm
        m.weights["head.w"] = np.asarray(w_lm, np.float32).ravel()
        m.weights["head.b"] = np.asarray(b_lm, np.float32).ravel()
        m.weights["head.g"] = np.asarray(g_lm, np.float32).ravel()
    if emb is not None:
        m.weights["tokenizer.embeddings"] = np.asarray(emb, np.float32).T.ravel()   # column-major V x d
        m.metadata["vocab_size"] = str(np.shape(emb)[0])
    m.metadata.update(metadata or {})
    return m


def unpack_full_model(m: AidenModel):
    """(all_weights, (w_lm, b_lm, g_lm) or None, embeddings [V][d] or None)."""
    d, h = int(m.config["d_r"]), int(m.config["h_slots"])
    w = join_all_weights(m.weights, d, h)
    lm = None
    if "head.w" in m.weights:
        lm = (m.weights["head.w"].reshape(-1, d), m.weights["head.b"], m.weights["head.g"])
    emb = None
    if "tokenizer.embeddings" in m.weights:
        e = m.weights["tokenizer.embeddings"]
        emb = e.reshape(d, -1).T.copy()
    return w, lm, emb


# ---------------------------------------------------------------- .opt
def save_opt(path: str, step: int, tensors: dict):
    """`Adam::save_state`: tensors maps full keys (e.g. ``m_vec.name``) to f32 arrays."""
    parts = [b"AIDENOPT", struct.pack("<Q", int(step))]
    for k, v in tensors.items():
        kb = k.encode("utf-8")
        a = np.ascontiguousarray(v, dtype="<f4").ravel()
        parts += [struct.pack("<I", len(kb)), kb, struct.pack("<I", a.size), a.tobytes()]
    with open(path, "wb") as f:
        f.write(b"".join(parts))


def load_opt(path: str):
    """`Adam::load_state`: (step, {key: f32 array}); a truncated tail ends the read."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 16 or data[:8] != b"AIDENOPT":
        raise ValueError("Invalid or corrupt .opt file")
    step = struct.unpack_from("<Q", data, 8)[0]
    pos, out = 16, {}
    while pos + 8 <= len(data):
        kl = struct.unpack_from("<I", data, pos)[0]
        pos += 4
        if pos + kl + 4 > len(data):
            break
        key = data[pos:pos + kl].decode("utf-8")
        pos += kl
        n = struct.unpack_from("<I", data, pos)[0]
        pos += 4
        if pos + 4 * n > len(data):
            break
        out[key] = np.frombuffer(data, dtype="<f4", count=n, offset=pos).astype(np.float32)
        pos += 4 * n
    return step, out


def adam_tensors(m_core, v_core, d, h, m_lm=None, v_lm=None) -> dict:
    """The library's Adam moments as `.opt` entries (``m_vec.`` / ``v_vec.`` + the
    .aidn tensor names)."""
    out = {}
    for pre, arr in (("m_vec.", m_core), ("v_vec.", v_core)):
        for k, t in split_all_weights(arr, d, h).items():
            out[pre + k] = t
    if m_lm is not None:
        out["m_vec.head"] = np.asarray(m_lm, np.float32)
        out["v_vec.head"] = np.asarray(v_lm, np.float32)
    return out


def adam_from_tensors(t: dict, d, h):
    strip = lambda pre: {k[len(pre):]: v for k, v in t.items() if k.startswith(pre) and k != pre + "head"}
    mc = join_all_weights(strip("m_vec."), d, h)
    vc = join_all_weights(strip("v_vec."), d, h)
    return mc, vc, t.get("m_vec.head"), t.get("v_vec.head")
