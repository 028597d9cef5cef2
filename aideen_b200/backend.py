"""Host-side mirror of the reference's `GpuDeqBackend` over the C ABI.

Method names follow `aideen-backbone/src/gpu_deq.rs` (`upload_weights`,
`run_forward_deq_no_readback`, `run_staged_adjoint_picard_no_readback`,
`apply_fused_deq_update`, `renormalize_spectral`, `read_*`), so a trainer
written against the reference reads the same here.  Every call goes through
`libaideen_b200.so` (include/aideen_b200.h); there is no CPU fallback: if the
library is missing or no GPU is visible, construction raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

from .layout import Layout

HOST, DEVICE = 0, 1

BUF = dict(hstar=0, pooled=1, signal=2, attn=3, iters=4, adj_v=5, gpre=6, dl_dh=7, hist_ctx=8,
           mstate=9, fpm_ctx=10, alpha=11, s_in=12, ds_in=13, lm_grads=14, pre=15, fpm_dm=16,
           fpm_carry=17, lm_samples=18)

RULE_ADAM, RULE_CLIPPED_SGD = 0, 1


class AideenError(RuntimeError):
    pass


class _Cfg(C.Structure):
    _fields_ = [("d_model", C.c_uint32), ("h_slots", C.c_uint32), ("max_batch", C.c_uint32),
                ("max_seq_len", C.c_uint32), ("vocab", C.c_uint32), ("flags", C.c_uint32)]


class Run(C.Structure):
    """`RunUniforms` (`deq_slot_attn_unified_clean.wgsl:1-21`)."""
    _fields_ = [("batch", C.c_uint32), ("seq_len", C.c_uint32), ("max_iters", C.c_uint32),
                ("epsilon", C.c_float), ("damping", C.c_float), ("slot_coord", C.c_uint32),
                ("fpm", C.c_uint32), ("fpm_alpha_m", C.c_float), ("fpm_tau", C.c_float),
                ("fpm_read_gate_min", C.c_float), ("anderson_m", C.c_uint32)]


class Stats(C.Structure):
    _fields_ = [("total_iters", C.c_uint64), ("max_iters_seen", C.c_uint32),
                ("unconverged", C.c_uint32), ("nonfinite", C.c_uint32), ("solves", C.c_uint32)]


class AdjArgs(C.Structure):
    _fields_ = [("batch", C.c_uint32), ("seq_len", C.c_uint32), ("iters", C.c_uint32),
                ("damping", C.c_float), ("anderson_m", C.c_uint32)]


class Update(C.Structure):
    _fields_ = [("rule", C.c_uint32), ("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("eps", C.c_float), ("weight_decay", C.c_float), ("grad_scale", C.c_float),
                ("step", C.c_uint32), ("allreduce", C.c_uint32), ("update_lm_head", C.c_uint32)]


class StepArgs(C.Structure):
    _fields_ = [("run", Run), ("adj_iters", C.c_uint32), ("anderson_m", C.c_uint32),
                ("update", Update), ("renorm", C.c_uint32), ("lm_samples", C.c_uint32),
                ("emb_update", C.c_uint32), ("emb_lr", C.c_float), ("sample_seed", C.c_uint64)]


_LIB = None
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libaideen_b200.so")

_P = C.c_void_p
_SIGS = {
    "aideen_create": (_P, [C.POINTER(_Cfg), C.c_int, C.POINTER(C.c_int)]),
    "aideen_destroy": (None, [_P]),
    "aideen_last_error": (C.c_char_p, [_P]),
    "aideen_set_stream": (C.c_int, [_P, _P]),
    "aideen_sync": (C.c_int, [_P]),
    "aideen_launch_count": (C.c_uint64, [_P]),
    "aideen_profile": (C.c_int, [_P, C.c_int]),
    "aideen_join": (C.c_int, [_P]),
    "aideen_profile_read": (C.c_int, [_P, _P, _P, C.c_int]),
    "aideen_all_weights_len": (C.c_size_t, [C.c_uint32, C.c_uint32]),
    "aideen_upload_weights": (C.c_int, [_P, _P, C.c_size_t, C.c_int]),
    "aideen_download_weights": (C.c_int, [_P, _P, C.c_size_t]),
    "aideen_download_grads": (C.c_int, [_P, _P, C.c_size_t]),
    "aideen_upload_lm_head": (C.c_int, [_P, _P, _P, _P]),
    "aideen_download_lm_head": (C.c_int, [_P, _P, _P, _P]),
    "aideen_download_embedding": (C.c_int, [_P, _P]),
    "aideen_temporal_scan": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_int]),
    "aideen_download_adam": (C.c_int, [_P, _P, _P, C.c_size_t, _P, _P]),
    "aideen_upload_adam": (C.c_int, [_P, _P, _P, C.c_size_t, _P, _P]),
    "aideen_upload_embedding": (C.c_int, [_P, _P]),
    "aideen_reset_state": (C.c_int, [_P]),
    "aideen_reset_optimizer": (C.c_int, [_P]),
    "aideen_forward": (C.c_int, [_P, C.POINTER(Run), _P, C.c_int, C.POINTER(Stats)]),
    "aideen_forward_tokens": (C.c_int, [_P, C.POINTER(Run), _P, C.c_int, C.POINTER(Stats)]),
    "aideen_lm_head_loss": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, C.c_int, C.POINTER(C.c_float)]),
    "aideen_adjoint": (C.c_int, [_P, C.POINTER(AdjArgs), _P, _P, C.c_int]),
    "aideen_adjoint_on": (C.c_int, [_P, C.POINTER(AdjArgs), _P, _P, _P, _P, C.c_int]),
    "aideen_source_grad": (C.c_int, [_P, _P, C.c_int]),
    "aideen_weight_grads": (C.c_int, [_P]),
    "aideen_apply_update": (C.c_int, [_P, C.POINTER(Update)]),
    "aideen_renormalize_spectral": (C.c_int, [_P, C.c_uint32, C.c_float, C.c_float, C.c_float,
                                              C.c_float, C.c_float, _P]),
    "aideen_train_step": (C.c_int, [_P, C.POINTER(StepArgs), _P, _P, C.c_int,
                                    C.POINTER(C.c_float), C.POINTER(Stats)]),
    "aideen_read": (C.c_int, [_P, C.c_int, _P, C.c_size_t]),
    "aideen_device_ptr": (_P, [_P, C.c_int]),
    "aideen_adjoint_noalloc": (C.c_int, [_P, _P, _P, _P, _P, C.c_uint32, C.c_uint32, C.c_uint32,
                                         C.c_uint32, C.c_float, C.c_uint32, _P, _P, _P, _P]),
    "aideen_gemm_selftest": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "aideen_comm_unique_id": (C.c_int, [_P]),
    "aideen_comm_init": (C.c_int, [_P, _P, C.c_int, C.c_int]),
    "aideen_allreduce_grads": (C.c_int, [_P, C.c_int]),
}


def load_library(path: str | None = None):
    """Load libaideen_b200.so and declare every C-ABI signature."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise AideenError(f"{p} is missing; build it with `python -m aideen_b200.build`")
    lib = C.CDLL(p)
    for name, (res, args) in _SIGS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def exported_symbols():
    return list(_SIGS)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


@dataclass
class RunConfig:
    max_iters: int = 12
    epsilon: float = 1e-4
    damping: float = 0.85
    slot_coord: bool = True
    fpm: bool = False
    fpm_alpha_m: float = 0.01
    fpm_tau: float = 0.5
    fpm_read_gate_min: float = 0.0
    anderson_m: int = 0            # forward Anderson depth (0 = plain Picard)

    def run(self, batch: int, seq_len: int) -> Run:
        return Run(batch, seq_len, self.max_iters, self.epsilon, self.damping, int(self.slot_coord),
                   int(self.fpm), self.fpm_alpha_m, self.fpm_tau, self.fpm_read_gate_min, self.anderson_m)


CFG_ASSOC = 1  # aideen_cfg.flags bit: associative branch on the upper slots


class GpuDeqBackend:
    """One context = one GPU, one CUDA stream, all device buffers."""

    def __init__(self, d_model: int, h_slots: int, max_batch: int, max_seq_len: int,
                 vocab: int = 0, device: int = 0, assoc: bool = False):
        """assoc: the reference's default associative branch on the upper h/2
        slots whenever the FPM memory is on (AIDEEN_CFG_ASSOC)."""
        self.lib = load_library()
        self.d, self.h, self.vocab = d_model, h_slots, vocab
        self.max_batch, self.max_seq_len = max_batch, max_seq_len
        self.layout = Layout(d_model, h_slots)
        st = C.c_int(0)
        cfg = _Cfg(d_model, h_slots, max_batch, max_seq_len, vocab, CFG_ASSOC if assoc else 0)
        self.ctx = self.lib.aideen_create(C.byref(cfg), device, C.byref(st))
        if not self.ctx:
            raise AideenError(f"aideen_create failed with status {st.value}")
        self.batch = self.seq_len = 0

    # ---- plumbing ---------------------------------------------------------
    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self.lib.aideen_last_error(self.ctx)
            raise AideenError(f"{what}: status {rc}: {msg.decode() if msg else ''}")

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.aideen_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def join(self):
        """Order the deferred LM-head update before later work on the context stream."""
        self._check(self.lib.aideen_join(self.ctx), "join")

    def sync(self):
        self._check(self.lib.aideen_sync(self.ctx), "sync")

    def set_stream(self, stream_handle: int):
        self._check(self.lib.aideen_set_stream(self.ctx, C.c_void_p(stream_handle)), "set_stream")

    @property
    def launch_count(self) -> int:
        return int(self.lib.aideen_launch_count(self.ctx))

    PROF_CLASSES = ("picard", "adjoint", "gemm", "lm_head", "optimizer", "other", "fpm_bwd")

    def profile(self, enable: bool = True):
        """Bracket every kernel launch with CUDA events (per-class device time)."""
        self._check(self.lib.aideen_profile(self.ctx, int(enable)), "profile")

    def profile_read(self, reset: bool = True) -> dict:
        ms = np.zeros(len(self.PROF_CLASSES), np.float32)
        n = np.zeros(len(self.PROF_CLASSES), np.uint64)
        self._check(self.lib.aideen_profile_read(self.ctx, _ptr(ms), _ptr(n), int(reset)), "profile_read")
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.PROF_CLASSES)}

    def device_ptr(self, name: str) -> int:
        return int(self.lib.aideen_device_ptr(self.ctx, BUF[name]) or 0)

    # ---- weights (gpu_deq.rs:3529, :5595) --------------------------------
    def upload_weights(self, all_weights):
        w = _f32(all_weights)
        self._check(self.lib.aideen_upload_weights(self.ctx, _ptr(w), w.size, HOST), "upload_weights")

    def upload_weights_device(self, ptr: int, n: int):
        self._check(self.lib.aideen_upload_weights(self.ctx, C.c_void_p(ptr), n, DEVICE),
                    "upload_weights")

    def read_weights(self) -> np.ndarray:
        out = np.empty(self.layout.total, np.float32)
        self._check(self.lib.aideen_download_weights(self.ctx, _ptr(out), out.size), "read_weights")
        return out

    def read_grads(self) -> np.ndarray:
        out = np.empty(self.layout.total, np.float32)
        self._check(self.lib.aideen_download_grads(self.ctx, _ptr(out), out.size), "read_grads")
        return out

    def upload_lm_head(self, w_lm, b_lm, g_lm):
        a, b, c = _f32(w_lm), _f32(b_lm), _f32(g_lm)
        self._check(self.lib.aideen_upload_lm_head(self.ctx, _ptr(a), _ptr(b), _ptr(c)), "upload_lm_head")

    def read_lm_head(self):
        a = np.empty((self.vocab, self.d), np.float32)
        b = np.empty(self.vocab, np.float32)
        c = np.empty(self.d, np.float32)
        self._check(self.lib.aideen_download_lm_head(self.ctx, _ptr(a), _ptr(b), _ptr(c)), "read_lm_head")
        return a, b, c

    def temporal_scan(self, batch, seq_len, hstar=None):
        """The simple temporal carrier (`temporal_step`) over a chunk of fixed
        points (default: the last forward's); memory rows land in hist_ctx."""
        hs = _f32(hstar) if hstar is not None else None
        self._check(self.lib.aideen_temporal_scan(self.ctx, batch, seq_len, _ptr(hs) if hs is not None else None,
                                                  HOST), "temporal_scan")
        self.batch, self.seq_len = batch, seq_len

    def read_adam(self):
        """(m_core, v_core, m_lm, v_lm): core moments in the packed AllWeights
        layout, LM-head moments as [vocab*d + vocab + d] (None without a head)."""
        n = self.layout.total
        mc, vc = np.empty(n, np.float32), np.empty(n, np.float32)
        nl = self.vocab * self.d + self.vocab + self.d if self.vocab else 0
        ml = np.empty(nl, np.float32) if nl else None
        vl = np.empty(nl, np.float32) if nl else None
        self._check(self.lib.aideen_download_adam(self.ctx, _ptr(mc), _ptr(vc), n,
                                                  _ptr(ml) if nl else None, _ptr(vl) if nl else None), "read_adam")
        return mc, vc, ml, vl

    def upload_adam(self, m_core, v_core, m_lm=None, v_lm=None):
        mc, vc = _f32(m_core), _f32(v_core)
        ml = _f32(m_lm) if m_lm is not None else None
        vl = _f32(v_lm) if v_lm is not None else None
        self._check(self.lib.aideen_upload_adam(self.ctx, _ptr(mc), _ptr(vc), mc.size,
                                                _ptr(ml) if ml is not None else None,
                                                _ptr(vl) if vl is not None else None), "upload_adam")

    def read_embedding(self):
        out = np.empty((self.vocab, self.d), np.float32)
        self._check(self.lib.aideen_download_embedding(self.ctx, _ptr(out)), "read_embedding")
        return out

    def upload_embedding(self, emb):
        e = _f32(emb)
        self._check(self.lib.aideen_upload_embedding(self.ctx, _ptr(e)), "upload_embedding")

    def reset_state(self):
        self._check(self.lib.aideen_reset_state(self.ctx), "reset_state")

    def reset_optimizer(self):
        self._check(self.lib.aideen_reset_optimizer(self.ctx), "reset_optimizer")

    # ---- forward (gpu_deq.rs:3855) ---------------------------------------
    def run_forward_deq_no_readback(self, s_in, batch: int, seq_len: int, cfg: RunConfig,
                                    stats: bool = False):
        s = _f32(s_in)
        r = cfg.run(batch, seq_len)
        st = Stats()
        self._check(self.lib.aideen_forward(self.ctx, C.byref(r), _ptr(s), HOST,
                                            C.byref(st) if stats else None), "forward")
        self.batch, self.seq_len = batch, seq_len
        return st if stats else None

    def run_forward_tokens(self, tokens, batch: int, seq_len: int, cfg: RunConfig, stats=False):
        t = _i32(tokens)
        r = cfg.run(batch, seq_len)
        st = Stats()
        self._check(self.lib.aideen_forward_tokens(self.ctx, C.byref(r), _ptr(t), HOST,
                                                   C.byref(st) if stats else None), "forward_tokens")
        self.batch, self.seq_len = batch, seq_len
        return st if stats else None

    def lm_head_loss(self, targets) -> float:
        t = _i32(targets)
        loss = C.c_float(0.0)
        self._check(self.lib.aideen_lm_head_loss(self.ctx, self.batch, self.seq_len, _ptr(t), HOST,
                                                 C.byref(loss)), "lm_head_loss")
        return float(loss.value)

    # ---- adjoint (gpu_deq.rs:4080, :4922) --------------------------------
    def run_staged_adjoint_picard_no_readback(self, damping: float, iters: int, dl_dh=None,
                                              rhs_slot=None, anderson_m: int = 0):
        a = AdjArgs(self.batch, self.seq_len, iters, damping, anderson_m)
        dl = _f32(dl_dh) if dl_dh is not None else None
        rs = _f32(rhs_slot) if rhs_slot is not None else None
        self._check(self.lib.aideen_adjoint(self.ctx, C.byref(a), _ptr(dl) if dl is not None else None,
                                            _ptr(rs) if rs is not None else None, HOST), "adjoint")

    def run_adjoint_on(self, hstar, branch, batch, seq_len, damping, iters, dl_dh=None,
                       rhs_slot=None, anderson_m=0):
        a = AdjArgs(batch, seq_len, iters, damping, anderson_m)
        hs, br = _f32(hstar), _f32(branch)
        dl = _f32(dl_dh) if dl_dh is not None else None
        rs = _f32(rhs_slot) if rhs_slot is not None else None
        self._check(self.lib.aideen_adjoint_on(self.ctx, C.byref(a), _ptr(hs), _ptr(br),
                                               _ptr(dl) if dl is not None else None,
                                               _ptr(rs) if rs is not None else None, HOST), "adjoint_on")
        self.batch, self.seq_len = batch, seq_len

    def reduce_clean_adjoint_to_source_grad(self) -> np.ndarray:
        out = np.empty((self.batch * self.seq_len, self.d), np.float32)
        self._check(self.lib.aideen_source_grad(self.ctx, _ptr(out), HOST), "source_grad")
        return out

    # ---- gradients + update (gpu_deq.rs:4980) ----------------------------
    def weight_grads(self):
        self._check(self.lib.aideen_weight_grads(self.ctx), "weight_grads")

    def apply_update(self, rule=RULE_ADAM, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                     weight_decay=0.0, grad_scale=1.0, step=1, allreduce=False, lm_head=False):
        u = Update(rule, lr, beta1, beta2, eps, weight_decay, grad_scale, step, int(allreduce),
                   int(lm_head))
        self._check(self.lib.aideen_apply_update(self.ctx, C.byref(u)), "apply_update")

    def apply_fused_deq_update(self, **kw):
        """Weight gradients then the update rule, as one call (gpu_deq.rs:4980)."""
        self.weight_grads()
        self.apply_update(**kw)

    def renormalize_spectral(self, n_iters=12, attn=0.10, win=0.30, fpm=0.70, wv=0.50, wo=0.50):
        sig = np.empty(5 * self.h + 2, np.float32)
        self._check(self.lib.aideen_renormalize_spectral(self.ctx, n_iters, attn, win, fpm, wv, wo,
                                                         _ptr(sig)), "renormalize_spectral")
        return sig

    def train_step(self, tokens, targets, batch, seq_len, cfg: RunConfig, adj_iters=12,
                   anderson_m=0, lr=1e-3, step=1, rule=RULE_ADAM, renorm=False, allreduce=False,
                   grad_scale=1.0, where=HOST, want_loss=True, raw_ptr=False, lm_samples=0,
                   emb_update=0, emb_lr=0.0, sample_seed=0):
        """One full step.  With raw_ptr=True, `tokens`/`targets` are integer
        addresses (device memory when where=DEVICE, pinned host memory when
        where=HOST) instead of arrays.  lm_samples > 0 selects the reference's
        sampled-softmax LM head; emb_update 1 / 2 trains the embedding rows
        from dL/dpooled / dL/dS_in (see aideen_step_args)."""
        a = StepArgs(cfg.run(batch, seq_len), adj_iters, anderson_m,
                     Update(rule, lr, 0.9, 0.999, 1e-8, 0.0, grad_scale, step, int(allreduce), 1),
                     int(renorm), lm_samples, emb_update, emb_lr, sample_seed)
        loss = C.c_float(0.0)
        if not raw_ptr:
            t, g = _i32(tokens), _i32(targets)
            tp, gp = _ptr(t), _ptr(g)
        else:
            tp, gp = C.c_void_p(tokens), C.c_void_p(targets)
        self._check(self.lib.aideen_train_step(self.ctx, C.byref(a), tp, gp, where,
                                               C.byref(loss) if want_loss else None, None), "train_step")
        self.batch, self.seq_len = batch, seq_len
        return float(loss.value)

    # ---- readbacks (gpu_deq.rs:5821-5886) --------------------------------
    def read(self, name: str, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype)
        self._check(self.lib.aideen_read(self.ctx, BUF[name], _ptr(out), out.size), f"read {name}")
        return out

    def read_hnext_seq(self):
        N = self.batch * self.seq_len
        return self.read("hstar", (self.batch, self.seq_len, self.h, self.d))

    def read_hpooled_seq(self):
        return self.read("pooled", (self.batch, self.seq_len, self.d))

    def read_adj_v_out(self):
        return self.read("adj_v", (self.h, self.batch * self.seq_len, self.d))

    def gemm_selftest(self, M, N, K, batch=1, trans_a=False, trans_b=False, presplit=False, tf32=False):
        """(relative L2 difference, ms tensor-core, ms CUDA-core) on seeded operands.
        presplit=True runs the persistent kernel on pre-split hi/lo operands;
        tf32=True single TF32 products instead of 3xTF32."""
        e, t1, t2 = C.c_float(), C.c_float(), C.c_float()
        flags = (1 if presplit else 0) | (2 if tf32 else 0)
        self._check(self.lib.aideen_gemm_selftest(self.ctx, M, N, K, batch, int(trans_a), int(trans_b),
                                                  flags, C.byref(e), C.byref(t1), C.byref(t2)),
                    "gemm_selftest")
        return e.value, t1.value, t2.value

    # ---- multi-GPU --------------------------------------------------------
    @staticmethod
    def comm_unique_id() -> bytes:
        lib = load_library()
        buf = C.create_string_buffer(128)
        rc = lib.aideen_comm_unique_id(buf)
        if rc != 0:
            raise AideenError("ncclGetUniqueId failed")
        return buf.raw

    def comm_init(self, uid: bytes, nranks: int, rank: int):
        buf = C.create_string_buffer(uid, 128)
        self._check(self.lib.aideen_comm_init(self.ctx, buf, nranks, rank), "comm_init")

    def allreduce_grads(self, timeout_ms: int = 60000):
        self._check(self.lib.aideen_allreduce_grads(self.ctx, timeout_ms), "allreduce_grads")
