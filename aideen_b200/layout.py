"""AllWeights flat-buffer layout of the AIDEEN DEQ block.

One fp32 buffer holds every DEQ-core parameter, in the order the reference's
compute block binds it:

    W_q[h][d][d] | q_bias[h][d] | W_k[h][d][d] | k_bias[h][d] | W_v[h][d][d]
    | W_o[h][d][d] | W_in[h][d][d] | W_x[d][d] | W_out[d][d] | A_log[h][d]
    | NormScale[d] | HistParams

(`aideen-block/src/deq_bridge.rs:103-137`, WGSL mirror
`aideen-block/src/shaders/deq_slot_attn_unified_clean.wgsl:189-237`).  The
HistParams sub-layout follows `aideen-backbone/src/gpu_deq.rs:260-422`
(`pack_history_params`, `history_params_len`).

Matrix convention (`deq_slot_attn_unified_clean.wgsl:773`): a d x d block M is
applied as y[o] = sum_j M[j*d + o] * x[j] ("input-major").  W_o is read by
head row: attn[o] = sum_{k<head_dim} W_o[k*d + o] * mix[k] (`:461`).  The
rank-32 FPM matrices follow the same rule with their own inner extent:
W_k_write/W_retain_up/W_q_mem/W_k_mem are [d][32] (y[r] = sum_j M[j*32+r] x[j]),
W_v_write/W_retain_down are [32][d] (y[o] = sum_r M[r*d+o] x[r]).

The C++ twin of this module is `aideen_b200/csrc/layout.h`; a CPU test checks
that both agree.
"""
from __future__ import annotations

from dataclasses import dataclass

RANK = 32          # RETAIN_RANK / MEM_READ_RANK / ASSOC_RANK
N_FLAGS = 21       # scalar flag block inside HistParams
HEAD_DIM = 32      # SLOT_ATTN_HEAD_DIM


def head_dim(d: int) -> int:
    """Slot-attention head width: min(d, 32) (`deq_slot_attn_unified_clean.wgsl:520`)."""
    return min(d, HEAD_DIM)


@dataclass(frozen=True)
class Layout:
    d: int
    h: int

    # ---- main block -------------------------------------------------------
    @property
    def wq(self) -> int: return 0
    @property
    def q_bias(self) -> int: return self.h * self.d * self.d
    @property
    def wk(self) -> int: return self.h * self.d * self.d + self.h * self.d
    @property
    def k_bias(self) -> int: return self.wk + self.h * self.d * self.d
    @property
    def wv(self) -> int: return self.wk + self.h * self.d * self.d + self.h * self.d
    @property
    def wo(self) -> int: return self.wv + self.h * self.d * self.d
    @property
    def win(self) -> int: return self.wo + self.h * self.d * self.d
    @property
    def wx(self) -> int: return self.win + self.h * self.d * self.d
    @property
    def wout(self) -> int: return self.wx + self.d * self.d
    @property
    def alog(self) -> int: return self.wout + self.d * self.d
    @property
    def nscale(self) -> int: return self.alog + self.h * self.d
    @property
    def hist(self) -> int: return self.nscale + self.d

    # ---- HistParams (absolute offsets) -----------------------------------
    @property
    def hist_mat(self) -> int: return self.hist
    @property
    def hist_scale(self) -> int: return self.hist + self.d * self.d
    @property
    def hist_bias(self) -> int: return self.hist_scale + self.h * self.d
    @property
    def hist_gate(self) -> int: return self.hist_bias + self.h * self.d
    @property
    def slot_anchor(self) -> int: return self.hist_gate + self.h
    @property
    def w_k_write(self) -> int: return self.slot_anchor + self.h * self.d
    @property
    def w_v_write(self) -> int: return self.w_k_write + self.h * self.d * RANK
    @property
    def b_delta(self) -> int: return self.w_v_write + self.h * RANK * self.d
    @property
    def flags(self) -> int: return self.b_delta + self.h * self.d
    @property
    def signal_zero(self) -> int: return self.flags + 9
    @property
    def signal_scale(self) -> int: return self.flags + 16
    @property
    def hist_gate_query(self) -> int: return self.flags + N_FLAGS
    @property
    def w_write_gate(self) -> int: return self.hist_gate_query + self.h * self.d
    @property
    def b_write_mem(self) -> int: return self.w_write_gate + self.h * self.d
    @property
    def hhist_gamma(self) -> int: return self.b_write_mem + self.h
    @property
    def w_retain_up(self) -> int: return self.hhist_gamma + self.h
    @property
    def w_retain_down(self) -> int: return self.w_retain_up + self.h * self.d * RANK
    @property
    def b_retain(self) -> int: return self.w_retain_down + self.h * RANK * self.d
    @property
    def w_q_mem(self) -> int: return self.b_retain + self.h * self.d
    @property
    def w_k_mem(self) -> int: return self.w_q_mem + self.h * self.d * RANK
    @property
    def b_read_mem(self) -> int: return self.w_k_mem + self.h * self.d * RANK
    @property
    def w_k_assoc(self) -> int: return self.b_read_mem + self.h
    @property
    def w_v_assoc(self) -> int: return self.w_k_assoc + self.h * self.d * RANK
    @property
    def w_q_assoc(self) -> int: return self.w_v_assoc + self.h * self.d * RANK
    @property
    def alpha_assoc(self) -> int: return self.w_q_assoc + self.h * self.d * RANK
    @property
    def w_event_assoc(self) -> int: return self.alpha_assoc + self.h
    @property
    def b_event_assoc(self) -> int: return self.w_event_assoc + self.h * self.d
    @property
    def total(self) -> int: return self.b_event_assoc + self.h

    @property
    def main_len(self) -> int:
        """Length of the part that receives weight decay in the clipped-SGD apply."""
        return self.hist

    @property
    def hist_len(self) -> int:
        return self.total - self.hist


def hist_params_len(d: int, h: int) -> int:
    """`history_params_len` (`aideen-backbone/src/gpu_deq.rs:393-422`)."""
    r = RANK
    return (d * d + 5 * h * d + 2 * h + h * d + N_FLAGS + h + 2 * h * d * r
            + 2 * h * d * r + h * d + 2 * h * d * r + h + 3 * h * d * r + h
            + h * d + h)


def all_weights_len(d: int, h: int) -> int:
    return Layout(d, h).total


# Offsets inside the 21-scalar flag block (`gpu_deq.rs:312-338`).
FLAG_DEFAULTS = [
    0.0,  # 0 hist_selective
    1.0,  # 1 alpha warmup factor
    0.0,  # 2 rms floor
    0.0,  # 3 contractivity floor
    1.0,  # 4 hist inject flag
    0.0,  # 5 minner zero
    0.0,  # 6 force no-fpm
    0.0,  # 7 prelude skip
    0.0,  # 8 loop force no-fpm
    0.0,  # 9 signal zero
    1.0,  # 10 attn out mode
    0.0,  # 11 attn uniform
    0.0,  # 12 attn freeze
    0.0, 0.0, 1.0,  # 13-15 reserved legacy V-path
    1.0,  # 16 signal scale
    0.0, 0.0, 0.0, 1.0,  # 17-20 reserved
]
assert len(FLAG_DEFAULTS) == N_FLAGS
