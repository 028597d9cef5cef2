// AllWeights offsets (C++ twin of aideen_b200/layout.py).
//
// Order and sizes follow aideen-block/src/deq_bridge.rs:103-137 and the WGSL
// mirror aideen-block/src/shaders/deq_slot_attn_unified_clean.wgsl:189-237;
// HistParams follows aideen-backbone/src/gpu_deq.rs:260-422.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace aideen {

constexpr int kRank = 32;     // RETAIN_RANK / MEM_READ_RANK / ASSOC_RANK
constexpr int kHeadDim = 32;  // SLOT_ATTN_HEAD_DIM (d >= 128 here, so min(d, 32) = 32)
constexpr int kFlags = 21;

struct Layout {
  size_t d, h;
  size_t wq, q_bias, wk, k_bias, wv, wo, win, wx, wout, alog, nscale, hist;
  size_t hist_scale, hist_bias, hist_gate, slot_anchor, w_k_write, w_v_write, b_delta, flags,
      signal_zero, signal_scale, hist_gate_query, w_write_gate, b_write_mem, hhist_gamma,
      w_retain_up, w_retain_down, b_retain, w_q_mem, w_k_mem, b_read_mem, total;

  explicit Layout(size_t d_, size_t h_) : d(d_), h(h_) {
    const size_t dd = d * d, r = kRank;
    wq = 0;
    q_bias = h * dd;
    wk = h * dd + h * d;
    k_bias = wk + h * dd;
    wv = wk + h * dd + h * d;
    wo = wv + h * dd;
    win = wo + h * dd;
    wx = win + h * dd;
    wout = wx + dd;
    alog = wout + dd;
    nscale = alog + h * d;
    hist = nscale + d;
    size_t o = hist + dd;  // hist_mat
    hist_scale = o; o += h * d;
    hist_bias = o; o += h * d;
    hist_gate = o; o += h;
    slot_anchor = o; o += h * d;
    w_k_write = o; o += h * d * r;
    w_v_write = o; o += h * r * d;
    b_delta = o; o += h * d;
    flags = o; o += kFlags;
    signal_zero = flags + 9;
    signal_scale = flags + 16;
    hist_gate_query = o; o += h * d;
    w_write_gate = o; o += h * d;
    b_write_mem = o; o += h;
    hhist_gamma = o; o += h;
    w_retain_up = o; o += h * d * r;
    w_retain_down = o; o += h * r * d;
    b_retain = o; o += h * d;
    w_q_mem = o; o += h * d * r;
    w_k_mem = o; o += h * d * r;
    b_read_mem = o; o += h;
    o += 3 * h * d * r;  // w_k_assoc, w_v_assoc, w_q_assoc (associative branch kept off)
    o += h;              // alpha_assoc
    o += h * d;          // w_event_assoc
    o += h;              // b_event_assoc
    total = o;
  }
};

}  // namespace aideen
