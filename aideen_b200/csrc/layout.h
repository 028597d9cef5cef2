// AllWeights offsets (C++ twin of aideen_b200/layout.py).
//
// Order and sizes follow aideen-block/src/deq_bridge.rs:103-137 and the WGSL
// mirror aideen-block/src/shaders/deq_slot_attn_unified_clean.wgsl:189-237;
// HistParams follows aideen-backbone/src/gpu_deq.rs:260-422.
//
// Two instances exist per context: the packed layout (align = 1) is the
// reference's wire format used at the C-ABI boundary; the device copy uses
// align = 64 floats so every tensor starts on a 256-byte boundary (the
// reference's 21-float flag block and h-long vectors would otherwise leave
// W_write_gate, W_retain_*, W_q_mem, W_k_mem off 16-byte alignment for
// vector loads).
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace aideen {

constexpr int kRank = 32;     // RETAIN_RANK / MEM_READ_RANK / ASSOC_RANK
constexpr int kHeadDim = 32;  // SLOT_ATTN_HEAD_DIM (d >= 128 here, so min(d, 32) = 32)
constexpr int kFlags = 21;
constexpr int kSegments = 36;

struct Layout {
  size_t d, h, align;
  size_t wq, q_bias, wk, k_bias, wv, wo, win, wx, wout, alog, nscale, hist;
  size_t hist_mat, hist_scale, hist_bias, hist_gate, slot_anchor, w_k_write, w_v_write, b_delta,
      flags, signal_zero, signal_scale, hist_gate_query, w_write_gate, b_write_mem, hhist_gamma,
      w_retain_up, w_retain_down, b_retain, w_q_mem, w_k_mem, b_read_mem, w_k_assoc, w_v_assoc,
      w_q_assoc, alpha_assoc, w_event_assoc, b_event_assoc, total;
  size_t seg_off[kSegments], seg_len[kSegments];

  explicit Layout(size_t d_, size_t h_, size_t align_ = 1) : d(d_), h(h_), align(align_) {
    const size_t dd = d * d, r = kRank;
    size_t o = 0;
    int k = 0;
    auto seg = [&](size_t len) {
      o = (o + align - 1) / align * align;
      const size_t at = o;
      seg_off[k] = at;
      seg_len[k] = len;
      ++k;
      o += len;
      return at;
    };
    wq = seg(h * dd);
    q_bias = seg(h * d);
    wk = seg(h * dd);
    k_bias = seg(h * d);
    wv = seg(h * dd);
    wo = seg(h * dd);
    win = seg(h * dd);
    wx = seg(dd);
    wout = seg(dd);
    alog = seg(h * d);
    nscale = seg(d);
    hist_mat = seg(dd);
    hist = hist_mat;
    hist_scale = seg(h * d);
    hist_bias = seg(h * d);
    hist_gate = seg(h);
    slot_anchor = seg(h * d);
    w_k_write = seg(h * d * r);
    w_v_write = seg(h * r * d);
    b_delta = seg(h * d);
    flags = seg(kFlags);
    signal_zero = flags + 9;
    signal_scale = flags + 16;
    hist_gate_query = seg(h * d);
    w_write_gate = seg(h * d);
    b_write_mem = seg(h);
    hhist_gamma = seg(h);
    w_retain_up = seg(h * d * r);
    w_retain_down = seg(h * r * d);
    b_retain = seg(h * d);
    w_q_mem = seg(h * d * r);
    w_k_mem = seg(h * d * r);
    b_read_mem = seg(h);
    w_k_assoc = seg(h * d * r);  // associative branch (kept off)
    w_v_assoc = seg(h * d * r);
    w_q_assoc = seg(h * d * r);
    alpha_assoc = seg(h);
    w_event_assoc = seg(h * d);
    b_event_assoc = seg(h);
    total = (o + align - 1) / align * align;
  }
};

}  // namespace aideen
