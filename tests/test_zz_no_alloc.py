"""The allocation-free adjoint entry point against the context-based one.

`aideen_adjoint_noalloc` exists for callers that must not allocate device
memory (allocators that forbid cudaMalloc once start-up is over, embedders
that own every byte of the device, host code that must not take the
allocator's lock).  It takes only device pointers and keeps its scratch in a
fixed device array, so two calls in a row must both match `aideen_adjoint_on`
(the existing entry point), and its NormScale gradient must match the same
reduction done on the host.  Arguments it cannot serve (sizes beyond the fixed
array or shared memory, misaligned pointers) are refused before any launch,
and a stage wait of the kernel that runs out comes back as AIDEEN_E_TIMEOUT.
This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_noalloc_adjoint_matches_context_adjoint_twice():
    import torch
    from aideen_b200.backend import GpuDeqBackend, load_library
    from aideen_b200.weights import init_all_weights

    lib = load_library()
    d, h, N = 512, 8, 96
    W = init_all_weights(d, h, seed=21)
    be = GpuDeqBackend(d, h, max_batch=1, max_seq_len=N)
    be.upload_weights(W)
    ns = W[be.layout.nscale:be.layout.nscale + d].copy()
    dev = torch.device("cuda", 0)
    for call, (m, iters, seed) in enumerate([(0, 12, 1), (4, 20, 2)]):
        rng = np.random.default_rng(seed)
        hs = rng.standard_normal((N, h, d)).astype(np.float32)
        br = rng.standard_normal((N, h, d)).astype(np.float32)
        dl = rng.standard_normal((N, d)).astype(np.float32)
        rs = rng.standard_normal((N, h, d)).astype(np.float32)
        # existing entry point (owns its memory)
        be.run_adjoint_on(hs, br, 1, N, 0.85, iters, dl_dh=dl, rhs_slot=rs, anderson_m=m)
        v_ref = be.read_adj_v_out()
        g_ref = be.read("gpre", (N, h, d))
        # allocation-free entry point on caller-owned device buffers
        t = {k: torch.from_numpy(x).to(dev) for k, x in dict(hs=hs, br=br, dl=dl, rs=rs, ns=ns).items()}
        v = torch.empty((h, N, d), device=dev)
        g = torch.empty((N, h, d), device=dev)
        nsg = torch.full((d,), float("nan"), device=dev)
        stream = torch.cuda.current_stream(dev)
        rc = lib.aideen_adjoint_noalloc(
            C.c_void_p(t["hs"].data_ptr()), C.c_void_p(t["br"].data_ptr()), C.c_void_p(t["dl"].data_ptr()),
            C.c_void_p(t["rs"].data_ptr()), C.c_void_p(t["ns"].data_ptr()), N, h, d, iters, 0.85, m,
            C.c_void_p(v.data_ptr()), C.c_void_p(g.data_ptr()), C.c_void_p(nsg.data_ptr()),
            C.c_void_p(stream.cuda_stream))
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert rel(v.cpu().numpy(), v_ref) < TOL
        assert rel(g.cpu().numpy(), g_ref) < TOL
        pre = hs.astype(np.float64) + br
        r = np.sqrt(np.mean(pre * pre, -1) + 1e-6)
        vt = np.transpose(v_ref, (1, 0, 2)).astype(np.float64)
        ns_ref = (0.85 * vt * pre / np.maximum(r, 1e-6)[..., None]).sum(axis=(0, 1))
        assert rel(nsg.cpu().numpy(), ns_ref) < TOL
    # sizes beyond the fixed scratch are refused, not truncated
    big = 1 << 20
    rc = lib.aideen_adjoint_noalloc(C.c_void_p(1 << 12), C.c_void_p(1 << 12), None, None, C.c_void_p(1 << 12),
                                    big, h, d, 1, 0.85, 0, C.c_void_p(1 << 12), C.c_void_p(1 << 12),
                                    C.c_void_p(1 << 12), None)
    assert rc == 1
    be.close()
    # misaligned pointers (a view at an odd float offset) are refused before any launch
    ok = C.c_void_p(1 << 12)
    bad = C.c_void_p((1 << 12) + 4)
    for i in range(8):
        args = [ok, ok, ok, ok, ok]
        outs = [ok, ok, ok]
        if i < 5:
            args[i] = bad
        else:
            outs[i - 5] = bad
        rc = lib.aideen_adjoint_noalloc(*args, 8, h, d, 1, 0.85, 0, *outs, None)
        assert rc == 1, f"misaligned pointer {i} not refused"
    # per-token stages larger than one block's shared memory are refused
    rc = lib.aideen_adjoint_noalloc(ok, ok, None, ok, ok, 8, 16, 1024, 1, 0.85, 0, ok, ok, None, None)
    assert rc == 1


def test_noalloc_adjoint_reports_a_wait_that_ran_out():
    """AIDEEN_ADJ_SPIN_LIMIT=0 makes every first stage wait of the adjoint give up
    at once (the copies still land; the kernel drains them before it returns):
    the entry points report AIDEEN_E_TIMEOUT, and the next normal call works."""
    import os
    import torch
    from aideen_b200.backend import AideenError, GpuDeqBackend, load_library
    from aideen_b200.weights import init_all_weights

    lib = load_library()
    d, h, N = 512, 8, 64
    W = init_all_weights(d, h, seed=5)
    be = GpuDeqBackend(d, h, max_batch=1, max_seq_len=N)
    be.upload_weights(W)
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(9)
    hs = torch.from_numpy(rng.standard_normal((N, h, d)).astype(np.float32)).to(dev)
    br = torch.from_numpy(rng.standard_normal((N, h, d)).astype(np.float32)).to(dev)
    ns = torch.from_numpy(W[be.layout.nscale:be.layout.nscale + d].copy()).to(dev)
    v = torch.empty((h, N, d), device=dev)
    g = torch.empty((N, h, d), device=dev)
    nsg = torch.empty((d,), device=dev)
    stream = torch.cuda.current_stream(dev)

    def call():
        return lib.aideen_adjoint_noalloc(
            C.c_void_p(hs.data_ptr()), C.c_void_p(br.data_ptr()), None, None, C.c_void_p(ns.data_ptr()),
            N, h, d, 8, 0.85, 0, C.c_void_p(v.data_ptr()), C.c_void_p(g.data_ptr()),
            C.c_void_p(nsg.data_ptr()), C.c_void_p(stream.cuda_stream))

    os.environ["AIDEEN_ADJ_SPIN_LIMIT"] = "0"
    try:
        assert call() == 4
        be.run_adjoint_on(hs.cpu().numpy(), br.cpu().numpy(), 1, N, 0.85, 8)
        with pytest.raises(AideenError, match="bounded"):
            be.sync()
    finally:
        del os.environ["AIDEEN_ADJ_SPIN_LIMIT"]
    assert call() == 0
    be.run_adjoint_on(hs.cpu().numpy(), br.cpu().numpy(), 1, N, 0.85, 8)
    assert rel(v.cpu().numpy(), be.read_adj_v_out()) < TOL
    be.close()
