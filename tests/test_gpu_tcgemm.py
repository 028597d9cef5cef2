"""tcgen05 3xTF32 GEMM vs the CUDA-core fp32 GEMM on every operand pattern the
hot path uses (projections: A row-major; weight gradients: A transposed;
backprop through weights: B transposed)."""
import pytest

from aideen_b200.backend import GpuDeqBackend

pytestmark = pytest.mark.gpu

SHAPES = [
    # M, N, K, batch, transA, transB
    (2048, 512, 512, 8, False, False),   # signal = S_in . W_in[s]
    (2048, 512, 32, 8, False, False),    # attn = n . W_o[s][:32]
    (512, 512, 2048, 8, True, False),    # gW_in = S_in^T . dsig
    (32, 512, 2048, 8, True, False),     # gW_o = n^T . da
    (2048, 512, 32, 8, False, True),     # dsrc += dQ . W[:, :32]^T
    (2048, 32, 512, 8, False, True),     # dn = da . W_o[s][:32]^T
    (300, 96, 100, 2, False, False),     # ragged M / K
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + f"_t{int(s[4])}{int(s[5])}")
def test_tensor_core_gemm_matches_fp32(shape):
    M, N, K, B, ta, tb = shape
    be = GpuDeqBackend(128, 2, 1, 1)
    err, t_tc, t_simt = be.gemm_selftest(M, N, K, B, ta, tb)
    print(f"{shape}: rel {err:.2e}  tc {t_tc:.3f} ms  simt {t_simt:.3f} ms")
    assert err < 5e-5   # fp32-level: both kernels round differently over K
    be.close()


SPLIT_SHAPES = [
    # the LM-head shapes (vocab rounded to 4) and smaller / ragged / batched cases
    (2048, 50260, 512, 1, False, True),    # logits = y . W_lm^T
    (2048, 512, 50260, 1, False, False),   # dy = dlogits . W_lm (split-K)
    (50260, 512, 2048, 1, True, False),    # dW_lm = dlogits^T . y
    (300, 520, 100, 2, False, False),      # ragged M / N / K, batched
    (256, 256, 64, 3, True, True),         # both operands transposed
]


@pytest.mark.parametrize("shape", SPLIT_SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + f"_t{int(s[4])}{int(s[5])}")
def test_presplit_persistent_gemm_matches_fp32(shape):
    M, N, K, B, ta, tb = shape
    be = GpuDeqBackend(128, 2, 1, 1)
    err, t_tc, t_simt = be.gemm_selftest(M, N, K, B, ta, tb, presplit=True)
    print(f"{shape}: rel {err:.2e}  tc {t_tc:.3f} ms  simt {t_simt:.3f} ms")
    assert err < 5e-5
    be.close()


@pytest.mark.parametrize("shape", [SPLIT_SHAPES[1], SPLIT_SHAPES[3], SPLIT_SHAPES[4]],
                         ids=lambda s: "x".join(map(str, s[:4])) + f"_t{int(s[4])}{int(s[5])}")
def test_presplit_narrow_tiles_match_fp32(shape, monkeypatch):
    """128-row tiles (the mode the logits GEMM with row statistics uses) on shapes
    that otherwise take the 256-row tiles."""
    monkeypatch.setenv("AIDEEN_SPLIT_NARROW", "1")
    M, N, K, B, ta, tb = shape
    be = GpuDeqBackend(128, 2, 1, 1)
    err, t_tc, t_simt = be.gemm_selftest(M, N, K, B, ta, tb, presplit=True)
    assert err < 5e-5
    be.close()
