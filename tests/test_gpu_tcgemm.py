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
    (2048, 96, 512, 8, False, False),    # Q|K|V = src . Wcat[s] (128-column tile, 32 columns past N)
    (1000, 64, 300, 3, True, True),      # 64-column tile, both operands transposed
]

TF32_SHAPES = [
    # single-TF32 weight gradients: C = A^T B with both operands MN-major
    (512, 512, 2048, 8, True, False),    # gW_in (256-column tile)
    (512, 96, 2048, 8, True, False),     # gW_q|k|v as one 96-column product
    (32, 512, 2048, 8, True, False),     # gW_o: 32 rows, formed transposed
    (32, 512, 16384, 1, True, False),    # W_retain_down-like, long K (split-K, transposed)
    (512, 512, 16384, 1, True, False),   # W_out
    (300, 200, 1000, 2, True, False),    # ragged
]


@pytest.mark.parametrize("shape", TF32_SHAPES, ids=lambda s: "x".join(map(str, s[:4])) + f"_t{int(s[4])}{int(s[5])}")
def test_single_tf32_gemm_matches_fp32(shape):
    """Operands rounded to nearest tf32 (relative error 2^-11 each), fp32
    accumulation: about 4e-4 relative on a sum of products."""
    M, N, K, B, ta, tb = shape
    be = GpuDeqBackend(128, 2, 1, 1)
    err, t_tc, t_simt = be.gemm_selftest(M, N, K, B, ta, tb, tf32=True)
    print(f"{shape}: rel {err:.2e}  tc {t_tc:.3f} ms  simt {t_simt:.3f} ms")
    assert err < 1e-3
    be.close()


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
