"""fp16 attention on the B200 vs the reference's flash-attention tile.

Tolerance: |got - exp| <= 1e-2 * |exp| + 2e-3 against the fp32-statistics
reference (the corpus harness uses atol 4e-3, rtol 8e-3 for this bundle and
that bound is checked too on its golden case).
"""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


def assert_attn_close(got, exp):
    g, e = got.astype(np.float64), exp.astype(np.float64)
    bad = np.abs(g - e) > 1e-2 * np.abs(e) + 2e-3
    assert not bad.any(), f"{bad.sum()} of {bad.size} off, worst {np.abs(g - e).max()}"


def test_flash_tile_harness_golden(hx):
    g = golden("flash_attn_tile_harness")
    SQ, SK, DH = g["dims"]
    got = hx.attn_f16(g["Q"].reshape(SQ, DH), g["K"].reshape(SK, DH), g["V"].reshape(SK, DH),
                      0.125, False)
    e = g["O"].astype(np.float32).reshape(SQ, DH)
    assert np.all(np.abs(got.astype(np.float32) - e) <= 4e-3 + 8e-3 * np.abs(e))
    assert_attn_close(got, g["O"].reshape(SQ, DH))


@pytest.mark.parametrize("name", ["flash_attn_256x64x64", "flash_attn_200x48x128"])
def test_flash_tile_golden(hx, name):
    g = golden(name)
    assert_attn_close(hx.attn_f16(g["Q"], g["K"], g["V"], 0.125, False), g["O"])


CASES = [(1, 1, 1, 64, True), (2, 17, 17, 64, True), (3, 130, 130, 128, True),
         (2, 256, 256, 128, False), (1, 300, 77, 128, False), (4, 384, 384, 128, True),
         (2, 129, 200, 64, False), (1, 1000, 1000, 128, True), (2, 64, 512, 32, False)]


@pytest.mark.parametrize("BH,SQ,SK,D,causal", CASES)
def test_attn_random(hx, oracle, BH, SQ, SK, D, causal):
    if causal and SQ != SK:
        pytest.skip("causal cases use square heads")
    rng = np.random.default_rng(BH * 100 + SQ + SK + D)
    Q = rng.standard_normal((BH, SQ, D)).astype(np.float16)
    K = rng.standard_normal((BH, SK, D)).astype(np.float16)
    V = rng.standard_normal((BH, SK, D)).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    assert_attn_close(hx.attn_f16(Q, K, V, scale, causal), oracle.attn_f16(Q, K, V, scale, causal))


def test_attn_large_scores(hx, oracle):
    # a query aligned with one late key: the running max moves late and
    # every earlier contribution must be rescaled
    rng = np.random.default_rng(9)
    Q = (rng.standard_normal((2, 512, 128)) * 0.5).astype(np.float16)
    K = (rng.standard_normal((2, 512, 128)) * 0.5).astype(np.float16)
    V = rng.standard_normal((2, 512, 128)).astype(np.float16)
    Q[:, 500] = 2.0
    K[:, 499] = 2.0
    for causal in (False, True):
        assert_attn_close(hx.attn_f16(Q, K, V, 0.125, causal),
                          oracle.attn_f16(Q, K, V, 0.125, causal))


@pytest.mark.slow
def test_attn_benchmark_shape(hx, oracle):
    """Causal SDPA B=8, H=32, S=4096, D=128, Q/K/V N(0,1), scale 1/sqrt(128):
    every head against an fp32 evaluation on the GPU (torch fp32, TF32 off,
    used only as the checker: scores, causal mask, softmax, P V all in fp32),
    and 16 whole heads against the oracle's restatement of the reference."""
    import torch
    from test_gpu_gemm import fp32_matmul_ieee
    B, H, S, D = 8, 32, 4096, 128
    rng = np.random.default_rng(0)
    Q = rng.standard_normal((B * H, S, D), dtype=np.float32).astype(np.float16)
    K = rng.standard_normal((B * H, S, D), dtype=np.float32).astype(np.float16)
    V = rng.standard_normal((B * H, S, D), dtype=np.float32).astype(np.float16)
    scale = 1.0 / np.sqrt(D)
    got = hx.attn_f16(Q, K, V, scale, True)
    fp32_matmul_ieee()
    mask = torch.ones((S, S), dtype=torch.bool, device="cuda").tril()
    for h0 in range(0, B * H, 8):
        q, k, v = (torch.from_numpy(t[h0:h0 + 8]).cuda().float() for t in (Q, K, V))
        s = (q @ k.transpose(1, 2)) * scale
        s.masked_fill_(~mask, float("-inf"))
        ref = (torch.softmax(s, -1) @ v).half().cpu().numpy()
        del q, k, v, s
        assert_attn_close(got[h0:h0 + 8], ref)
    for h in np.linspace(0, B * H - 1, 16).astype(int):
        O = np.empty((1, S, D), np.float16)
        a = oracle.attn_args(Q=Q[h:h + 1], K=K[h:h + 1], V=V[h:h + 1], O=O, BH=1, SQ=S, SK=S,
                             D=D, scale=scale, causal=1)
        oracle.parallel(oracle.OP_ATTN_F16, a, 0, S, oracle.nthreads_default())
        assert_attn_close(got[h], O[0])
