"""Row operators on the B200 vs the oracle and the reference's golden outputs.

Tolerance (fp32 storage): |got - exp| <= 1e-5 * |exp| + 1e-5 * max_row |exp|,
where exp is the sequential-sum oracle; an element that misses it passes only
if it meets the same bound against a float64 evaluation (the GPU's tree sum
may be closer to the exact value than the reference's sequential sum).
fp16 storage: the corpus harness tolerance (hvx_close_f16bits, atol 4e-3,
rtol 8e-3) and at most 1 fp16 ulp from the reference.
"""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def f64_softmax(x):
    x = x.astype(np.float64)
    e = np.exp(x - x.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def f64_layernorm(x, g, b, eps):
    x = x.astype(np.float64)
    mean = x.mean(-1, keepdims=True)
    var = np.maximum((x * x).mean(-1, keepdims=True) - mean * mean, 0)
    return (x - mean) / np.sqrt(var + eps) * g.astype(np.float64) + b.astype(np.float64)


def assert_f32_close(got, exp, exact):
    got, exp, exact = (np.asarray(a, np.float64) for a in (got, exp, exact))
    scale = np.abs(exp).max(-1, keepdims=True)
    tol = RTOL * np.abs(exp) + RTOL * scale
    bad = np.abs(got - exp) > tol
    if bad.any():
        tol64 = RTOL * np.abs(exact) + RTOL * scale
        bad &= np.abs(got - exact) > tol64
    assert not bad.any(), f"{bad.sum()} elements off; worst {np.abs(got - exp).max()}"


def assert_f16_close(got, exp, max_ulp=1):
    g = got.astype(np.float32).ravel()
    e = exp.astype(np.float32).ravel()
    assert np.all(np.abs(g - e) <= 4e-3 + 8e-3 * np.abs(e))
    gi = got.view(np.int16).astype(np.int32).ravel()
    ei = exp.view(np.int16).astype(np.int32).ravel()
    assert np.abs(gi - ei).max() <= max_ulp


SHAPES = [(8, 256), (37, 1000), (5, 1023), (64, 4096), (16, 8192), (3, 12345), (2, 40000),
          (1, 1), (130, 4)]


@pytest.mark.parametrize("R,C", SHAPES)
def test_softmax_f32(hx, oracle, R, C):
    rng = np.random.default_rng(R * 1000 + C)
    x = (rng.standard_normal((R, C)) * 8).astype(np.float32)
    got = hx.softmax(x)
    assert_f32_close(got, oracle.softmax(x), f64_softmax(x))


@pytest.mark.parametrize("R,C", SHAPES)
def test_layernorm_f32(hx, oracle, R, C):
    rng = np.random.default_rng(R * 7 + C)
    x = (rng.standard_normal((R, C)) * 8).astype(np.float32)
    g = rng.normal(1, 0.1, C).astype(np.float32)
    b = rng.normal(0, 0.1, C).astype(np.float32)
    got = hx.layernorm(x, g, b, 1e-5)
    assert_f32_close(got, oracle.layernorm(x, g, b, 1e-5), f64_layernorm(x, g, b, 1e-5))


@pytest.mark.parametrize("R,C", SHAPES)
@pytest.mark.parametrize("op", [0, 1])
def test_rowreduce_f32(hx, oracle, R, C, op):
    rng = np.random.default_rng(R + C + op)
    x = (rng.standard_normal((R, C)) * 8).astype(np.float32)
    got = hx.rowreduce(x, op)
    exp = oracle.rowreduce(x, op)
    if op == 1:
        np.testing.assert_array_equal(got, exp)
    else:
        assert_rowsum_close(got, exp, x)


def assert_rowsum_close(got, exp, x):
    """fp32 row sums: within 1e-5 * sum|x| of the exact (float64) sum.  The
    sequential-sum oracle `exp` (the reference's order) is held to the same
    bound, so both sums are checked against one yardstick."""
    x64 = np.asarray(x, np.float64)
    exact = x64.sum(-1)
    lim = 1e-5 * np.abs(x64).sum(-1)
    got, exp = np.asarray(got, np.float64), np.asarray(exp, np.float64)
    assert np.all(np.abs(got - exact) <= lim), np.max(np.abs(got - exact) / np.maximum(lim, 1e-30))
    assert np.all(np.abs(exp - exact) <= lim)


def test_rowsum_mined_golden(hx):
    g = golden("rowsum_fp32_mined")
    x = g["x"].reshape(1, -1)
    assert_rowsum_close(hx.rowreduce(x, 0), g["out"][:1], x)


def test_rowsum_cancellation(hx, oracle):
    """Rows whose sum nearly cancels (sum|x| far above |sum|): the bound is
    relative to sum|x|, as for any fp32 summation."""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 4096)) * 8).astype(np.float32)
    x[:, 2048:] = -x[:, :2048]
    x[:, 7] += 1e-3
    assert_rowsum_close(hx.rowreduce(x, 0), oracle.rowreduce(x, 0), x)


def test_rmsnorm_f32_device(hx, oracle):
    import torch
    from hexkernels_b200 import device
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((33, 4096)) * 8).astype(np.float32)
    g = rng.normal(1, 0.1, 4096).astype(np.float32)
    xt, gt = torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda()
    out = torch.empty_like(xt)
    device.bind_stream(0)
    device.launch("rmsnorm_f32", 0, xt, gt, out, 33, 4096, 1e-5)
    torch.cuda.synchronize()
    device.sync(0)
    exp = oracle.rmsnorm(x, g, 1e-5)
    x64 = x.astype(np.float64)
    exact = x64 / np.sqrt((x64 * x64).mean(-1, keepdims=True) + 1e-5) * g
    assert_f32_close(out.cpu().numpy(), exp, exact)


@pytest.mark.parametrize("name", ["softmax_f16_harness", "softmax_f16_96x256"])
def test_softmax_f16_golden(hx, name):
    g = golden(name)
    got = hx.softmax(g["x"].reshape(-1, 256))
    assert_f16_close(got.ravel(), g["out"].ravel())


def test_layernorm_f16_golden(hx):
    g = golden("layernorm_f16_harness")
    got = hx.layernorm(g["x"].reshape(1, -1), g["gamma"], g["beta"], 1e-3)
    assert_f16_close(got.ravel(), g["out"])


def test_rmsnorm_f16_golden(hx):
    g = golden("rmsnorm_f16_harness")
    got = hx.rmsnorm_f16(g["x"].reshape(1, -1), g["gamma"], 1e-3)
    assert_f16_close(got.ravel(), g["out"])


def test_online_softmax_step_golden(hx):
    g = golden("online_softmax_step_harness")
    for c in range(3):
        st = g[f"c{c}_state_in"]
        m, s, acc = hx.online_softmax_step_f16(g[f"c{c}_scores"], g[f"c{c}_V"].reshape(24, 48),
                                               st[0], st[1], st[2:])
        got = np.concatenate([[m, s], acc]).astype(np.float16)
        assert_f16_close(got, g[f"c{c}_state_out"])


@pytest.mark.slow
def test_benchmark_shape_65536x4096(hx, oracle):
    """The benchmark configuration itself: 65536 x 4096 fp32, x = 8 N(0,1),
    gamma N(1, 0.1), beta N(0, 0.1), eps 1e-5.  Every row is checked by
    size-independent properties; every 509th row against the oracle."""
    R, C = 65536, 4096
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((R, C), dtype=np.float32) * 8)
    g = rng.normal(1, 0.1, C).astype(np.float32)
    b = rng.normal(0, 0.1, C).astype(np.float32)
    sm = hx.softmax(x)
    assert np.all(np.abs(sm.sum(-1, dtype=np.float64) - 1) < 1e-4)
    assert np.all(sm >= 0)
    rows = np.arange(0, R, 509)
    assert_f32_close(sm[rows], oracle.softmax(x[rows]), f64_softmax(x[rows]))
    ln = hx.layernorm(x, g, b, 1e-5)
    z = (ln - b) / g
    assert np.all(np.abs(z.mean(-1, dtype=np.float64)) < 1e-3)
    assert_f32_close(ln[rows], oracle.layernorm(x[rows], g, b, 1e-5),
                     f64_layernorm(x[rows], g, b, 1e-5))
    del sm, ln, z
    # row sum and max over every row of the benchmark matrix
    assert_rowsum_close(hx.rowreduce(x, 0), oracle.rowreduce(x, 0), x)
    np.testing.assert_array_equal(hx.rowreduce(x, 1), x.max(-1))
