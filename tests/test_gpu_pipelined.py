"""Host-pointer entries that pipeline a call in row chunks (GEMMs cut along M,
attention along heads, the elementwise requant): shapes large enough for
several chunks, with a ragged last chunk, give the same bytes as one
device-pointer launch over the whole problem, and the integer GEMMs equal
the oracle.  A chunk holds a multiple of 16 rows of about 16 MiB for GEMMs
and attention, 32 MiB for the row operators and the elementwise requant
(counted on the larger of a row's input and output bytes)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def test_u8s8_gemm_chunks_equal_oracle(hx, oracle):
    from hexkernels_b200 import _lib
    torch = _torch()
    rng = np.random.default_rng(11)
    # K = 8192: 2048 rows of A per chunk -> chunks 2048, 2048, 37
    M, N, K = 4133, 96, 8192
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = np.round(rng.normal(0, 4000, N)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, N, dtype=np.int64).astype(np.int32)
    shift = rng.integers(36, 42, N).astype(np.int32)
    got = hx.gemm_u8s8_pc(A, B, bias, 131, mult, shift, 128)
    np.testing.assert_array_equal(got, oracle.gemm_u8s8_pc(A, B, bias, 131, mult, shift, 128))
    # one device launch over all rows
    lib = _lib.load()
    d = {k: torch.from_numpy(v).cuda() for k, v in
         dict(A=A, B=B, bias=bias, mult=mult, shift=shift).items()}
    out = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    _lib.check(lib.hexcuda_gemm_u8s8_pc(0, d["A"].data_ptr(), d["B"].data_ptr(),
                                        d["bias"].data_ptr(), out.data_ptr(), M, N, K, 131,
                                        d["mult"].data_ptr(), d["shift"].data_ptr(), 128))
    _lib.check(lib.hexcuda_sync(0))
    np.testing.assert_array_equal(got, out.cpu().numpy())


@pytest.mark.parametrize("store,act,res", [("i32", "relu", None), ("i8_sat", "none", "i8"),
                                           ("acc_i32", "none", "i32")])
def test_hmx_gemm_chunks_equal_oracle(hx, oracle, store, act, res):
    rng = np.random.default_rng(12)
    # int32 out: a row is N * 4 bytes -> 16 MiB / 16 KiB = 1024 rows per chunk
    M, N, K = 2100, 4096, 256
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = rng.integers(-5000, 5000, N).astype(np.int32)
    kw = dict(store=store, act=act, bias=bias)
    if res == "i8":
        kw["res"] = rng.integers(-128, 128, (M, N), dtype=np.int8)
    elif res == "i32":
        kw["res"] = rng.integers(-2**20, 2**20, (M, N)).astype(np.int32)
    got = hx.gemm_hmx_ex(A, B, zpA=7, **kw)
    np.testing.assert_array_equal(got, oracle.gemm_hmx_ex(A, B, zpA=7, **kw))


def test_hmx_plain_entry_chunks(hx, oracle):
    rng = np.random.default_rng(13)
    M, N, K = 2100, 4096, 128
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    bias = rng.integers(-5000, 5000, N).astype(np.int32)
    for kind in (hx.HMX_OUT_I32, hx.HMX_OUT_U8_BIAS_RELU):
        np.testing.assert_array_equal(hx.gemm_hmx(A, B, kind, bias=bias, zpA=3),
                                      oracle.gemm_hmx(A, B, kind, bias=bias, zpA=3))


def test_f16_gemm_chunks_equal_one_launch(hx):
    from hexkernels_b200 import _lib
    torch = _torch()
    rng = np.random.default_rng(14)
    # 2 * K = 8 KiB per row of A, 2 * N = 8 KiB of out -> 2048 rows per chunk
    M, N, K = 4200, 4096, 4096
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    Bt = (rng.standard_normal((N, K)) * 0.5).astype(np.float16)
    got = hx.gemm_f16_nt(A, Bt)
    lib = _lib.load()
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(Bt).cuda()
    out = torch.empty((M, N), dtype=torch.float16, device="cuda")
    _lib.check(lib.hexcuda_gemm_f16_nt(0, dA.data_ptr(), dB.data_ptr(), out.data_ptr(), M, N, K))
    _lib.check(lib.hexcuda_sync(0))
    one = out.cpu().numpy()
    np.testing.assert_array_equal(got, one)
    # and against fp32 math on a band of rows around each chunk boundary
    rows = np.r_[0:8, 2040:2056, 4088:4104, 4192:4200]
    exp = (torch.from_numpy(A[rows]).float() @ torch.from_numpy(Bt).float().T).numpy()
    np.testing.assert_allclose(got[rows].astype(np.float32), exp, rtol=2e-3, atol=2e-1)


def test_f16_gemm_ex_residual_chunks(hx):
    torch = _torch()
    rng = np.random.default_rng(15)
    M, N, K = 4200, 2048, 2048
    A = (rng.standard_normal((M, K)) * 0.5).astype(np.float16)
    B = (rng.standard_normal((K, N)) * 0.5).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float16)
    res = rng.standard_normal((M, N)).astype(np.float16)
    got = hx.gemm_f16_ex(A, B, act="relu", bias=bias, res=res)
    exp = torch.relu(torch.from_numpy(A).float() @ torch.from_numpy(B).float()
                     + torch.from_numpy(bias).float() + torch.from_numpy(res).float()).numpy()
    np.testing.assert_allclose(got.astype(np.float32), exp, rtol=4e-3, atol=2e-1)
    # a residual row lands on its own output row in every chunk
    np.testing.assert_array_equal(hx.gemm_f16_ex(A, B, bias=bias, res=res)[4100:4200],
                                  hx.gemm_f16_ex(A[4100:4200], B, bias=bias, res=res[4100:4200]))


@pytest.mark.parametrize("causal", [True, False])
def test_attention_head_chunks_equal_one_launch(hx, causal):
    from hexkernels_b200 import _lib
    torch = _torch()
    rng = np.random.default_rng(16)
    # 768 KiB of Q, K, V per head -> 32 heads per chunk (21 rounded up to
    # a multiple of 16): chunks 32, 32, 6
    BH, S, D = 70, 1024, 128
    Q = rng.standard_normal((BH, S, D)).astype(np.float16)
    K = rng.standard_normal((BH, S, D)).astype(np.float16)
    V = rng.standard_normal((BH, S, D)).astype(np.float16)
    scale = 1 / np.sqrt(D)
    got = hx.attn_f16(Q, K, V, scale, causal)
    lib = _lib.load()
    dq, dk, dv = (torch.from_numpy(t).cuda() for t in (Q, K, V))
    out = torch.empty_like(dq)
    _lib.check(lib.hexcuda_attn_f16(0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                    out.data_ptr(), BH, S, S, D, scale, int(causal)))
    _lib.check(lib.hexcuda_sync(0))
    np.testing.assert_array_equal(got, out.cpu().numpy())
    heads = [0, 31, 32, 63, 64, 69]
    exp = torch.nn.functional.scaled_dot_product_attention(
        *(torch.from_numpy(t[heads]).float() for t in (Q, K, V)), is_causal=causal,
        scale=scale).numpy()
    np.testing.assert_allclose(got[heads].astype(np.float32), exp, rtol=1e-2, atol=4e-3)


def test_requant_ew_chunks_equal_oracle(hx, oracle):
    rng = np.random.default_rng(17)
    # int32 pairs: 8 input bytes per element -> 4 Mi elements per chunk (row
    # operators' 32 MiB chunks): chunks 4 Mi, 4 Mi and a ragged rest
    n = 3 * (32 << 20) // 9 + 1237
    a = rng.integers(-2**24, 2**24, n).astype(np.int32)
    b = rng.integers(-2**24, 2**24, n).astype(np.int32)
    kw = dict(pre="add", mult=1518500250, shift=33, zp=-3)
    np.testing.assert_array_equal(hx.requant_ew(a, b, **kw), oracle.requant_ew(a, b, **kw))
    a8 = rng.integers(-128, 128, n, dtype=np.int8)
    b8 = rng.integers(-128, 128, n, dtype=np.int8)
    kw = dict(pre="add_relu", mult=1 << 30, shift=31, zp=5)
    np.testing.assert_array_equal(hx.requant_ew(a8, b8, **kw), oracle.requant_ew(a8, b8, **kw))


FIRST_CALLS = {
    # each runs as the first libhexcuda call of a fresh process (no init):
    # the host entry initialises the library itself
    "u8s8": "A = rng.integers(0, 256, (300, 256), dtype=np.uint8);"
            "B = rng.integers(-128, 128, (256, 192), dtype=np.int8);"
            "bias = rng.integers(-999, 999, 192).astype(np.int32);"
            "mult = np.full(192, 1 << 30, np.int32); shift = np.full(192, 36, np.int32);"
            "out = ops.gemm_u8s8_pc(A, B, bias, 5, mult, shift, 128);"
            "exp = o.gemm_u8s8_pc(A, B, bias, 5, mult, shift, 128)",
    "hmx": "A = rng.integers(0, 256, (300, 256), dtype=np.uint8);"
           "B = rng.integers(-128, 128, (256, 192), dtype=np.int8);"
           "bias = rng.integers(-999, 999, 192).astype(np.int32);"
           "out = ops.gemm_hmx_ex(A, B, 'i32', 'relu', bias=bias);"
           "exp = o.gemm_hmx_ex(A, B, 'i32', 'relu', bias=bias)",
    "hmx_plain": "A = rng.integers(0, 256, (300, 256), dtype=np.uint8);"
                 "B = rng.integers(-128, 128, (256, 192), dtype=np.int8);"
                 "out = ops.gemm_hmx(A, B, 0); exp = o.gemm_hmx(A, B, 0)",
    "requant": "a = rng.integers(-2**20, 2**20, 5000).astype(np.int32);"
               "b = rng.integers(-2**20, 2**20, 5000).astype(np.int32);"
               "out = ops.requant_ew(a, b, pre='add', mult=1 << 30, shift=40);"
               "exp = o.requant_ew(a, b, pre='add', mult=1 << 30, shift=40)",
    "f16": "A = rng.standard_normal((200, 128)).astype(np.float16);"
           "Bt = rng.standard_normal((64, 128)).astype(np.float16);"
           "out = ops.gemm_f16_nt(A, Bt).astype(np.float32);"
           "exp = o.gemm_f16_nt(A, Bt).astype(np.float32)",
    "attn": "Q, K, V = (rng.standard_normal((2, 256, 128)).astype(np.float16) for _ in range(3));"
            "out = ops.attn_f16(Q, K, V, 0.125, True).astype(np.float32);"
            "exp = o.attn_f16(Q, K, V, 0.125, True).astype(np.float32)",
    "layernorm": "x = rng.standard_normal((64, 512)).astype(np.float32);"
                 "g = np.ones(512, np.float32); b = np.zeros(512, np.float32);"
                 "out = ops.layernorm(x, g, b, 1e-5); exp = o.layernorm(x, g, b, 1e-5)",
}


@pytest.mark.parametrize("name", sorted(FIRST_CALLS))
def test_host_entry_as_first_call_of_a_process(name):
    import subprocess
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    code = ("import numpy as np\n"
            "from hexkernels_b200 import ops\n"
            "from oracle import oracle as o\n"
            "rng = np.random.default_rng(3)\n"
            + FIRST_CALLS[name] + "\n"
            "np.testing.assert_allclose(out, exp, rtol=1e-2, atol=4e-3)\n"
            "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=repo, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.returncode, r.stdout,
                                                                    r.stderr[-2000:])


def test_pipelined_entries_empty_inputs(hx):
    """Zero rows (and zero columns) through every pipelined entry: nothing to
    do, no error, empty outputs."""
    u8 = np.zeros((0, 256), np.uint8)
    B = np.zeros((256, 64), np.int8)
    v32 = np.zeros(64, np.int32)
    assert hx.gemm_u8s8_pc(u8, B, v32, 3, v32 + (1 << 30), v32 + 40, 128).shape == (0, 64)
    assert hx.gemm_hmx_ex(u8, B, "i32", "relu", bias=v32).shape == (0, 64)
    assert hx.gemm_hmx(u8, B, 0).shape == (0, 64)
    assert hx.gemm_f16_nt(np.zeros((0, 64), np.float16),
                          np.zeros((32, 64), np.float16)).shape == (0, 32)
    assert hx.gemm_f16_nt(np.zeros((8, 64), np.float16),
                          np.zeros((0, 64), np.float16)).shape == (8, 0)
    q = np.zeros((0, 128, 128), np.float16)
    assert hx.attn_f16(q, q, q, 0.125, True).shape == (0, 128, 128)
    z = np.zeros(0, np.int32)
    assert hx.requant_ew(z, z, pre="add", mult=1 << 30, shift=31).shape == (0,)
    x = np.zeros((0, 512), np.float32)
    assert hx.softmax(x).shape == (0, 512)
    assert hx.layernorm(x, np.ones(512, np.float32), np.zeros(512, np.float32),
                        1e-5).shape == (0, 512)
