"""The task evaluator (hexkernels_b200.evaluate): output parsing, roofline
arithmetic and the build line on the CPU; full runs of prebuilt reference
harnesses on the GPU."""
import os
from pathlib import Path

import pytest

from hexkernels_b200 import evaluate as ev

# a checkout of the reference corpus, when one is named in HEXKERNELS_REF
CORPUS = Path(os.environ["HEXKERNELS_REF"]) if os.environ.get("HEXKERNELS_REF") else None
REPO = Path(__file__).resolve().parent.parent


def test_feedback_defaults():
    fb = ev.new_feedback("i8_gemm_requant", None)
    for k in ("task_id", "candidate", "compiled", "correct", "errors", "n", "error_text",
              "timed_out", "target", "achieved", "AI", "binding_level", "ceiling", "eta",
              "roofline_unavailable", "kernel_us", "launches", "used_gpu"):
        assert k in fb, k
    assert fb["compiled"] is False and fb["correct"] is False and fb["eta"] is None


def test_parse_output():
    out = ("HEXCUDA_KERNEL_US kernel=12.500 wall=80.000 launches=2\n"
           "HEXCUDA_KERNEL_US kernel=2.500 wall=20.000 launches=1\n"
           "HVXENV_CORRECT errors=0 n=2048\n")
    p = ev.parse_output(out, "")
    assert p["correct"] and p["errors"] == 0 and p["n"] == 2048
    assert p["kernel_us"] == 15.0 and p["wall_us"] == 100.0 and p["launches"] == 3 and p["used_gpu"]
    p = ev.parse_output("HVXENV_INCORRECT errors=7 n=64 first_bad=3 got=1 exp=2\n",
                        "HEXCUDA_ERROR 3 no usable device\n")
    assert p["correct"] is False and p["errors"] == 7 and "HEXCUDA_ERROR" in p["error_text"]
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=-1000.000 wall=3.0 launches=0\n", "")
    assert p["kernel_us"] is None and p["launches"] == 0 and not p["used_gpu"]
    # a timing line from an older harness without the launch count
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=1.000 wall=2.000\nHVXENV_CORRECT errors=0 n=1\n", "")
    assert p["kernel_us"] == 1.0 and "launches" not in p


def test_roofline_arithmetic():
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1500.0, "source": "test"}
    # int8 GEMM 8192^3: AI far above the ridge -> tensor-bound, ceiling 3000 TOPS
    fb = {"kernel_us": 1000.0}
    ev.attach_roofline(fb, 2.0 * 8192 ** 3, 3 * 8192 ** 2, "int8->int32", peaks)
    assert fb["binding_level"] == "tensor" and fb["ceiling"] == 3.0e15
    assert abs(fb["eta"] - (2.0 * 8192 ** 3 / 1e-3) / 3.0e15) < 1e-12
    # elementwise requant: AI 1/9 op per byte -> HBM-bound
    fb = {"kernel_us": 100.0}
    ev.attach_roofline(fb, 1e8, 9e8, "int32+int32->int8", peaks)
    assert fb["binding_level"] == "HBM"
    assert abs(fb["ceiling"] - 1e8 / 9e8 * 6000e9) < 1
    fb = ev.new_feedback("x", None)
    ev.attach_roofline(fb, None, None)
    assert fb["eta"] is None and "useful_ops" in fb["roofline_unavailable"]


def test_harness_command_builds_the_task_harness_unchanged(tmp_path):
    cmd = ev.harness_command(Path("/corpus/kernels/expert/t"), Path("cand.c"), tmp_path / "h")
    assert "/corpus/kernels/expert/t/harness.c" in cmd and "cand.c" in cmd
    assert cmd[cmd.index("-include") + 1] == "/corpus/kernels/expert/t/kernel_api.h"
    assert "-lhexcuda" in cmd and f"-I{REPO / 'hexkernels_b200' / 'harness'}" in cmd


def test_missing_inputs_are_reported():
    fb = ev.evaluate("no_such_task", corpus=str(REPO))
    assert not fb["compiled"] and "not found" in fb["error_text"]
    fb = ev.evaluate("no_such_task", harness=str(REPO / "nope"))
    assert not fb["compiled"] and "no corpus" in fb["error_text"]


@pytest.mark.skipif(CORPUS is None or not (CORPUS / "kernels" / "expert").is_dir(),
                    reason="no corpus checkout named in HEXKERNELS_REF")
def test_build_from_corpus_without_gpu():
    """Builds the task's own harness with the default shim; without a usable
    GPU the run reports the library's error and an incorrect result."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    fb = ev.evaluate("i8_gemm_requant", corpus=str(CORPUS), timeout=120)
    assert fb["compiled"] and not fb["correct"]
    assert "HEXCUDA_ERROR" in fb["error_text"]


@pytest.mark.gpu
@pytest.mark.parametrize("task", ["i8_gemm_requant", "fp16_softmax", "hmx_matmul_i8_bias",
                                  "residual_add_requant", "fp16_flash_attention_tile"])
def test_evaluate_prebuilt_harness_on_gpu(hx, task):
    exe = REPO / "oracle" / "_ref" / f"gpu_harness_{task}"
    if not exe.exists():
        pytest.skip("reference harnesses not built (make -C oracle ref-gpu)")
    fb = ev.evaluate(task, harness=str(exe), useful_ops=1e6, work_bytes=1e6, dtype="int8")
    assert fb["compiled"] and fb["correct"], fb
    assert fb["used_gpu"] and fb["launches"] >= 1 and fb["kernel_us"] > 0
    assert fb["eta"] is not None and fb["binding_level"] in ("HBM", "tensor")
    # the mechanism verdict: what ran agrees with the static evidence
    if task in ("i8_gemm_requant", "hmx_matmul_i8_bias"):
        assert fb["static_tcgen05"] and fb["used_tcgen05"] and fb["used_tma"]
        assert fb["mechanism"] == "tcgen05"
    if task in ("fp16_softmax", "residual_add_requant"):
        assert not fb["static_tcgen05"] and fb["used_tcgen05"] is False
        assert fb["mechanism"] == "cuda-core"
        # HBM-bound: the 16-byte vector path (rows of 256 fp16; 1024 bytes)
        assert fb["static_vec128"] and fb["used_vec128"]


def test_mechanism_fields_from_the_timing_line():
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=5.000 wall=9.000 launches=2 mech=0x3\n"
                        "HVXENV_CORRECT errors=0 n=4\n", "")
    assert p["used_tcgen05"] and p["used_tma"] and p["mechanism"] == "tcgen05"
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=5.000 wall=9.000 launches=1 mech=0x0\n", "")
    assert p["used_tcgen05"] is False and p["mechanism"] == "cuda-core"
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=-1000.000 wall=2.0 launches=0 mech=0x0\n", "")
    assert p["mechanism"] == "cpu" and not p["used_gpu"]
    # several timed calls: the bits of all of them
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=1.0 wall=2.0 launches=1 mech=0x0\n"
                        "HEXCUDA_KERNEL_US kernel=1.0 wall=2.0 launches=1 mech=0x1\n", "")
    assert p["used_tcgen05"] and not p["used_tma"] and p["used_vec128"] is False
    p = ev.parse_output("HEXCUDA_KERNEL_US kernel=1.0 wall=2.0 launches=1 mech=0x4\n", "")
    assert p["used_vec128"] and not p["used_tcgen05"] and p["mechanism"] == "cuda-core"


def test_static_scan_tells_scalar_from_tensor_core_candidates(tmp_path):
    scalar = tmp_path / "scalar.c"
    scalar.write_text("""
#include <stdint.h>
/* a candidate that never reaches the GPU: hexcuda_host_gemm_u8s8_pc( in a comment */
void candidate_kernel(const int8_t *A, const int8_t *B, int8_t *out, int M, int N, int K,
                      int32_t mult, int shift, int8_t zp) {
    for (int i = 0; i < M * N; i++) out[i] = 0;
}
""")
    s = ev.scan_candidate(scalar)
    assert s == {"calls": [], "static_tcgen05": False, "static_tma": False,
                 "static_vec128": False}
    s = ev.scan_candidate(REPO / "hexkernels_b200" / "shims" / "i8_gemm_requant.c")
    assert s["calls"] == ["hexcuda_host_gemm_i8_requant"]
    assert s["static_tcgen05"] and s["static_tma"]
    s = ev.scan_candidate(REPO / "hexkernels_b200" / "shims" / "fp16_softmax.c")
    assert s["calls"] and not s["static_tcgen05"] and not s["static_tma"]
    assert s["static_vec128"]           # the row kernels' 16-byte vector path
    own = tmp_path / "own.cu"
    own.write_text('__global__ void k() { asm volatile("tcgen05.mma.cta_group::1.kind::f16 '
                   '[%0], %1, %2, %3, p;" ::); }\n')
    s = ev.scan_candidate(own)
    assert s["static_tcgen05"] and not s["static_tma"]


def test_library_mechanism_map():
    m = ev.library_mechanisms()
    for e in ("hexcuda_host_gemm_u8s8_pc", "hexcuda_host_gemm_f16_nt", "hexcuda_host_attn_f16",
              "hexcuda_host_gemm_hmx_ex", "hexcuda_gemm_u8s8_pc_noalloc"):
        assert m[e][:2] == (True, True), e
    # the HBM-bound operators: no tensor cores, 16-byte vector loads / stores
    for e in ("hexcuda_host_softmax_f32", "hexcuda_host_layernorm_f32", "hexcuda_host_rowreduce_f32",
              "hexcuda_host_requant_ew", "hexcuda_host_reduce_int", "hexcuda_softmax_f32",
              "hexcuda_reduce_int"):
        assert m[e] == (False, False, True), e
