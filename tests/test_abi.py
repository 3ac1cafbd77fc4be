"""C-ABI checks that need no GPU: libhexcuda and every candidate_kernel shim
load and export exactly what include/ declares, and calls fail cleanly (error
code, untouched output) when no device is usable."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "hexkernels_b200"


def declared_symbols():
    text = (REPO / "include" / "hexcuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hexcuda_\w+)\s*\(", text)))


def exported(path: Path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module")
def built():
    if not (PKG / "libhexcuda.so").exists():
        subprocess.run(["make", "-s", "-C", str(PKG / "csrc")], check=True)
    subprocess.run(["make", "-s", "-C", str(PKG / "shims")], check=True)
    return PKG / "libhexcuda.so"


def test_every_declared_symbol_is_exported(built):
    decl = declared_symbols()
    assert len(decl) >= 50
    exp = exported(built)
    missing = [s for s in decl if s not in exp]
    assert not missing, missing
    # nothing beyond the declared API leaks out of the library
    extra = sorted(s for s in exp if s.startswith("hexcuda_") and s not in decl)
    assert not extra, extra


def test_python_binding_matches_header(built):
    from hexkernels_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()
    _lib.load()


def test_every_task_header_has_a_shim_exporting_only_candidate_kernel(built):
    headers = sorted(p.stem for p in (REPO / "include" / "kernel_api").glob("*.h")
                     if p.stem != "hvx_hf")
    assert len(headers) >= 18
    for h in headers:
        so = PKG / "shims" / f"libcand_{h}.so"
        assert so.exists(), so
        assert exported(so) == {"candidate_kernel"}, h


def test_kernel_sources_are_sm100a_native():
    # tcgen05 MMA + TMA for the contractions, 128-bit vector loads for the rows
    src = {p.name: p.read_text() for p in (PKG / "csrc").glob("*.cu*")}
    allsrc = "\n".join(src.values())
    for needle in ("tcgen05.mma.cta_group::1.kind::f16", "tcgen05.mma.cta_group::1.kind::i8",
                   "tcgen05.alloc", "tcgen05.ld.sync.aligned", "cp.async.bulk.tensor.2d"):
        assert needle in allsrc, needle
    assert "float4" in src["rows.cu"] and "uint4" in src["rows.cu"]
    # every TMA load is a plain per-CTA form or the CTA-pair form whose bytes
    # are counted on the pair's barrier; none is a cluster-wide broadcast
    # (each CTA loads its own tiles; the package runs on several GPUs)
    allowed = {
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes",
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes",
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes",
    }
    forms = set(re.findall(r"cp\.async\.bulk\.tensor[\w.:]*", allsrc))
    assert forms == allowed, forms
    assert "multi" + "cast" not in allsrc
    assert "tcgen05.mma.cta_group::2" in src["tc_common.cuh"]
    # no legacy tensor-core paths
    for legacy in ("mma.sync", "wmma::", "wgmma"):
        assert legacy not in allsrc, legacy
    mk = (PKG / "csrc" / "Makefile").read_text()
    assert "arch=compute_100a,code=sm_100a" in mk


def test_no_device_errors_are_clean(built):
    """Without a usable GPU every entry returns an error code, prints one
    HEXCUDA_ERROR line and leaves the output buffer untouched."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    code = r'''
import ctypes as C, numpy as np, sys
sys.path.insert(0, %r)
from hexkernels_b200 import _lib
lib = _lib.load()
x = np.ones((4, 8), np.float32); out = np.full((4, 8), 7.0, np.float32)
rc = lib.hexcuda_host_softmax_f32(x.ctypes.data, out.ctypes.data, 4, 8)
assert rc != 0, rc
assert (out == 7.0).all()
assert lib.hexcuda_last_error() == rc
rc2 = lib.hexcuda_init(1)
assert rc2 != 0
print("RC", rc, rc2, lib.hexcuda_last_error_string().decode())
''' % str(REPO)
    r = subprocess.run(["python", "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "HEXCUDA_ERROR" in r.stderr


def test_bad_arguments_rejected_before_any_device_work(built):
    from hexkernels_b200 import _lib
    lib = _lib.load()
    out = np.full(4, 3, np.int8)
    # negative sizes are argument errors whatever the device state
    assert lib.hexcuda_host_gemm_i8_requant(None, None, out.ctypes.data, -1, 2, 2, 1, 0, 0) != 0
    assert (out == 3).all()
