"""Task evaluator for the B200 kernels: the counterpart of the corpus's
``hexkernels.core.evaluate`` (hexkernels/core/evaluate.py:402-674), which
compiles a candidate with a task's harness, runs it on the Hexagon simulator
and returns a feedback dict.  Here the harness runs natively against
libhexcuda on the GPU:

    build   the task's own harness.c (from a corpus checkout) + the candidate
            (a C file defining candidate_kernel, free to call hexcuda_*; by
            default the task's shim in hexkernels_b200/shims/) + the B200
            harness_common.h, linked with libhexcuda -- or, without a corpus,
            a prebuilt harness binary (oracle/_ref/gpu_harness_<task>);
    run     with a timeout;
    parse   the corpus's result line (HVXENV_CORRECT / HVXENV_INCORRECT
            errors= n=, harness_common.h) and the B200 timing line
            (HEXCUDA_KERNEL_US kernel= wall= launches=), plus any
            HEXCUDA_ERROR lines;
    score   achieved / roofline ceiling when the task's work facts
            (useful_ops, work_bytes) are known, against the measured B200
            peaks.

    python -m hexkernels_b200.evaluate --task-id i8_gemm_requant [--candidate c.c] [--corpus DIR]

prints the feedback dict as JSON.  Keys shared with the corpus evaluator keep
their names and meaning (task_id, candidate, compiled, correct, errors, n,
error_text, timed_out, target, achieved, AI, binding_level, ceiling, eta,
roofline_unavailable); Hexagon-only keys (cycles, packets) have no B200
meaning and are left out.

Mechanism verdict (the B200 counterpart of the corpus's ELF check,
hexkernels/anticheat/anticheat.py:71-345, merged into its feedback at
hexkernels/core/evaluate.py:573-597).  Reading compiled GPU code is not an
option, so the verdict comes from two kinds of evidence:
    static  a scan of the candidate's own source (the hexcuda_* entries it
            calls, inline tcgen05 / TMA PTX) and of libhexcuda's sources:
            whether a called entry reaches, through the library's functions,
            a kernel that issues tcgen05.mma or cp.async.bulk.tensor, or
            that moves 16-byte vectors (int4 / uint4 / float4 accesses, or
            .v4 / .v8 global loads and stores in PTX) (static_tcgen05,
            static_tma, static_vec128; "may", since an entry can choose
            between kernels by shape and alignment);
    run     the library's own record of which kinds of kernel the call
            launched (hexcuda_mechanisms, printed as mech= on the timing
            line): used_tcgen05, used_tma, and used_vec128 for the HBM-bound
            kernels' 128-bit vector path (the north star's LDG.128).
mechanism = "tcgen05" when the run launched tensor-core kernels, "cuda-core"
when it launched only other kernels, "cpu" when it launched none.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
TARGET = "B200 (sm_100a)"
# measured peaks of this pool's B200s (driver-written); fallback figures when
# the file is absent
PEAKS_FILE = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

_CORRECT = re.compile(r"^HVXENV_(CORRECT|INCORRECT) errors=(\d+) n=(\d+)", re.M)
_TIMING = re.compile(r"^HEXCUDA_KERNEL_US kernel=(-?[0-9.]+) wall=([0-9.]+)(?: launches=(\d+))?"
                     r"(?: mech=0x([0-9a-fA-F]+))?", re.M)
MECH_TCGEN05, MECH_TMA, MECH_VEC128 = 1, 2, 4
_HXERR = re.compile(r"^HEXCUDA_ERROR.*$", re.M)


def new_feedback(task_id: str, candidate: str | None) -> dict:
    """The feedback dict with every key at its pre-run default."""
    return {
        "task_id": task_id,
        "candidate": os.path.abspath(candidate) if candidate else "default (hexkernels_b200 shim)",
        "compiled": False, "correct": False,
        "errors": None, "n": None,
        "kernel_us": None,      # device time of the call's last libhexcuda launch (cudaEvent)
        "wall_us": None,        # host wall time of the candidate_kernel call
        "launches": None,       # libhexcuda kernel launches made by the call
        "used_gpu": False,      # at least one libhexcuda launch ran
        # mechanism verdict: static source evidence, then what the run launched
        "calls": [], "static_tcgen05": False, "static_tma": False, "static_vec128": False,
        "used_tcgen05": None, "used_tma": None, "used_vec128": None, "mechanism": None,
        "error_text": "", "timed_out": False,
        "target": TARGET,
        "achieved": None, "AI": None, "binding_level": None, "ceiling": None, "eta": None,
        "roofline_unavailable": None,
    }


def parse_output(stdout: str, stderr: str) -> dict:
    """Fields of the feedback dict read from one harness run's output."""
    out = {}
    m = _CORRECT.search(stdout)
    if m:
        out["correct"] = m.group(1) == "CORRECT"
        out["errors"], out["n"] = int(m.group(2)), int(m.group(3))
    t = _TIMING.findall(stdout)
    if t:
        # a harness may time several calls (parameter sweeps): report the sum;
        # a negative device time means the call made no launch
        dev = [float(k) for k, _, _, _ in t if float(k) >= 0]
        out["kernel_us"] = round(sum(dev), 3) if dev else None
        out["wall_us"] = round(sum(float(w) for _, w, _, _ in t), 3)
        if all(n != "" for _, _, n, _ in t):
            out["launches"] = sum(int(n) for _, _, n, _ in t)
            out["used_gpu"] = out["launches"] > 0
        if all(m != "" for _, _, _, m in t):
            bits = 0
            for _, _, _, m in t:
                bits |= int(m, 16)
            out["used_tcgen05"] = bool(bits & MECH_TCGEN05)
            out["used_tma"] = bool(bits & MECH_TMA)
            out["used_vec128"] = bool(bits & MECH_VEC128)
        if "used_gpu" in out:
            out["mechanism"] = ("tcgen05" if out.get("used_tcgen05") else
                                "cuda-core" if out["used_gpu"] else "cpu")
    errs = _HXERR.findall(stderr)
    if errs:
        out["error_text"] = "\n".join(errs[:5])
    return out


def load_peaks() -> dict:
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def _compute_peak_ops(dtype: str, peaks: dict) -> float | None:
    """Dense tensor-core peak (ops/s) for a task dtype string, None when the
    task has no tensor-core path (its ceiling is then bandwidth alone).  The
    int8 rate is twice the measured bf16 rate on this part."""
    d = (dtype or "").split("->")[0].lower()
    if re.search(r"\b(u?int8|i8|u8)\b", d):
        return 2.0 * peaks["bf16_tflops"] * 1e12
    if re.search(r"(fp16|bf16|half|__fp16|hvx_hf)", d):
        return peaks["bf16_tflops"] * 1e12
    return None


def attach_roofline(fb: dict, useful_ops, work_bytes, dtype: str = "",
                    peaks: dict | None = None) -> dict:
    """achieved = useful_ops / device time; ceiling = min(compute peak,
    AI x HBM bandwidth); eta = achieved / ceiling (the corpus's roofline
    efficiency, hexkernels/core/roofline.py, with B200 levels: HBM or the
    tensor cores)."""
    if not useful_ops or not work_bytes:
        fb["roofline_unavailable"] = "no useful_ops / work_bytes for this task"
        return fb
    if not fb.get("kernel_us"):
        fb["roofline_unavailable"] = "no device time (the run did not reach a launch)"
        return fb
    peaks = peaks or load_peaks()
    secs = fb["kernel_us"] * 1e-6
    ai = float(useful_ops) / float(work_bytes)
    bw = peaks["hbm_gbs"] * 1e9
    comp = _compute_peak_ops(dtype, peaks)
    mem_ceiling = ai * bw
    if comp is not None and comp < mem_ceiling:
        fb["binding_level"], ceiling = "tensor", comp
    else:
        fb["binding_level"], ceiling = "HBM", mem_ceiling
    fb["AI"] = ai
    fb["achieved"] = float(useful_ops) / secs
    fb["ceiling"] = ceiling
    fb["eta"] = fb["achieved"] / ceiling
    fb["peaks_source"] = peaks.get("source", "measured")
    return fb


# ------------------------------------------------------- static source scan

_TC_PTX = re.compile(r"tcgen05\.mma")
_TMA_PTX = re.compile(r"cp\.async\.bulk\.tensor")
_VEC128 = re.compile(r"\b(?:u?int4|float4|double2|u?longlong2)\b"
                     r"|\b(?:ld|st)\.global[\w.:]*\.v[48]\b")
_WORD = re.compile(r"\b[A-Za-z_]\w*\b")
_CALL = re.compile(r"\b(hexcuda_\w+)\s*\(")


def _strip_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def _blank_strings(text: str) -> str:
    """The text with the contents of string and character literals replaced
    by spaces (same length), so braces inside inline-PTX strings do not count."""
    out = list(text)
    i, n = 0, len(text)
    while i < n:
        c = text[i]
        if c in "\"'":
            j = i + 1
            while j < n and text[j] != c:
                j += 2 if text[j] == "\\" else 1
            for k in range(i + 1, min(j, n)):
                if out[k] != "\n":
                    out[k] = " "
            i = j + 1
        else:
            i += 1
    return "".join(out)


def _top_level_functions(text: str, types: dict | None = None) -> dict:
    """name -> text (signature and body) of every function defined at
    namespace scope of one C++ / CUDA source (comments already removed).
    Namespaces and extern "C" blocks are entered; initialisers and
    declarations are skipped; struct / class / union definitions go to
    `types` (name -> body, specialisations joined) when it is given."""
    funcs: dict = {}
    # preprocessor lines carry no code of interest and no statement end
    text = re.sub(r"(?m)^[ \t]*#[^\n]*", lambda m: " " * len(m.group(0)), text)
    bl = _blank_strings(text)
    i, n, head0 = 0, len(bl), 0
    while i < n:
        c = bl[i]
        if c == ";":
            head0 = i + 1
        elif c == "}":                       # end of an entered namespace
            head0 = i + 1
        elif c == "{":
            head = bl[head0:i].strip()
            if re.match(r"(namespace\b|extern\s+\"C\")", head) or head.startswith("extern"):
                head0 = i + 1
                i += 1
                continue
            depth, j = 1, i + 1
            while j < n and depth:
                depth += {"{": 1, "}": -1}.get(bl[j], 0)
                j += 1
            is_type = re.match(r"(template\s*<.*>\s*)?(struct|class|enum|union)\b", head, re.S)
            if is_type and types is not None:
                m = re.search(r"\b(?:struct|class|union)\s+([A-Za-z_]\w*)", head)
                if m:
                    types.setdefault(m.group(1), []).append(text[head0:j])
            if "(" in head and not is_type and not head.endswith("="):
                # name: the identifier before the last parenthesised group
                k, depth_p = len(head) - 1, 0
                while k >= 0:
                    if head[k] == ")":
                        depth_p += 1
                    elif head[k] == "(":
                        depth_p -= 1
                        if depth_p == 0:
                            break
                    k -= 1
                m = re.search(r"([A-Za-z_]\w*)\s*$", head[:max(k, 0)])
                if m:
                    funcs.setdefault(m.group(1), []).append(text[head0:j])
            i = j
            head0 = j
            continue
        i += 1
    return {k: "\n".join(v) for k, v in funcs.items()}


_LIB_MECH = None


def library_mechanisms() -> dict:
    """hexcuda_* entry -> (reaches tcgen05.mma, reaches cp.async.bulk.tensor,
    reaches 16-byte vector accesses) through the functions defined in
    libhexcuda's sources."""
    global _LIB_MECH
    if _LIB_MECH is not None:
        return _LIB_MECH
    funcs: dict = {}
    for f in sorted((PKG / "csrc").glob("*.c*")):
        types: dict = {}
        for k, v in _top_level_functions(_strip_comments(f.read_text()), types).items():
            funcs[k] = funcs.get(k, "") + "\n" + v
        # a type's members count for the functions that name it (e.g. a
        # vector-width trait whose loads a kernel uses)
        for k, v in types.items():
            funcs.setdefault(k, "")
            funcs[k] += "\n" + "\n".join(v)
    names = set(funcs)
    edges = {k: (set(_WORD.findall(v)) & names) - {k} for k, v in funcs.items()}
    own = {k: (bool(_TC_PTX.search(v)), bool(_TMA_PTX.search(v)), bool(_VEC128.search(v)))
           for k, v in funcs.items()}
    memo: dict = {}

    def reach(k, stack=()):
        if k in memo:
            return memo[k]
        tc, tma, vec = own[k]
        for c in edges[k]:
            if c in stack:
                continue
            a, b, v = reach(c, stack + (k,))
            tc, tma, vec = tc or a, tma or b, vec or v
        memo[k] = (tc, tma, vec)
        return memo[k]

    _LIB_MECH = {k: reach(k) for k in funcs if k.startswith("hexcuda_")}
    return _LIB_MECH


def scan_candidate(path) -> dict:
    """Static evidence from a candidate's own source: the libhexcuda entries
    it calls, and whether those (or its own code) reach tcgen05 MMAs, TMA
    loads and 16-byte vector accesses."""
    text = _strip_comments(Path(path).read_text())
    calls = sorted(set(_CALL.findall(text)))
    lib = library_mechanisms()
    none = (False, False, False)
    tc = bool(_TC_PTX.search(text)) or any(lib.get(c, none)[0] for c in calls)
    tma = bool(_TMA_PTX.search(text)) or any(lib.get(c, none)[1] for c in calls)
    vec = bool(_VEC128.search(text)) or any(lib.get(c, none)[2] for c in calls)
    return {"calls": calls, "static_tcgen05": tc, "static_tma": tma, "static_vec128": vec}


def find_task_dir(corpus: Path, task_id: str) -> Path | None:
    for sub in ("expert", "mined", ""):
        d = corpus / "kernels" / sub / task_id if sub else corpus / task_id
        if (d / "harness.c").exists():
            return d
    return None


def harness_command(task_dir: Path, candidate: Path, exe: Path, cc: str = "gcc") -> list:
    """The compile + link line: the task's harness.c and kernel_api.h
    unchanged, the B200 harness_common.h first on the include path."""
    return [cc, "-O2", "-D__fp16=_Float16", f"-I{task_dir}", f"-I{PKG / 'harness'}",
            f"-I{REPO / 'include'}", "-include", str(task_dir / "kernel_api.h"),
            "-o", str(exe), str(task_dir / "harness.c"), str(candidate),
            f"-L{PKG}", "-lhexcuda", "-lm", f"-Wl,-rpath,{PKG}"]


def evaluate(task_id: str, candidate: str | None = None, corpus: str | None = None,
             harness: str | None = None, timeout: float = 300.0, useful_ops=None,
             work_bytes=None, dtype: str | None = None, keep: bool = False) -> dict:
    fb = new_feedback(task_id, candidate)
    spec = {}
    corpus = corpus or os.environ.get("HEXKERNELS_CORPUS")
    tmp = Path(tempfile.mkdtemp(prefix=f"hxeval_{task_id}_"))
    try:
        exe = None
        if corpus:
            task_dir = find_task_dir(Path(corpus), task_id)
            if task_dir is None:
                fb["error_text"] = f"task {task_id} not found under {corpus}"
                return fb
            if (task_dir / "spec.json").exists():
                spec = json.loads((task_dir / "spec.json").read_text())
            cand = Path(candidate) if candidate else PKG / "shims" / f"{task_id}.c"
            if not cand.exists():
                fb["error_text"] = f"no candidate source {cand}"
                return fb
            fb.update(scan_candidate(cand))
            exe = tmp / "harness"
            r = subprocess.run(harness_command(task_dir, cand, exe), capture_output=True, text=True)
            if r.returncode != 0:
                fb["error_text"] = r.stderr[-4000:]
                return fb
        else:
            if candidate:
                fb["error_text"] = "a candidate source needs the task's harness.c (--corpus)"
                return fb
            pre = Path(harness) if harness else REPO / "oracle" / "_ref" / f"gpu_harness_{task_id}"
            if not pre.exists():
                fb["error_text"] = f"no corpus given and no prebuilt harness {pre}"
                return fb
            exe = pre
            shim = PKG / "shims" / f"{task_id}.c"
            if shim.exists():
                fb.update(scan_candidate(shim))
        fb["compiled"] = True
        try:
            r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=timeout)
        except subprocess.TimeoutExpired:
            fb["timed_out"] = True
            fb["error_text"] = f"harness exceeded {timeout} s"
            return fb
        fb.update(parse_output(r.stdout, r.stderr))
        if r.returncode != 0 and not fb["error_text"]:
            fb["error_text"] = (r.stdout + r.stderr)[-2000:]
        attach_roofline(fb, useful_ops or spec.get("useful_ops"),
                        work_bytes or spec.get("work_bytes"), dtype or spec.get("dtype", ""))
        return fb
    finally:
        if keep:
            fb["workdir"] = str(tmp)
        else:
            for f in tmp.iterdir():
                f.unlink()
            tmp.rmdir()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--task-id", required=True)
    ap.add_argument("--candidate", help="C file defining candidate_kernel (default: the task's shim)")
    ap.add_argument("--corpus", help="hexkernels checkout (default: $HEXKERNELS_CORPUS)")
    ap.add_argument("--harness", help="prebuilt harness binary (no corpus)")
    ap.add_argument("--timeout", type=float, default=300.0)
    ap.add_argument("--useful-ops", type=float)
    ap.add_argument("--work-bytes", type=float)
    ap.add_argument("--dtype")
    a = ap.parse_args(argv)
    fb = evaluate(a.task_id, a.candidate, a.corpus, a.harness, a.timeout, a.useful_ops,
                  a.work_bytes, a.dtype)
    print(json.dumps(fb))
    return 0 if fb["correct"] else 1


if __name__ == "__main__":
    sys.exit(main())
