#!/usr/bin/env python3
"""Compile problems with the UNMODIFIED reference compiler into oracle/_ref/ptx/.

TEST INFRASTRUCTURE ONLY (a second oracle and a same-GPU baseline): the reference's own
sm_89 PTX (mma.sync / SIMT), assembled for sm_100a on the B200 and launched with
meta.json's own grid, block and shared memory, next to this back end's kernels.

The reference imports ``emmy.compiler.graph.Graph`` (``compiler/loader.py:14``); emmy-ml is
not installable here, so a shim package maps that import to this repository's own
``Graph.from_dict`` restatement.  The reference runs in a subprocess with only its own
checkout and the shim on ``sys.path`` (both packages are called ``compiler``).

Only kernels whose reference lowering uses no ``exp`` are built: the reference's ``exp``
(``compiler/ops.py:55-78``) reproduces a CUDA math-library sequence, so its softmax and
attention PTX is not used here.  Output (git-ignored, travels to the GPU box):
``oracle/_ref/ptx/<problem>/{<entry>.ptx, meta.json}``.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
# the reference checkout: $REFERENCE, else a "reference" folder beside this repository
REFERENCE = Path(os.environ.get("REFERENCE", ROOT.parent / "reference"))
OUT = ROOT / "oracle" / "_ref" / "ptx"
GOLDEN = ROOT / "tests" / "golden" / "problems"

# golden fixtures (parity) and BASELINE-family problems (timing)
FIXTURES = ["x_h_mm_1024", "x_h_mm_256", "x_h_mm_relu", "f01_rmsnorm", "f03_l2norm", "x_l_rmsnorm_w",
            "r02_big_sum", "r04_row_sum", "x_r_unpinned_sum", "x_r_rowsum_wide"]

SHIM = '''
import importlib.util, sys
spec = importlib.util.spec_from_file_location("emmy_b200_ir", {ir!r})
mod = importlib.util.module_from_spec(spec); sys.modules["emmy_b200_ir"] = mod; spec.loader.exec_module(mod)
Graph = mod.Graph
'''

DRIVER = '''
import sys, json
from pathlib import Path
sys.path.insert(0, {ref!r}); sys.path.insert(0, {shim!r})
from compiler import compile_kernel, load
src, dst = Path(sys.argv[1]), Path(sys.argv[2])
meta = json.loads((src / "meta.json").read_text())
dst.mkdir(parents=True, exist_ok=True)
for k in meta["kernels"]:
    ptx = compile_kernel(load(src / (k["entry"] + ".ir.json")))
    if "ex2.approx" in ptx:
        raise SystemExit("exp-based kernel: not built")
    (dst / (k["entry"] + ".ptx")).write_text(ptx)
(dst / "meta.json").write_text(json.dumps(meta))
'''


def bf16_gemm_problem(n: int, problem_id: str) -> tuple[dict, dict]:
    """The reference's f16 GEMM family (x_h_mm_1024: 32 x 256 CTA tiles, a two-stage
    cp.async pipeline over K in steps of 32, mma.sync m16n8k16) retyped to bf16 and
    grown to n^3.  Emmy's schedule for it is fixed by the IR: the row / column block
    axes (a0_b, a1_b) and the K loop (_ks) grow with n, the per-CTA tile does not, and
    the launch grows to (n / 32) x (n / 256) CTAs.  The K pipeline's prefetch clamp
    (``_ks + 32 < K ? _ks + 32 : K - 32``) is rewritten for the new K."""
    from compiler.synth import FAMILIES, rescale
    if n % 256:
        raise ValueError("the x_h_mm_1024 schedule tiles N by 256")
    irs, meta = rescale(FAMILIES / "x_h_mm_1024",
                        axes={("a0", 1024): n, ("a1", 1024): n, ("_ks", 1024): n,
                              ("a0_b", 32): n // 32, ("a1_b", 4): n // 256},
                        dtypes={"f16": "bf16"},
                        shapes={"x0": [n, n], "x1": [n, n], "matmul": [n, n]},
                        problem_id=problem_id)
    old = ("right=Literal(value=1024, dtype='int')), if_true=BinaryExpr(op='+', left=Var(name='_ks'), "
           "right=Literal(value=32, dtype='int')), if_false=Literal(value=992, dtype='int')")
    new = old.replace("value=1024", f"value={n}").replace("value=992", f"value={n - 32}")
    for ir in irs.values():
        for node in ir["nodes"].values():
            if node["op"] == "KernelOp":
                body = node["op_fields"]["body"]
                if not any(old in s for s in body):
                    raise ValueError("x_h_mm_1024: the K prefetch clamp was not found")
                node["op_fields"]["body"] = [s.replace(old, new) for s in body]
    meta["kernels"][0]["grid"] = [(n // 32) * (n // 256), 1, 1]
    return irs, meta


def baseline_reference_problems() -> dict:
    """BASELINE configurations (or the largest size the reference's 32-bit indexing
    reaches) in the reference's own IR families."""
    from compiler.synth import rmsnorm_family, sum_family
    return {"ref_rmsnorm_4096": rmsnorm_family(4096, 4096, "ref_rmsnorm_4096"),
            "ref_sum_2p30": sum_family(1 << 30, "ref_sum_2p30"),
            "ref_gemm_bf16_2048": bf16_gemm_problem(2048, "ref_gemm_bf16_2048")}


def main() -> int:
    if not (REFERENCE / "compiler").exists():
        print(f"reference checkout not found at {REFERENCE}", file=sys.stderr)
        return 1
    sys.path.insert(0, str(ROOT / "emmy-hackathon-2026_b200"))
    from compiler.synth import write_problem
    with tempfile.TemporaryDirectory() as td:
        shim = Path(td) / "shim"
        (shim / "emmy" / "compiler").mkdir(parents=True)
        (shim / "emmy" / "__init__.py").write_text("")
        (shim / "emmy" / "compiler" / "__init__.py").write_text("")
        ir_py = ROOT / "emmy-hackathon-2026_b200" / "compiler" / "ir.py"
        (shim / "emmy" / "compiler" / "graph.py").write_text(SHIM.format(ir=str(ir_py)))
        driver = Path(td) / "drive.py"
        driver.write_text(DRIVER.format(ref=str(REFERENCE), shim=str(shim)))
        jobs = [(GOLDEN / f, f) for f in FIXTURES]
        # BASELINE-family sizes the reference's 32-bit indexing can address
        for name, (irs, meta) in baseline_reference_problems().items():
            jobs.append((write_problem(irs, meta, Path(td) / name), name))
        ok = 0
        for src, name in jobs:
            r = subprocess.run([sys.executable, str(driver), str(src), str(OUT / name)],
                               capture_output=True, text=True, env={**os.environ, "PYTHONPATH": ""})
            status = "ok" if r.returncode == 0 else "skipped: " + (r.stderr.strip().splitlines() or ["?"])[-1]
            ok += r.returncode == 0
            print(f"{name}: {status}")
    print(f"{ok} reference modules in {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
