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
REFERENCE = Path(os.environ.get("REFERENCE", "/root/reference"))
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


def main() -> int:
    if not (REFERENCE / "compiler").exists():
        print(f"reference checkout not found at {REFERENCE}", file=sys.stderr)
        return 1
    sys.path.insert(0, str(ROOT / "emmy-hackathon-2026_b200"))
    from compiler.synth import rescale, write_problem
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
        irs, meta = rescale(GOLDEN / "x_l_rmsnorm_w", {64: 4096, 512: 4096},
                            constants={"mean_count": 4096.0}, problem_id="ref_rmsnorm_4096")
        jobs.append((write_problem(irs, meta, Path(td) / "rms"), "ref_rmsnorm_4096"))
        irs, meta = rescale(GOLDEN / "x_r_unpinned_sum", {64: 1 << 20, 65536: 1 << 30},
                            problem_id="ref_sum_2p30")
        jobs.append((write_problem(irs, meta, Path(td) / "sum"), "ref_sum_2p30"))
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
