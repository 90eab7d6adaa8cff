"""Every BASELINE configuration's per-GPU shard at 1 / 2 / 4 / 8 GPUs, synthesised from its IR
family and compiled on the CPU: the kernel each rank of ``bench.py --gpus N`` launches is
the template the configuration's family selects, its launch fits one SM's shared memory
and the persistent grid, and the work it states adds up to the whole problem's."""

import json

import pytest

from conftest import ROOT  # noqa: F401  (puts the package on sys.path)

KIND = {"gemm": "gemm", "attention": "attention", "rmsnorm": "row_reduce", "softmax": "row_reduce",
        "sum": "full_reduce"}


def _compile(name, rank, world, tmp_path):
    import baseline_configs as bc
    from compiler import compile_kernel, parse_launch, synth
    from compiler.loader import load
    irs, meta = bc.shard_problem(name, rank, world)
    d = synth.problem_dir(irs, meta, root=tmp_path)
    k = meta["kernels"][0]
    return parse_launch(compile_kernel(load(d / f"{k['entry']}.ir.json"))), meta


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("name", ["gemm_8192", "gemm_4096x14336x4096", "gemm_2048", "gemm_512",
                                  "attention", "rmsnorm", "softmax", "sum"])
def test_shard_module(name, world, tmp_path):
    import baseline_configs as bc
    family = bc.CONFIGS[name].family
    for rank in sorted({0, world - 1}):
        launch, meta = _compile(name, rank, world, tmp_path)
        assert launch["kind"] == KIND[family if family != "row" else name], launch["kind"]
        assert launch.get("smem", 0) <= 232448
        grid = launch["grid"][0]
        if launch["kind"] in ("gemm", "attention"):
            assert grid <= 148
        if family == "gemm":
            assert launch["flops"] == bc.work(name, rank, world)
        if name == "attention":
            assert launch["flops"] == bc.work(name, rank, world)
        if name == "sum":
            assert launch["count"] * 4 == bc.work(name, rank, world)
            scratch = [e for e in launch["extra_params"] if e["kind"] == "scratch"]
            assert scratch and scratch[0]["bytes"] == 16 + 8 * grid
        json.dumps(meta)                   # the shard's meta.json is plain JSON
    if family == "gemm":
        assert sum(bc.work(name, r, world) for r in range(world)) == bc.work(name, 0, 1)
