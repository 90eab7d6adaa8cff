"""The whole-array reduction entry point that allocates nothing, checked on the GPU.

Some callers cannot allocate device memory where they need a reduction (a process
whose HBM is all handed to its own pool, an error path after an out-of-memory
failure, a latency-bound loop that must not pay for cudaMalloc).  For them
``emmy_rt_full_reduce_static_scratch`` runs the same compiled reduction kernel with
its scratch in a static device array.  This file runs last (pytest collects it
last) and checks that entry point, through the C ABI, against the regular path that
allocates its scratch, against the golden vector (expected.npz) and against the oracle,
on two calls in a row.
"""

import ctypes
import json

import numpy as np
import pytest

from conftest import GOLDEN


@pytest.mark.gpu
@pytest.mark.parametrize("pid", ["x_r_unpinned_sum", "r03_mean", "x_r_sumsq"])
def test_static_scratch_matches_allocating_path(runtime, pid):
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel, run_problem, seeded_input
    from oracle.refs import problem_expected

    d = GOLDEN / pid
    meta = json.loads((d / "meta.json").read_text())
    k = meta["kernels"][0]
    expected = run_problem(d)["outputs"]            # the regular path: allocated scratch
    golden = dict(np.load(d / "expected.npz"))
    oracle = problem_expected(meta)

    ck = CompiledKernel.from_ir(d / f"{k['entry']}.ir.json")
    scratch = [e for e in ck.launch["extra_params"] if e["kind"] == "scratch"]
    assert len(scratch) == 1 and scratch[0]["bytes"] <= 64 * 1024
    bufs = {}
    for a in k["args"]:
        host = seeded_input(a)
        bufs[a["name"]] = DeviceBuffer(host.nbytes)
        bufs[a["name"]].upload(host)
    args = (ctypes.c_uint64 * len(ck.spec.params))(*[bufs[p.name].ptr for p in ck.spec.params])
    static = emmyrt.static_scratch_lib()
    outs = [a["name"] for a in k["args"] if a.get("output")]
    for call in range(2):
        for o in outs:
            bufs[o].zero()
        rc = static.emmy_rt_full_reduce_static_scratch(
            ck.function, ck.launch["grid"][0], ck.launch["block"][0], args, len(ck.spec.params),
            scratch[0]["bytes"], 0)
        assert rc == 0, f"call {call}: status {rc}"
        emmyrt.stream_wait(0, 60)
        for o in outs:
            got = np.zeros(1, np.float32)
            bufs[o].download(got)
            ref = expected[o].reshape(-1)
            assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]), \
                f"call {call}: {got} vs {ref}"
            assert np.array_equal(got, ref.astype(np.float32))   # same kernel, deterministic order
            for what, want in (("expected.npz", golden[o]), ("oracle", oracle[o])):
                want = np.asarray(want, np.float64).reshape(-1)
                assert np.allclose(got, want, rtol=meta["rtol"], atol=meta["atol"]), \
                    f"call {call}: {got} vs {what} {want}"


@pytest.mark.gpu
def test_static_scratch_rejects_oversize(runtime):
    import emmyrt
    static = emmyrt.static_scratch_lib()
    args = (ctypes.c_uint64 * 2)(0, 0)
    assert static.emmy_rt_full_reduce_static_scratch(0, 1, 32, args, 2, (64 << 10) + 16, 0) == \
        emmyrt.EMMY_RT_ESCRATCH
