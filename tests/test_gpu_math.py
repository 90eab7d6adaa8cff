"""This back end's own elementwise math on the B200, against its stated error bounds.

exp (Cody-Waite split of x log2 e + ex2.approx), log (lg2.approx * ln 2) and erf
(Abramowitz & Stegun 7.1.26) are written here from the mathematics, not taken from a
math library; each is checked over a sweep of f32 inputs against f64 numpy / math.
The kernels are one-op element maps built in emmy's IR format.
"""

import math

import numpy as np
import pytest

F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"


def _unary_spec(op: str, n: int):
    from compiler.ir import parse_stmt
    from compiler.loader import KernelSpec, Param
    body = parse_stmt(
        f"Tile(axes=(Axis(name='a0', extent=Dim({n}), window=None),), body=("
        f"Load(names=('in0',), input='x', index=(Var(name='a0'),), dtype={F32}), "
        f"Assign(name='v0', op=ElementwiseImpl('{op}'), args=('in0',), dtype={F32}), "
        f"Write(output='y', index=(Var(name='a0'),), values=('v0',), value_dtype={F32}, atomic=False, "
        f"swizzle='NONE')), block_threads=256, aux_threads=0, raster_axes=None, raster_group=None, "
        f"raster_orient='m')")
    params = (Param("x", "f32", (n,)), Param("y", "f32", (n,)))
    return KernelSpec(f"k_{op}_sweep", (body,), params, None, None, {},
                      buffers={p.name: p for p in params})


def _run(op: str, x: np.ndarray) -> np.ndarray:
    import emmyrt
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    x = np.ascontiguousarray(x, dtype=np.float32)
    ck = CompiledKernel.from_spec(_unary_spec(op, x.size))
    dx, dy = DeviceBuffer(x.nbytes), DeviceBuffer(x.nbytes)
    dx.upload(x)
    ck({"x": dx.ptr, "y": dy.ptr})
    emmyrt.stream_wait(0, 60)
    y = np.zeros_like(x)
    dy.download(y)
    return y


@pytest.mark.gpu
def test_erf_within_abramowitz_stegun_bound(runtime):
    x = np.linspace(-6, 6, 1 << 16, dtype=np.float32)
    got = _run("erf", x).astype(np.float64)
    ref = np.array([math.erf(float(v)) for v in x])
    # the method's 1.5e-7 in exact arithmetic, plus its f32 evaluation: the rounding of
    # x^2 inside exp(-x^2), of the degree-5 polynomial in t and of 1 - q e (measured:
    # 5.0e-7 at worst over this sweep)
    assert np.max(np.abs(got - ref)) <= 6e-7


@pytest.mark.gpu
def test_exp_relative_error(runtime):
    x = np.linspace(-80, 80, 1 << 16, dtype=np.float32)
    got = _run("exp", x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert np.max(rel) <= 4e-7          # a few ulp: ex2.approx plus the split argument


@pytest.mark.gpu
def test_log_error(runtime):
    x = np.exp(np.linspace(-40, 40, 1 << 16)).astype(np.float32)
    got = _run("log", x).astype(np.float64)
    ref = np.log(x.astype(np.float64))
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)) <= 1e-6


@pytest.mark.gpu
def test_tanh_error(runtime):
    # the series below |x| = 0.55, 1 - 2 / (exp(2|x|) + 1) above: a few ulp relative
    x = np.concatenate([np.linspace(-12, 12, 1 << 16), np.linspace(-0.6, 0.6, 1 << 14),
                        [0.0, -0.0, 1e-30, -1e-30, 100.0, -100.0]]).astype(np.float32)
    got = _run("tanh", x).astype(np.float64)
    ref = np.tanh(x.astype(np.float64))
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)) <= 6e-7
    assert np.array_equal(np.signbit(got[x == 0]), np.signbit(x[x == 0]))


@pytest.mark.gpu
def test_sigmoid_error(runtime):
    x = np.linspace(-100, 100, 1 << 16, dtype=np.float32)
    got = _run("sigmoid", x).astype(np.float64)
    ref = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    tiny = ref > 1e-30
    assert np.max(np.abs(got[tiny] - ref[tiny]) / ref[tiny]) <= 6e-7


F64 = "DataType(name='f64', np=dtype('float64'), nbytes=8)"


def _run_f64_exp(x: np.ndarray) -> np.ndarray:
    import emmyrt
    from compiler.ir import parse_stmt
    from compiler.loader import KernelSpec, Param
    from emmyrt import DeviceBuffer
    from emmyrt.runner import CompiledKernel
    n = x.size
    body = parse_stmt(
        f"Tile(axes=(Axis(name='a0', extent=Dim({n}), window=None),), body=("
        f"Load(names=('in0',), input='x', index=(Var(name='a0'),), dtype={F64}), "
        f"Assign(name='v0', op=ElementwiseImpl('exp'), args=('in0',), dtype={F64}), "
        f"Write(output='y', index=(Var(name='a0'),), values=('v0',), value_dtype={F64}, atomic=False, "
        f"swizzle='NONE')), block_threads=256, aux_threads=0, raster_axes=None, raster_group=None, "
        f"raster_orient='m')")
    params = (Param("x", "f64", (n,)), Param("y", "f64", (n,)))
    ck = CompiledKernel.from_spec(KernelSpec("k_exp_f64_sweep", (body,), params, None, None, {},
                                             buffers={p.name: p for p in params}))
    dx, dy = DeviceBuffer(x.nbytes), DeviceBuffer(x.nbytes)
    dx.upload(x)
    ck({"x": dx.ptr, "y": dy.ptr})
    emmyrt.stream_wait(0, 60)
    y = np.zeros_like(x)
    dy.download(y)
    return y


@pytest.mark.gpu
def test_exp_f64_error(runtime):
    # Cody-Waite reduction with ln 2 in two parts and the Taylor series to r^13: a few ulp
    x = np.concatenate([np.linspace(-708, 709.78, 1 << 16), np.linspace(-1, 1, 1 << 14)])
    got = _run_f64_exp(x)
    ref = np.exp(x)
    assert np.max(np.abs(got - ref) / ref) <= 8 * 2.0 ** -53
    # subnormal results, the overflow threshold, the limits and NaN
    edge = np.array([-720.0, -740.0, 709.782, -800.0, 800.0, 0.0, np.nan])
    g = _run_f64_exp(edge)
    assert np.allclose(g[:3], np.exp(edge[:3]), rtol=1e-12, atol=2e-323)   # (subnormal spacing 5e-324)
    assert np.array_equal(g[3:6], [0.0, np.inf, 1.0]) and np.isnan(g[6])


@pytest.mark.gpu
@pytest.mark.parametrize("op,fn", [("sin", np.sin), ("cos", np.cos)])
def test_sin_cos_error(runtime, op, fn):
    # Cody-Waite by pi/2 and the Taylor series on |r| <= pi/4: a few ulp of 1 (absolute)
    x = np.concatenate([np.linspace(-100, 100, 1 << 16), np.linspace(-4, 4, 1 << 14),
                        [0.0, np.pi / 2, np.pi, 3000.0]]).astype(np.float32)
    got = _run(op, x).astype(np.float64)
    ref = fn(x.astype(np.float64))
    assert np.max(np.abs(got - ref)) <= 4e-7
