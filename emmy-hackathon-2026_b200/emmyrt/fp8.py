"""FP8 e4m3 GEMM pipeline on the B200: per-tensor amax -> quantise -> tcgen05 GEMM.

The amax kernel is the whole-array reduction template compiled from an abs-max IR
in emmy's own format (the ``x_r_abs_max`` family: ``acc = maximum(acc, abs(x))``
over one cooperative tile, warp shuffle + tree combine, lane-0 write), the quantiser
and the GEMM are the templates in ``compiler/kernels/quant.py``.  Quantisation is
bit-exact with torch's ``(x / (amax / 448)).to(float8_e4m3fn)``.
"""

from __future__ import annotations

import numpy as np

from . import DeviceBuffer
from .runner import CompiledKernel

_F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"


def absmax_spec(n: int, name: str = "k_amax"):
    """KernelSpec of ``amax = max(|x|)`` over ``n`` f32 values, in emmy's IR format."""
    from compiler.ir import parse_stmt
    from compiler.loader import KernelSpec, Param
    w = 256
    comb = "(Assign(name='acc0', op=ElementwiseImpl('maximum'), args=('acc0', 'acc0__o'), dtype=None),)"
    body = parse_stmt(
        f"Tile(axes=(Axis(name='a0_co', extent=Dim({w}), window=None),), body=("
        f"StridedLoop(axis=Axis(name='a0', extent=Dim({n}), window=None), start=Var(name='a0_co'), "
        f"step=Literal(value={w}, dtype='int'), body=("
        f"Load(names=('in0',), input='x', index=(Var(name='a0'),), dtype={_F32}), "
        f"Assign(name='v0', op=ElementwiseImpl('abs'), args=('in0',), dtype={_F32}), "
        f"Accum(name='acc0', value='v0', op=ElementwiseImpl('maximum'), dtype={_F32}, axes=('a0',), "
        f"base=None)), unroll=False, end=None, seed=True), "
        f"WarpShuffle(state=('acc0',), state_b=('acc0__o',), combine_states={comb}, length=32, "
        f"dtype={_F32}), "
        f"Smem(name='acc0_smem', extents=({w // 32},), dtype='float', align=0), "
        f"Cond(cond=BinaryExpr(op='==', left=Var(name='lane'), right=Literal(value=0, dtype='int')), "
        f"body=(Write(output='acc0_smem', index=(Var(name='warp'),), values=('acc0',), "
        f"value_dtype={_F32}, atomic=False, swizzle='NONE'),), else_body=()), "
        f"Sync(barrier_id=0, count=None, warp=False), "
        f"TreeHalve(bufs=('acc0_smem',), state=('acc0',), state_b=('acc0__o',), combine_states={comb}, "
        f"length={w // 32}, tid_var='warp', dtype={_F32}, barrier_id=0, barrier_count=None, inner=None), "
        f"Cond(cond=BinaryExpr(op='==', left=Var(name='a0_co'), right=Literal(value=0, dtype='int')), "
        f"body=(Write(output='amax', index=(), values=('acc0',), value_dtype={_F32}, atomic=False, "
        f"swizzle='NONE'),), else_body=())), block_threads={w}, aux_threads=0, raster_axes=None, "
        f"raster_group=None, raster_orient='m')")
    params = (Param("x", "f32", (n,)), Param("amax", "f32", (1,)))
    return KernelSpec(name, (body,), params, None, None, {},
                      buffers={p.name: p for p in params})


class Fp8Gemm:
    """C = (e4m3(A / s_a) . e4m3(B / s_b)) * s_a * s_b, s = amax / 448, for fixed shapes."""

    def __init__(self, M: int, N: int, K: int):
        from compiler.kernels.quant import emit_fp8_gemm_module, emit_quantize_module
        self.M, self.N, self.K = M, N, K
        self.amax_a = CompiledKernel.from_spec(absmax_spec(M * K, "k_amax_a"))
        self.amax_b = CompiledKernel.from_spec(absmax_spec(K * N, "k_amax_b"))
        self.quant_a = CompiledKernel.from_module(emit_quantize_module(M * K, "k_quant_a"), "k_quant_a",
                                                  ["x", "amax", "q", "scale"])
        self.quant_b = CompiledKernel.from_module(emit_quantize_module(K * N, "k_quant_b"), "k_quant_b",
                                                  ["x", "amax", "q", "scale"])
        self.gemm = CompiledKernel.from_module(emit_fp8_gemm_module(M, N, K), "k_gemm_e4m3",
                                               ["a", "b", "c", "sa", "sb"])
        self.qa, self.qb = DeviceBuffer(M * K), DeviceBuffer(K * N)
        self.am = DeviceBuffer(16)
        self.bm = DeviceBuffer(16)
        self.sa, self.sb = DeviceBuffer(16), DeviceBuffer(16)

    def quantize(self, a_ptr: int, b_ptr: int, stream: int = 0, amax_b_hook=None) -> None:
        """Quantise A and B on ``stream``.  When B is one GPU's N-panel of a larger B,
        ``amax_b_hook(ptr, stream)`` turns the panel's amax (one f32 on the device) into
        the whole B's before B is quantised (an all-reduce with max over the GPUs)."""
        self.amax_a({"x": a_ptr, "amax": self.am.ptr}, stream)
        self.amax_b({"x": b_ptr, "amax": self.bm.ptr}, stream)
        if amax_b_hook is not None:
            amax_b_hook(self.bm.ptr, stream)
        self.quant_a({"x": a_ptr, "amax": self.am.ptr, "q": self.qa.ptr, "scale": self.sa.ptr}, stream)
        self.quant_b({"x": b_ptr, "amax": self.bm.ptr, "q": self.qb.ptr, "scale": self.sb.ptr}, stream)

    def gemm_params(self, c_ptr: int) -> list:
        return self.gemm.params({"a": self.qa.ptr, "b": self.qb.ptr, "c": c_ptr, "sa": self.sa.ptr,
                                 "sb": self.sb.ptr})

    def scales(self) -> tuple[float, float]:
        a, b = np.zeros(4, np.float32), np.zeros(4, np.float32)
        self.sa.download(a)
        self.sb.download(b)
        return float(a[0]), float(b[0])


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> f32 values (sign, 4-bit exponent with bias 7, 3-bit mantissa)."""
    q = np.asarray(q, dtype=np.uint8).astype(np.int32)
    s = np.where(q & 0x80, -1.0, 1.0)
    e = (q >> 3) & 0xF
    m = q & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    val = np.where((q & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)
