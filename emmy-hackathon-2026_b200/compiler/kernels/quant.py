"""FP8 (e4m3) per-tensor quantisation and the FP8 GEMM configuration.

The reference has no FP8 GEMM (``compiler/mma.py:143-155`` rejects non-16-bit
fragments); its FP8 support is rounding values to e4m3 in registers with torch's
``float8_e4m3fn`` semantics -- round to nearest even, saturate to +-448
(``compiler/dtypes.py:181-227``).  The BASELINE FP8 configuration quantises A and B
with per-tensor scales ``s = amax / 448`` and multiplies the e4m3 operands with f32
accumulation, dequantising in the epilogue: ``C = (A_q . B_q) * s_a * s_b`` in bf16.

* amax: the whole-array reduction template on the abs-max IR family
  (``tests/problems/x_r_abs_max``), rescaled to the operand size;
* quantise: ``q = e4m3(x / s)`` with ``div.rn.f32`` (IEEE division, as torch's
  ``x / s``) and ``cvt.rn.satfinite.e4m3x2.f32`` (nearest even, saturating), 128-bit
  loads, 32-bit stores of four e4m3 values;
* GEMM: the tcgen05 GEMM template with ``kind::f8f6f4`` (K = 32 per instruction,
  128 K per 128-byte stage row) and the ``scale2`` epilogue.
"""

from __future__ import annotations

from ..ptx import Ptx, entry, f32_hex, module
from .gemm import GemmConfig, choose_tiling, emit_gemm_module

FP8_MAX = 448.0
SMS = 148


def emit_quantize_module(n: int, name: str = "k_quantize_e4m3") -> str:
    """``q[i] = e4m3(x[i] / (amax[0] / 448))``; also writes the scale to ``scale[0]``.
    Parameters: x (f32), amax (f32 scalar), q (e4m3 bytes), scale (f32 scalar)."""
    if n % 4:
        raise NotImplementedError("quantisation of a length that is not a multiple of 4")
    p = Ptx()
    regs = {}
    for nm in ("x", "amax", "q", "scale"):
        r = p.reg("b64")
        p.emit(f"ld.param.u64 {r}, [param_{nm}]\ncvta.to.global.u64 {r}, {r}")
        regs[nm] = r
    am, s = p.reg("f32"), p.reg("f32")
    p.emit(f"ld.global.f32 {am}, [{regs['amax']}]\ndiv.rn.f32 {s}, {am}, {f32_hex(FP8_MAX)}")
    tid, cta, gi = p.reg("u32"), p.reg("u32"), p.reg("b64")
    pz = p.reg("pred")
    cta_n = 256
    grid = min(SMS * 8, max(1, -(-n // (4 * cta_n))))
    p.emit(f"""
        mov.u32 {tid}, %tid.x
        mov.u32 {cta}, %ctaid.x
        or.b32 {tid}, {tid}, {cta}
        setp.eq.u32 {pz}, {tid}, 0
        @{pz} st.global.f32 [{regs['scale']}], {s}
        mov.u32 {tid}, %tid.x
        mad.wide.u32 {gi}, {cta}, {cta_n}, 0
    """)
    w = p.reg("b64")
    p.emit(f"cvt.u64.u32 {w}, {tid}\nadd.s64 {gi}, {gi}, {w}")
    loop, done = p.label("q"), p.label("q_done")
    pg = p.reg("pred")
    p.place(loop)
    p.emit(f"setp.ge.u64 {pg}, {gi}, {n // 4}\n@{pg} bra {done}")
    ax, aq = p.reg("b64"), p.reg("b64")
    x = p.regs("f32", 4)
    y = p.regs("f32", 4)
    h0, h1, out = p.reg("b16"), p.reg("b16"), p.reg("b32")
    p.emit(f"""
        mad.lo.s64 {ax}, {gi}, 16, {regs['x']}
        mad.lo.s64 {aq}, {gi}, 4, {regs['q']}
        ld.global.nc.v4.f32 {{{', '.join(x)}}}, [{ax}]
        div.rn.f32 {y[0]}, {x[0]}, {s}
        div.rn.f32 {y[1]}, {x[1]}, {s}
        div.rn.f32 {y[2]}, {x[2]}, {s}
        div.rn.f32 {y[3]}, {x[3]}, {s}
        cvt.rn.satfinite.e4m3x2.f32 {h0}, {y[1]}, {y[0]}
        cvt.rn.satfinite.e4m3x2.f32 {h1}, {y[3]}, {y[2]}
        mov.b32 {out}, {{{h0}, {h1}}}
        st.global.b32 [{aq}], {out}
        add.s64 {gi}, {gi}, {grid * cta_n}
        bra.uni {loop}
    """)
    p.place(done)
    p.emit("ret")
    params = [".param .u64 param_x", ".param .u64 param_amax", ".param .u64 param_q",
              ".param .u64 param_scale"]
    text = entry(name, params, p, maxntid=cta_n)
    launch = {"kind": "quantize", "grid": [grid, 1, 1], "block": [cta_n, 1, 1], "cluster": [1, 1, 1],
              "smem": 0, "extra_params": [], "bytes": 5 * n}
    return module([text], launch)


def fp8_gemm_config(M: int, N: int, K: int, name: str = "k_gemm_e4m3") -> GemmConfig:
    """C[M,N] (bf16) = (A_q[M,K] . B_q[K,N]) * s_a * s_b with e4m3 operands.
    Parameters: a, b (e4m3), c (bf16), sa, sb (f32 scalars)."""
    return GemmConfig(M=M, N=N, K=K, ab="e4m3", c="bf16", b_kmajor=False, **choose_tiling(M, N, 1, 128),
                      epilogue=(("scale2", "sa", "sb"),), name=name, a_param="a", b_param="b",
                      c_param="c", buffers=("a", "b", "c", "sa", "sb"))


def emit_fp8_gemm_module(M: int, N: int, K: int, name: str = "k_gemm_e4m3") -> str:
    if K % 16 or N % 16:
        raise NotImplementedError("e4m3 operand rows must be 16-byte aligned (TMA)")
    return emit_gemm_module(fp8_gemm_config(M, N, K, name))
