"""Hand-written sm_100a PTX templates, one per kernel family the IR lowers to."""

from __future__ import annotations


def _has(body, kinds) -> bool:
    for s in body:
        k = type(s).__name__
        if k in kinds:
            return True
        for attr in ("body", "else_body"):
            sub = getattr(s, attr, None)
            if isinstance(sub, tuple) and _has(sub, kinds):
                return True
    return False


def select(spec) -> str:
    """Pick the template for ``spec`` and emit its module."""
    body = spec.body
    if _has(body, {"MmaSyncPtx"}):
        if _has(body, {"FragmentRowReduce"}):
            from .attention import emit_attention
            return emit_attention(spec)
        from .gemm import emit_gemm
        try:
            return emit_gemm(spec)
        except NotImplementedError as err:
            # two contractions in one kernel (a shared-A pair, or a chain through an A
            # tile computed in the kernel): an element map of the same arithmetic
            from .fused import chained_gemm_spec, dual_gemm_spec, emit_chained_rows
            from .pointwise import emit_map
            try:
                return emit_chained_rows(spec)
            except NotImplementedError:
                pass
            for synth in (dual_gemm_spec, chained_gemm_spec):
                try:
                    return emit_map(synth(spec))
                except NotImplementedError:
                    continue
            raise err
    if _has(body, {"WarpShuffle"}):
        # emmy's SIMT form of attention (an online softmax over streamed keys) runs on the
        # tensor-core attention template; every other cooperative reduction on the
        # streaming reduction template
        from .attention import analyze_simt, emit_attention_module
        try:
            cfg = analyze_simt(spec)
        except NotImplementedError:
            cfg = None
        if cfg is not None:
            return emit_attention_module(cfg)
        # a dot product per output element, reduced across the warp: a matmul
        from .gemm import analyze_f32, emit_gemm_module
        try:
            gcfg = analyze_f32(spec)
        except NotImplementedError:
            gcfg = None
        if gcfg is not None:
            return emit_gemm_module(gcfg)
        from .reduce import emit_reduction
        if any(q.dtype in ("i32", "i64", "f64") for q in spec.params):
            # integer / f64 buffers: one thread per output, the reduction serial
            from .pointwise import emit_map, serialize_cooperative
            return emit_map(serialize_cooperative(spec))
        return emit_reduction(spec)
    # emmy's register-tiled f32 attention (an online softmax per output element): one
    # warp per query row over keys staged in shared memory
    from .attention_f32 import analyze as analyze_attn_f32, emit_module as emit_attn_f32
    try:
        acfg = analyze_attn_f32(spec)
    except NotImplementedError:
        acfg = None
    if acfg is not None:
        return emit_attn_f32(spec, acfg)
    # emmy's SIMT f32 matmuls (FMA over cp.async-staged tiles) run on the tensor cores
    # as 3xTF32
    from .gemm import analyze_f32, emit_gemm_module
    try:
        cfg = analyze_f32(spec)
    except NotImplementedError:
        cfg = None
    if cfg is not None:
        return emit_gemm_module(cfg)
    # no cooperative combine and no tensor-core work: one element per thread (the sum
    # of split-K partial slices, elementwise tails)
    from .pointwise import emit_map
    try:
        return emit_map(spec)
    except NotImplementedError:
        pass
    raise NotImplementedError(
        f"kernel {spec.name}: no sm_100a template for this IR family "
        "(tensor-core GEMM, tensor-core attention and cooperative reductions are supported)")
