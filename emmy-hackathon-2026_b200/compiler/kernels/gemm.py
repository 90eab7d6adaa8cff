"""tcgen05 GEMM template (in progress)."""


def emit_gemm(spec):
    raise NotImplementedError(f"kernel {spec.name}: tcgen05 GEMM template not built yet")
