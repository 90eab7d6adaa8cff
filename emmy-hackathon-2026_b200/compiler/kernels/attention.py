"""tcgen05 attention template (in progress)."""


def emit_attention(spec):
    raise NotImplementedError(f"kernel {spec.name}: tcgen05 attention template not built yet")
