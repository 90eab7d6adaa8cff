"""Host (numpy) representations of the IR's buffer types.

Pure numpy: importing this module loads no native library, so CPU-only callers (the
CPU baseline, tests without a GPU) use the same conversions as the runtime.

* ``NP_DTYPE``: the numpy array type a buffer of each IR dtype is held in on the host
  (bf16 as its raw 16-bit patterns, e4m3 as bytes);
* ``f32_to_bf16_bits`` / ``bf16_bits_to_f32``: round to nearest even, as torch's
  ``.to(torch.bfloat16)`` does, and the exact widening back.
"""

from __future__ import annotations

import numpy as np

NP_DTYPE = {"f32": np.float32, "f16": np.float16, "f64": np.float64, "i32": np.int32,
            "i64": np.int64, "bf16": np.uint16, "e4m3": np.uint8, "u8": np.uint8}


def f32_to_bf16_bits(a, out: np.ndarray | None = None) -> np.ndarray:
    """bf16 bit patterns of f32 values (nearest even; NaN stays a quiet NaN)."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    bits = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        bits[nan] = 0x7FC0
    if out is None:
        return bits
    out[...] = bits
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
