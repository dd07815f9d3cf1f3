"""bfloat16 rounding on float32 numpy arrays (test infrastructure).

Values are carried as float32 arrays whose contents are exactly representable in
bfloat16; ``rnd`` performs round-to-nearest-even, the conversion XLA applies when an
op's output dtype is bfloat16 (e.g. ``.astype(x.dtype)`` in
``src/counterfact_kv_eviction/jax_inference.py:618,632-633``).
"""

from __future__ import annotations

import numpy as np


def rnd(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    r = ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        r = r.copy()
        r[nan] = np.float32("nan")
    return r.reshape(a.shape)


def to_u16(x) -> np.ndarray:
    """Bit pattern (uint16) of bfloat16-representable float32 values."""
    a = np.ascontiguousarray(rnd(x), dtype=np.float32)
    return (a.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_u16(bits) -> np.ndarray:
    """float32 values of raw bfloat16 bit patterns."""
    b = np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return b.view(np.float32)
