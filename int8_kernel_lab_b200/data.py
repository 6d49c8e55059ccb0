"""Seeded synthetic inputs.

The reference draws x, w from uniform_int_distribution(-4, 4) and the bias from
(-31, 31) with std::mt19937(20260925) (src/conv_lab.cu:149-157).  The B200
benchmark uses the full int8 range and a bias in [-65536, 65536].  Both ranges
are available.  Generation is MT19937 seeded with the reference seed (numpy's
legacy RandomState uses the same seeding as std::mt19937(seed)); the mapping to
integers differs from libstdc++'s distribution, which does not matter because
the oracle and the GPU always consume the same host buffers.
"""
from __future__ import annotations

import numpy as np

from .shape import ConvShape

REFERENCE_SEED = 20260925

RANGES = {
    # name: (x/w low, x/w high, bias low, bias high), inclusive
    "full": (-128, 127, -65536, 65536),
    "reference": (-4, 4, -31, 31),
}


def make_inputs(shape: ConvShape, seed: int = REFERENCE_SEED, values: str = "full"):
    """(input NHWC int8, filter KRSC int8, bias K int32) as numpy arrays."""
    lo, hi, blo, bhi = RANGES[values]
    rng = np.random.RandomState(seed)
    x = rng.randint(lo, hi + 1, size=shape.input_elements, dtype=np.int16).astype(np.int8)
    w = rng.randint(lo, hi + 1, size=shape.filter_elements, dtype=np.int16).astype(np.int8)
    b = rng.randint(blo, bhi + 1, size=shape.k, dtype=np.int64).astype(np.int32)
    return x, w, b
