"""Shared helpers for the test-suite (golden fixtures, engines, library)."""
from __future__ import annotations

import functools
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")

# North-star parity gates: logits within 2e-2 max-abs of the
# fp32 oracle; greedy argmax equal wherever the oracle's top-2 margin > 1e-2.
LOGIT_TOL = 2e-2
MARGIN = 1e-2


def golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def lib():
    from megakernel_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        _lib.build()
    return _lib.load()


@functools.lru_cache(maxsize=None)
def weights(shape_name: str, seed: int = 0):
    from megakernel_b200 import weights as W
    from megakernel_b200.shapes import SHAPES
    shape = SHAPES[shape_name]
    w = W.random_weights(shape, seed)
    flat, offs = W.flat_bytes(shape, w)
    return shape, w, flat, offs
