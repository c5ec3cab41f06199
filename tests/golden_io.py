"""Helpers to read the golden fixtures written by ``tests/golden/make_golden.py``."""

from __future__ import annotations

import os

import numpy as np

from oracle import int4_oracle as orc

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name: str) -> dict:
    with np.load(os.path.join(HERE, name)) as z:
        return {k: z[k] for k in z.files}


def to_f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    """Decode a stored array (raw uint16 bits for 16-bit floats) to float32."""
    if dtype == "bf16":
        return orc.bf16_bits_to_f32(arr)
    if dtype == "f16":
        return arr.view(np.float16).astype(np.float32)
    return arr.astype(np.float32)


def cases(d: dict) -> list[str]:
    return sorted({k.rsplit(".", 1)[0] for k in d})
