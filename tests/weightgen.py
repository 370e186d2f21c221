"""Seeded synthetic projection weights in the GGUF block layouts (test helper).

Every byte pattern of the quant payload is a valid weight, so blocks are
random bytes with the fp16 scales drawn from a range that gives the product
W.x roughly unit variance for unit-variance x.  The layouts are those of
cpp/quant.hpp:33-74 (F32/F16 rows are plain arrays).
"""
from __future__ import annotations

import numpy as np

from picolm_qwen_b200 import abi

BLOCK = {abi.WT_F32: (1, 4), abi.WT_F16: (1, 2), abi.WT_Q4_0: (32, 18), abi.WT_Q8_0: (32, 34),
         abi.WT_Q4_K: (256, 144), abi.WT_Q6_K: (256, 210)}
NAMES = {abi.WT_F32: "F32", abi.WT_F16: "F16", abi.WT_Q4_0: "Q4_0", abi.WT_Q8_0: "Q8_0",
         abi.WT_Q4_K: "Q4_K", abi.WT_Q6_K: "Q6_K"}


def _f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float16).view(np.uint16)


def make(wtype: int, n_in: int, n_out: int, rng: np.random.Generator) -> np.ndarray:
    """n_out rows of n_in weights as uint8 bytes."""
    e, b = BLOCK[wtype]
    assert n_in % e == 0
    nb = n_out * (n_in // e)
    a = 1.0 / np.sqrt(n_in)
    if wtype == abi.WT_F32:
        return (rng.uniform(-np.sqrt(3) * a, np.sqrt(3) * a, (n_out, n_in))).astype(np.float32).view(np.uint8).ravel()
    if wtype == abi.WT_F16:
        return (rng.uniform(-np.sqrt(3) * a, np.sqrt(3) * a, (n_out, n_in))).astype(np.float16).view(np.uint8).ravel()
    blk = rng.integers(0, 256, (nb, b), dtype=np.uint8)
    if wtype == abi.WT_Q4_0:    # d * (nibble - 8): nibbles ~ U{0..15}, std ~ 4.6
        blk[:, 0:2] = _f16_bits(rng.uniform(0.5, 1.5, nb) * a / 4.6).view(np.uint8).reshape(nb, 2)
    elif wtype == abi.WT_Q8_0:  # d * int8: std ~ 74
        blk[:, 0:2] = _f16_bits(rng.uniform(0.5, 1.5, nb) * a / 74).view(np.uint8).reshape(nb, 2)
    elif wtype == abi.WT_Q4_K:  # d*sc*q - dmin*mn: sc, mn 6-bit, q 4-bit
        blk[:, 0:2] = _f16_bits(rng.uniform(0.5, 1.5, nb) * a / 140).view(np.uint8).reshape(nb, 2)
        blk[:, 2:4] = _f16_bits(rng.uniform(0.0, 1.0, nb) * a / 100).view(np.uint8).reshape(nb, 2)
    elif wtype == abi.WT_Q6_K:  # d * sc * (q - 32): sc int8, q 6-bit
        blk[:, 208:210] = _f16_bits(rng.uniform(0.5, 1.5, nb) * a / (74 * 18)).view(np.uint8).reshape(nb, 2)
    return blk.ravel()
