#!/usr/bin/env python3
"""Golden vectors for the K-quant oracle (Q4_K, Q6_K).

mote-reference rejects K-quants, so the published ggml dequantization is the
reference here, as the ``gguf`` Python package (llama.cpp project, version
0.19.0, MIT) implements it in ``gguf.quants``.  This script draws seeded
random blocks (finite f16 scales, every other bit random), decodes them with
gguf 0.19.0 and stores blocks and f32 results in ``kquant_golden.npz``.  The
tests compare the oracle (and, on a GPU, the device decode) with the stored
values bit for bit, without importing gguf.

    python tests/golden/make_kquant_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np


def random_blocks(rng, fmt: str, n: int) -> np.ndarray:
    if fmt == "q4_k":
        b = rng.integers(0, 256, (n, 144), dtype=np.uint8)
        # d, dmin: positive finite f16 in the range real weights use
        d = (rng.uniform(1e-4, 4e-3, n)).astype(np.float16).view(np.uint8).reshape(n, 2)
        dm = (rng.uniform(1e-4, 4e-3, n)).astype(np.float16).view(np.uint8).reshape(n, 2)
        b[:, 0:2], b[:, 2:4] = d, dm
    else:
        b = rng.integers(0, 256, (n, 210), dtype=np.uint8)
        d = (rng.uniform(1e-5, 2e-4, n)).astype(np.float16).view(np.uint8).reshape(n, 2)
        b[:, 208:210] = d
    return b


def main() -> None:
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    from importlib.metadata import version

    assert version("gguf") == "0.19.0", version("gguf")
    rng = np.random.default_rng(20240611)
    out = {}
    for fmt, qt in (("q4_k", T.Q4_K), ("q6_k", T.Q6_K)):
        blocks = random_blocks(rng, fmt, 48)
        # edge blocks: all-zero, all-ones bytes with a unit scale
        blocks[0, :] = 0
        blocks[1, :] = 0xFF
        if fmt == "q4_k":
            blocks[1, 0:4] = np.array([0x3C00, 0x3C00], np.uint16).view(np.uint8)
        else:
            blocks[1, 208:210] = np.array([0x3C00], np.uint16).view(np.uint8)
        vals = quants.dequantize(blocks.reshape(-1), qt).reshape(-1).astype(np.float32)
        out[f"{fmt}_blocks"] = blocks
        out[f"{fmt}_values"] = vals.view(np.uint32)
    out["gguf_version"] = np.array("0.19.0")
    np.savez_compressed(Path(__file__).with_name("kquant_golden.npz"), **out)


if __name__ == "__main__":
    main()
