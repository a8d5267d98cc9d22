"""Generates tests/golden/quant_golden.npz from gguf-py (the GGML project's Python
implementation of the GGUF block formats, installed with the reference's converter
dependencies).  Run from the repository root:  python tests/golden/make_golden.py

Contents:
  q4k_blocks/q4k_values, q6k_blocks/q6k_values, q80_blocks/q80_values:
      random raw blocks and gguf.quants.dequantize of them;
  q80_src/q80_quant: float rows and gguf.quants.quantize(..., Q8_0), which gguf-py
      documents as bit-exact with ggml-quants.c.
"""
import pathlib

import numpy as np
from gguf import GGMLQuantizationType as QT
from gguf import quants

rng = np.random.default_rng(20261201)


def f16_bytes(v):
    return np.asarray(v, dtype=np.float16).view(np.uint8).reshape(-1, 2)


def q4k(n):
    d = f16_bytes(rng.uniform(1e-4, 2e-2, n))
    dmin = f16_bytes(rng.uniform(1e-5, 5e-3, n))
    rest = rng.integers(0, 256, size=(n, 140), dtype=np.uint8)  # 12 scale bytes + 128 nibble bytes
    return np.concatenate([d, dmin, rest], axis=1)


def q6k(n):
    body = rng.integers(0, 256, size=(n, 208), dtype=np.uint8)  # ql 128, qh 64, scales 16
    d = f16_bytes(rng.uniform(1e-5, 1e-3, n))
    return np.concatenate([body, d], axis=1)


def q80(n):
    d = f16_bytes(rng.uniform(1e-4, 1e-2, n))
    qs = rng.integers(0, 256, size=(n, 32), dtype=np.uint8)
    return np.concatenate([d, qs], axis=1)


out = {}
for name, fn, qt, blk in [("q4k", q4k, QT.Q4_K, 256), ("q6k", q6k, QT.Q6_K, 256), ("q80", q80, QT.Q8_0, 32)]:
    b = fn(48)
    out[f"{name}_blocks"] = b.reshape(-1)
    out[f"{name}_values"] = quants.dequantize(b.reshape(-1), qt).astype(np.float32).reshape(-1)
src = rng.standard_normal((16, 64)).astype(np.float32) * np.array([1e-3, 0.02, 1.0, 30.0] * 4, np.float32)[:, None]
src[3] = 0.0
out["q80_src"] = src.reshape(-1)
out["q80_quant"] = quants.quantize(src, QT.Q8_0).reshape(-1)
path = pathlib.Path(__file__).with_name("quant_golden.npz")
np.savez_compressed(path, **out)
print("wrote", path, {k: v.shape for k, v in out.items()})
