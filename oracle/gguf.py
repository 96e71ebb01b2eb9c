"""CPU restatement of the GGUF block decoders -- TEST INFRASTRUCTURE ONLY.

The reference decodes the GGUF quantized types that image checkpoints use (tfimage/gguf_load.py:17-73) with torch ops
on the GPU; the block formats themselves are ggml's (published in ggml's ``ggml-common.h`` / ``dequantize_row_*``;
gguf-py 0.19.0 ``gguf/quants.py`` restates them in numpy). This module restates the same decoders in numpy with the
reference's fp32 arithmetic, one IEEE rounding per operation in the reference's order:

    Q8_0  (34 B / 32 values)   y = f16(d) * int8(q)                                        gguf_load.py:21-23
    Q4_K  (144 B / 256 values) y = (f16(d) * sc[j]) * q4 - (f16(dmin) * m[j])               gguf_load.py:53-59
    Q5_K  (176 B / 256 values) y = (f16(d) * sc[j]) * (q4 | hbit << 4) - (f16(dmin) * m[j]) gguf_load.py:62-71
    Q6_K  (210 B / 256 values) y = (f16(d) * int8(sc[j])) * ((q4 | q2 << 4) - 32)           gguf_load.py:26-37

then ``dequantize`` rounds to the requested output type (``.to(dtype)``, gguf_load.py:84: round to nearest even).
``tests/test_oracle.py`` pins these against gguf-py's decoders and against ``tests/golden/gguf.npz`` (the
reference's own decoders run on CPU by ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np

from .nvfp4 import bf16_round

QK_K = 256
# type name -> (values per block, bytes per block, ggml type id)
TYPES = {"Q8_0": (32, 34, 8), "Q4_K": (256, 144, 12), "Q5_K": (256, 176, 13), "Q6_K": (256, 210, 14)}


def _f16(b: np.ndarray) -> np.ndarray:
    """[n, 2] little-endian bytes -> [n] fp32 values of the fp16 numbers."""
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32).reshape(-1)


def scale_min_k4(s12: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """12 packed bytes per block -> 8 six-bit scales and 8 six-bit mins (gguf_load.py:40-50, ggml get_scale_min_k4):
    entries 0-3 are the low 6 bits of bytes 0-3 / 4-7; entries 4-7 take their low 4 bits from bytes 8-11 (low /
    high nibble) and their top 2 bits from the top bits of bytes 0-3 / 4-7."""
    q = s12.astype(np.int32)
    sc = np.empty((q.shape[0], 8), dtype=np.int32)
    mn = np.empty_like(sc)
    sc[:, :4] = q[:, 0:4] & 63
    mn[:, :4] = q[:, 4:8] & 63
    sc[:, 4:] = (q[:, 8:12] & 15) | ((q[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc.astype(np.float32), mn.astype(np.float32)


def q8_0(raw: np.ndarray) -> np.ndarray:
    blk = raw.reshape(-1, 34)
    d = _f16(blk[:, :2])
    q = blk[:, 2:].view(np.int8).astype(np.float32)
    return (d[:, None] * q).reshape(-1)


def _nibbles(qs: np.ndarray) -> np.ndarray:
    """[n, 128] bytes as 4 runs of 32 -> [n, 8, 32] 4-bit values: run j's low nibbles, then its high nibbles."""
    r = qs.reshape(-1, 4, 32).astype(np.int32)
    return np.stack([r & 15, r >> 4], axis=2).reshape(-1, 8, 32)


def q4_k(raw: np.ndarray) -> np.ndarray:
    blk = raw.reshape(-1, 144)
    d, dmin = _f16(blk[:, 0:2]), _f16(blk[:, 2:4])
    sc, mn = scale_min_k4(blk[:, 4:16])
    q = _nibbles(blk[:, 16:144]).astype(np.float32)
    ds = (d[:, None] * sc)[:, :, None]
    dm = (dmin[:, None] * mn)[:, :, None]
    return (ds * q - dm).reshape(-1)


def q5_k(raw: np.ndarray) -> np.ndarray:
    blk = raw.reshape(-1, 176)
    d, dmin = _f16(blk[:, 0:2]), _f16(blk[:, 2:4])
    sc, mn = scale_min_k4(blk[:, 4:16])
    qh = blk[:, 16:48].astype(np.int32)                                  # bit j of qh[l] = 5th bit of sub-block j
    hi = np.stack([(qh >> j) & 1 for j in range(8)], axis=1)
    q = (_nibbles(blk[:, 48:176]) | (hi << 4)).astype(np.float32)
    ds = (d[:, None] * sc)[:, :, None]
    dm = (dmin[:, None] * mn)[:, :, None]
    return (ds * q - dm).reshape(-1)


def q6_k(raw: np.ndarray) -> np.ndarray:
    """Two 128-value halves; in half h, run r (0-3) of 32 values takes its low 4 bits from ql[h*64 + (r%2)*32 + l]
    (low nibble for r < 2, high for r >= 2), its top 2 bits from qh[h*32 + l] >> 2r, and scale h*8 + 2r + l//16."""
    blk = raw.reshape(-1, 210)
    ql = blk[:, 0:128].astype(np.int32).reshape(-1, 2, 2, 32)           # [n, half, ql run, l]
    qh = blk[:, 128:192].astype(np.int32).reshape(-1, 2, 32)
    sc = blk[:, 192:208].view(np.int8).astype(np.float32).reshape(-1, 2, 4, 2)
    d = _f16(blk[:, 208:210])
    lo = np.stack([ql[:, :, 0] & 15, ql[:, :, 1] & 15, ql[:, :, 0] >> 4, ql[:, :, 1] >> 4], axis=2)
    hi = np.stack([(qh >> (2 * r)) & 3 for r in range(4)], axis=2)
    q = ((lo | (hi << 4)) - 32).astype(np.float32)                       # [n, 2, 4, 32]
    s = np.repeat(sc, 16, axis=3)                                        # [n, 2, 4, 32]: scale of value l is l // 16
    return ((d[:, None, None, None] * s) * q).reshape(-1)


DECODERS = {"Q8_0": q8_0, "Q4_K": q4_k, "Q5_K": q5_k, "Q6_K": q6_k}


def dequantize(kind: str, raw, out: str = "f32") -> np.ndarray:
    """Raw block bytes of ``kind`` -> fp32 values, rounded to ``out`` ("f32", "bf16" or "f16"; returned as fp32)."""
    raw = np.ascontiguousarray(np.asarray(raw).view(np.uint8).reshape(-1))
    vals, nbytes, _ = TYPES[kind]
    if raw.size % nbytes:
        raise ValueError(f"{kind}: {raw.size} bytes is not a whole number of {nbytes}-byte blocks")
    y = DECODERS[kind](raw).astype(np.float32)
    if out == "bf16":
        return bf16_round(y)
    if out == "f16":
        return y.astype(np.float16).astype(np.float32)
    return y


def random_blocks(kind: str, n_blocks: int, seed: int) -> np.ndarray:
    """Seeded blocks with finite fp16 block scales (NaN payloads are not compared) and uniformly random other bytes."""
    rng = np.random.default_rng(seed)
    vals, nbytes, _ = TYPES[kind]
    raw = rng.integers(0, 256, size=(n_blocks, nbytes), dtype=np.uint8)

    def f16(n, lo, hi):
        return rng.uniform(lo, hi, size=n).astype(np.float16).view(np.uint8).reshape(n, 2)

    if kind == "Q8_0":
        raw[:, 0:2] = f16(n_blocks, -0.05, 0.05)
    elif kind in ("Q4_K", "Q5_K"):
        raw[:, 0:2] = f16(n_blocks, 0.0, 0.01)
        raw[:, 2:4] = f16(n_blocks, 0.0, 0.01)
    else:
        raw[:, 208:210] = f16(n_blocks, -0.01, 0.01)
    return raw.reshape(-1)
