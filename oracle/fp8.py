"""FP8 E4M3 W8A8 CPU restatement of ``Fp8Linear`` (tfimage/linear.py:70-102) -- TEST INFRASTRUCTURE ONLY.

Pinned: ``tests/golden/make_golden.py`` runs the reference ``Fp8Linear`` on CPU and records its ``w8``/``ws`` and the
quantized activations it hands to ``torch._scaled_mm``; ``tests/test_oracle.py`` checks these functions against
them bit for bit. The per-output-channel weight scale is this build's superset; with a
broadcast scalar it reduces to the reference.
"""

from __future__ import annotations

import numpy as np

from .nvfp4 import E4M3_MAX, bf16_round, e4m3_decode, e4m3_encode


def weight(w, per_channel: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """linear.py:76-80: s = max(amax(W) / 448, 1e-12); w8 = e4m3(W / s). Per channel: one s per output row."""
    w = np.asarray(w, dtype=np.float32)
    if per_channel:
        s = np.maximum(np.abs(w).max(axis=1) / np.float32(E4M3_MAX), np.float32(1e-12)).astype(np.float32)
        q = (w / s[:, None]).astype(np.float32)
    else:
        s = np.maximum(np.abs(w).max() / np.float32(E4M3_MAX), np.float32(1e-12)).astype(np.float32)
        q = (w / s).astype(np.float32)
    return e4m3_encode(q), np.asarray(s, dtype=np.float32)


def act_scale(x) -> np.float32:
    """linear.py:86: (amax(x).float() / 448).clamp_min(1e-12), fp32."""
    a = np.float32(np.abs(np.asarray(x, dtype=np.float32)).max()) / np.float32(E4M3_MAX)
    return np.float32(max(a, np.float32(1e-12)))


def quantize(x, a) -> np.ndarray:
    """linear.py:95: e4m3((x.float() / a).clamp(-448, 448))."""
    v = (np.asarray(x, dtype=np.float32) / np.float32(a)).astype(np.float32)
    return e4m3_encode(np.clip(v, -E4M3_MAX, E4M3_MAX))


def gemm(xq, a, w8, ws) -> np.ndarray:
    """_scaled_mm(xq, w8.t(), scale_a=a, scale_b=ws) -> bf16 (returned as fp32 values). ws: scalar or [N]."""
    acc = e4m3_decode(xq).astype(np.float64) @ e4m3_decode(w8).astype(np.float64).T
    ws = np.asarray(ws, dtype=np.float64)
    return bf16_round((acc * np.float64(a) * (ws[None, :] if ws.ndim else ws)).astype(np.float32))


def linear(x, w8, ws, act=None) -> np.ndarray:
    a = act_scale(x) if act is None else np.float32(act)
    return gemm(quantize(x, a), a, w8, ws)
