"""CPU restatements of the fused elementwise ops and the RoPE table -- TEST INFRASTRUCTURE ONLY.

Each function follows the reference's arithmetic (fp32 inside, bf16 out) and cites the lines it restates. The
reference Triton kernels themselves were run in the build container under ``TRITON_INTERPRET=1`` to make
``tests/golden/fusions.npz``; ``tests/test_oracle.py`` checks these restatements against that file.
"""

from __future__ import annotations

import numpy as np

from .nvfp4 import bf16_round, bf16_round_f64, bf16_trunc

_ROUND = {"rne": bf16_round, "rz": bf16_trunc}
# float64 results to bf16: one correct rounding ("rne"), or via fp32 then toward zero ("rz": Triton's CPU
# interpreter computes in fp32 and truncates on a bf16 store)
_ROUND64 = {"rne": bf16_round_f64, "rz": lambda y: bf16_trunc(np.asarray(y).astype(np.float32))}

AXES = (16, 56, 56)
THETA = 10000.0


def adaln(x, scale, eps: float, shift=None, rounding: str = "rne") -> np.ndarray:
    """kernels.py:14-26: bf16((x - mean) * rsqrt(var + eps) * (1 + scale[b])) (+ shift[b], this build's superset).

    x [B, N, D]; scale / shift [B, D] (or [B, 1, D]). Statistics in float64 (the exact value the fp32 kernels
    approximate); the result is rounded to bf16 once (``rounding="rz"`` reproduces Triton's CPU interpreter, which
    rounds toward zero on a bf16 store; the GPU reference and this build round to nearest even)."""
    x = np.asarray(x, dtype=np.float64)
    B, N, D = x.shape
    s = np.asarray(scale, dtype=np.float32).astype(np.float64).reshape(B, 1, D)
    mean = x.mean(-1, keepdims=True)
    xc = x - mean
    var = (xc * xc).mean(-1, keepdims=True)
    y = xc / np.sqrt(var + eps) * (1.0 + s)
    if shift is not None:
        y = y + np.asarray(shift, dtype=np.float32).astype(np.float64).reshape(B, 1, D)
    return _ROUND64[rounding](y)


def rms_rope(src, part: int, w, cos, sin, eps: float, rounding: str = "rne") -> np.ndarray:
    """kernels.py:40-60: per (row, head) RMSNorm over D with weight, then RoPE on interleaved pairs (2i, 2i+1).

    src [B, N, 3, H, D] -> [B, N, H, D] (fp32 values of bf16)."""
    x = np.asarray(src, dtype=np.float64)[:, :, part]
    w = np.asarray(w, dtype=np.float32).astype(np.float64)
    rr = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    xn = x * rr * w
    x0, x1 = xn[..., 0::2], xn[..., 1::2]
    c = np.asarray(cos, dtype=np.float32).astype(np.float64)[None, :, None, :]
    s = np.asarray(sin, dtype=np.float32).astype(np.float64)[None, :, None, :]
    out = np.stack([c * x0 - s * x1, s * x0 + c * x1], -1).reshape(x.shape)
    return _ROUND64[rounding](out)


def silu_bf16(g, rounding: str = "rne") -> np.ndarray:
    """bf16(silu(g)) of bf16 values g (kernels.py:80 rounds silu to bf16 before the product).

    ``"rne"``: the correctly rounded bf16 of the exact silu (float64, one rounding) -- the value the standalone GPU
    SwiGLU kernel of this build produces bit for bit, and one the reference's fp32 formula with an approximate exp
    reaches within one bf16 ulp. ``"rz"``: the reference formula in fp32 (g / (1 + exp(-g))) truncated to bf16,
    which is what the reference Triton kernel computes under the CPU interpreter (the golden fixture)."""
    if rounding == "rz":
        g = np.asarray(g, dtype=np.float32)
        return bf16_trunc((g / (np.float32(1.0) + np.exp(-g))).astype(np.float32))
    g = np.asarray(g, dtype=np.float64)
    with np.errstate(over="ignore"):
        return bf16_round_f64(g / (1.0 + np.exp(-g)))


def swiglu(gu, rounding: str = "rne") -> np.ndarray:
    """kernels.py:73-81: bf16(bf16(silu(g)) * u) for [M, 2F] = [gate | up]."""
    gu = np.asarray(gu, dtype=np.float32)
    F = gu.shape[1] // 2
    return _ROUND[rounding]((silu_bf16(gu[:, :F], rounding) * gu[:, F:]).astype(np.float32))


def swiglu_pair(g, u) -> np.ndarray:
    return bf16_round((silu_bf16(g) * np.asarray(u, dtype=np.float32)).astype(np.float32))


def rope_table(ids, axes=AXES, theta: float = THETA) -> tuple[np.ndarray, np.ndarray]:
    """qwen_image21.py:63-72: ids [N, 3] -> cos, sin [N, sum(axes)/2]; frequencies in float64, results fp32."""
    ids = np.asarray(ids, dtype=np.float64)
    angles = []
    for axis, dim in enumerate(axes):
        scale = np.linspace(0, (dim - 2) / dim, dim // 2, dtype=np.float64)
        omega = 1.0 / (theta ** scale)
        angles.append(ids[:, axis][:, None] * omega[None])
    a = np.concatenate(angles, axis=1)
    return np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)


def image_ids(h: int, w: int, pos: int, target_hw) -> np.ndarray:
    """qwen_image21.py:164-169: (pos, centred row, centred column) per latent token, fp32 [h*w, 3]."""
    hh = np.arange(h, dtype=np.float32) - (h - h // 2) + 0.5 * (h % 2 - target_hw[0] % 2)
    ww = np.arange(w, dtype=np.float32) - (w - w // 2) + 0.5 * (w % 2 - target_hw[1] % 2)
    ids = np.stack([np.full((h, w), float(pos), dtype=np.float32), np.broadcast_to(hh[:, None], (h, w)),
                    np.broadcast_to(ww[None, :], (h, w))], -1)
    return ids.reshape(-1, 3).astype(np.float32)


def text_ids(n: int, start: int = 0) -> np.ndarray:
    """qwen_image21.py:232: sequential positions on all three axes."""
    return np.repeat(np.arange(start, start + n, dtype=np.float32)[:, None], 3, axis=1)
