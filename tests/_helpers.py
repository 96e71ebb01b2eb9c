"""Shared helpers for the GPU parity tests: seeded inputs (generated on the CPU, then moved), numpy views."""

import numpy as np
import torch

from oracle import nvfp4 as onv


def bf16_cpu(shape, seed, scale=1.0, outliers=0):
    """Seeded N(0, scale) bf16 tensor on the CPU; ``outliers`` channels (chosen by the seed) scaled x20."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers:
        idx = torch.randperm(shape[-1], generator=g)[:outliers]
        x[..., idx] *= 20
    return x.to(torch.bfloat16)


def f32(t: torch.Tensor) -> np.ndarray:
    """bf16/fp32 tensor (any device) -> fp32 numpy."""
    return t.detach().float().cpu().numpy()


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().view(torch.uint8).cpu().numpy()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ulp_bf16(v):
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


def quant_weight(w_cpu_bf16: torch.Tensor):
    """Oracle NVFP4 weight: (codes, row scales, g) from a CPU bf16 weight."""
    w = w_cpu_bf16.float().numpy()
    g = onv.weight_global(np.abs(w).max())
    c, s = onv.quantize(w, g)
    return c, s, g
