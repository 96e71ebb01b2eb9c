"""GGUF diffusion checkpoints -> torch tensors, the quantized blocks decoded by one CUDA kernel per tensor.

Same interface as the reference's tfimage/gguf_load.py (``QK_K``, ``DECODERS``, ``dequantize``, ``tensors``) and
the same types: BF16 / F16 / F32 pass through a cast; Q8_0, Q6_K, Q5_K, Q4_K are decoded by ``tfb_gguf_dequant``
(csrc/gguf.cu), which reads each raw block once and writes each value once in the requested type, with the
reference's fp32 arithmetic (bit-equal to gguf_load.py:17-86 and to gguf-py's decoders). Anything else is refused
by name, as in the reference. Decoding needs a CUDA device: there is no CPU path.
"""

from __future__ import annotations

from pathlib import Path
from typing import Iterator

import numpy as np
import torch

from . import _lib

QK_K = 256
PASSTHROUGH = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


def _decoder(kind: str):
    def decode(raw: torch.Tensor) -> torch.Tensor:
        """Raw uint8 blocks on a CUDA device -> fp32 values, one row per block (gguf_load.py:21-71)."""
        vals, nbytes = _lib.gguf_block(kind)
        out = torch.empty((raw.numel() // nbytes, vals), dtype=torch.float32, device=raw.device)
        _lib.gguf_dequant(kind, raw.reshape(-1), out)
        return out
    decode.__name__ = f"_{kind.lower()}"
    return decode


DECODERS = {kind: _decoder(kind) for kind in ("Q8_0", "Q6_K", "Q5_K", "Q4_K")}


def dequantize(kind: str, data: np.ndarray, shape: tuple[int, ...], device="cuda",
               dtype=torch.bfloat16) -> torch.Tensor:
    """One GGUF tensor's bytes -> a ``shape`` tensor (torch order: the reverse of GGUF's) on ``device``
    (gguf_load.py:74-86). Quantized types are decoded straight into ``dtype`` when it is f32 / f16 / bf16."""
    raw = torch.from_numpy(np.ascontiguousarray(data).view(np.uint8).reshape(-1)).to(device, non_blocking=True)
    if kind in PASSTHROUGH:
        return raw.view(PASSTHROUGH[kind]).view(shape).to(dtype)
    if kind not in DECODERS:
        raise ValueError(f"GGUF tensor type {kind} is not decoded by tfimage (decoded: BF16, F16, F32, "
                         f"{', '.join(DECODERS)})")
    if raw.device.type != "cuda":
        raise _lib.TfbError("GGUF blocks are decoded by the CUDA kernel only (there is no CPU path)")
    direct = dtype in _lib.OUT_DTYPES
    out = torch.empty(shape, dtype=dtype if direct else torch.float32, device=raw.device)
    _lib.gguf_dequant(kind, raw, out)
    return out if direct else out.to(dtype)


def tensors(path: str | Path, device="cuda", dtype=torch.bfloat16) -> Iterator[tuple[str, torch.Tensor]]:
    """(name, tensor) for every tensor of a GGUF file, dequantized one at a time on ``device`` (gguf_load.py:89-97)."""
    from gguf import GGUFReader

    reader = GGUFReader(str(path))
    for t in reader.tensors:
        shape = tuple(int(v) for v in reversed(t.shape.tolist()))
        yield t.name, dequantize(t.tensor_type.name, t.data, shape, device, dtype)
