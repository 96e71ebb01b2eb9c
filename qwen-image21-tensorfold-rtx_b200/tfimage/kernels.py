"""Fused elementwise kernels for a DiT block on B200 (libtfb CUDA kernels): each reads its input once and writes
its output once. Drop-in for the reference ``tfimage/kernels.py`` (same functions and arguments; new arguments are
optional and default to the reference behaviour). fp32 inside, bf16 out.
"""

from __future__ import annotations

import torch

from . import _lib


def adaln(x: torch.Tensor, scale: torch.Tensor, eps: float, out: torch.Tensor | None = None,
          shift: torch.Tensor | None = None, quant=None):
    """kernels.py:28-37: LayerNorm(x) * (1 + scale) (+ shift): x [B, N, D] bf16, scale/shift [B, 1, D] (any float)
    -> bf16 [B, N, D].

    ``quant``: an input scale (float) or an ``Nvfp4Linear`` whose ``act`` to use; then the bf16-rounded result is
    also NVFP4-quantized in the same pass and an ``Nvfp4Act`` is returned (with ``.out`` set to the bf16 tensor if
    ``out`` was given, else None), ready to feed that linear without a separate quantizer pass."""

    B, N, D = x.shape
    x = x.contiguous()
    s = scale.reshape(B, D).float().contiguous()
    sh = shift.reshape(B, D).float().contiguous() if shift is not None else None
    if quant is None:
        out = torch.empty_like(x) if out is None else out
        _lib.adaln(x, s, sh, eps, out=out)
        return out
    from .linear import Nvfp4Act, Nvfp4Linear

    act = quant.lin.act if isinstance(quant, Nvfp4Linear) else float(quant)
    M = B * N
    codes = torch.empty((M, D // 2), dtype=torch.uint8, device=x.device)
    sf = torch.empty((_lib.sf_tiled_bytes(M, D),), dtype=torch.uint8, device=x.device)
    _lib.adaln(x, s, sh, eps, out=out, q_global=act, codes=codes, sf=sf)
    q = Nvfp4Act(codes, sf, act, M, D)
    q.out = out
    return q


def rms_rope(src: torch.Tensor, part: int, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float,
             dst: torch.Tensor) -> None:
    """kernels.py:58-70: RMSNorm + RoPE of ``src``'s ``part`` (0 = q, 1 = k of a [B, N, 3, H, D] qkv) into ``dst``
    [B, N, H, D] (``dst`` may be a row slice of a larger [B, P + N, H, D] buffer: its strides are used as they are;
    rows outside it are not touched)."""

    if src.stride(-1) != 1 or src.stride(-2) != src.shape[-1] or src.stride(-3) != src.shape[-1] * src.shape[-2]:
        raise _lib.TfbError("rms_rope: src must be [B, N, 3, H, D] with contiguous (3, H, D) rows")
    if dst.stride(-1) != 1 or dst.stride(-2) != dst.shape[-1]:
        raise _lib.TfbError("rms_rope: dst rows must be contiguous [H, D]")
    _lib.rms_rope(src, part, w.float().contiguous(), cos.float().contiguous(), sin.float().contiguous(), eps, dst)


def rms_rope_qkv(src: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 eps: float, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """This build's addition: ``rms_rope(src, 0, wq, ...) -> q``, ``rms_rope(src, 1, wk, ...) -> k`` and
    ``v.copy_(src[:, :, 2])`` in one pass (the reference block's attention inputs, qwen_image21.py:180-191). q, k, v
    are [B, N, H, D] with contiguous [H, D] rows (k / v may be row slices of kept-prefix buffers)."""

    if src.stride(-1) != 1 or src.stride(-2) != src.shape[-1] or src.stride(-3) != src.shape[-1] * src.shape[-2]:
        raise _lib.TfbError("rms_rope_qkv: src must be [B, N, 3, H, D] with contiguous (3, H, D) rows")
    for t in (q, k, v):
        if t.stride(-1) != 1 or t.stride(-2) != t.shape[-1]:
            raise _lib.TfbError("rms_rope_qkv: destinations need contiguous [H, D] rows")
    f = lambda t: t.float().contiguous()   # noqa: E731
    _lib.rms_rope_qkv(src, f(wq), f(wk), f(cos), f(sin), eps, q, k, v)


def qkv_rms_rope(qkv_linear, x, wq: torch.Tensor, wk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float,
                 q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """This build's addition: ``rms_rope_qkv(qkv_linear(x).view(B, N, 3, H, D), ...)`` with the normalisation,
    rotation and v copy in the qkv GEMM's epilogue (no qkv tensor in HBM), bit-equal to the two-step form. x: the
    [B, N, dim] bf16 rows or their ``Nvfp4Act`` (e.g. from ``adaln(quant=)``); q, k, v as in ``rms_rope_qkv``.
    False (nothing done) when the layer is not a static-scale NVFP4 linear, D != 128 or N % 32 != 0."""
    from .linear import Nvfp4Act, Nvfp4Linear

    B, N, H, D = q.shape
    if not isinstance(qkv_linear, Nvfp4Linear) or qkv_linear.dynamic or D != 128 or N % 32:
        return False
    for t in (q, k, v):
        if t.stride(-1) != 1 or t.stride(-2) != D or tuple(t.shape) != (B, N, H, D):
            raise _lib.TfbError("qkv_rms_rope: destinations need contiguous [H, D] rows")
    lin = qkv_linear.lin
    if lin.n != 3 * H * D:
        raise _lib.TfbError(f"qkv_rms_rope: the layer has {lin.n} outputs, not 3 x {H} x {D}")
    a = x if isinstance(x, Nvfp4Act) else qkv_linear.quantize(x.reshape(B * N, -1))
    f = lambda t: t.float().contiguous()   # noqa: E731
    _lib.gemm_nvfp4_qkv(a.codes, a.sf, lin.codes, lin.bs, B, N, H, lin.k, a.act * lin.scale, f(wq), f(wk), f(cos),
                        f(sin), eps, q, k, v)
    return True


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """kernels.py:84-92: [M, 2F] = [gate | up] bf16 -> silu(gate) * up, [M, F] bf16."""

    M, F2 = gu.shape
    out = torch.empty((M, F2 // 2), dtype=torch.bfloat16, device=gu.device)
    _lib.swiglu(gu.contiguous(), out)
    return out
