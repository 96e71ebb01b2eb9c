"""One DiT block on the CPU, composed of the oracle's pieces -- TEST INFRASTRUCTURE ONLY.

Restates the block of the reference DiT (tfimage/qwen_image21.py:204-216 ``_block``, :171-199 ``_attention``) with
the reference's CPU arithmetic for each op:

    a   = adaln(x, scale1) + shift1                                   kernels.py:14-37 (bf16)
    qkv = bf16(deq(quant(a, act_qkv)) @ deq(W_qkv)^T)                 linear.py:125-130, tools/gemm_tf.py:43-44
    q,k = rms_rope(qkv), v = qkv[:, :, 2]                             kernels.py:40-70
    o   = attention(q, [prefix; k], [prefix; v])                       torch SDPA in the reference (kept as is)
    x   = bf16(x + out(o) * gate1)                                    qwen_image21.py:213 (addcmul_)
    m   = adaln(x, scale2) + shift2
    x   = bf16(x + down(swiglu(gate_up(m))) * gate2)                  the unfused MLP chain, oracle.mlp

Attention is not part of the quantized-linear path: the reference calls torch SDPA (bf16, flash / cuDNN). ``block``
takes the attention op as an argument; ``attention`` below is a float64 softmax attention for use where no GPU
SDPA is at hand. The difference matters downstream: the out projection re-quantizes the attention output to NVFP4,
and a ~2e-3 change of its input moves ~3 % of the per-16 E4M3 block scales by one step, i.e. ~1-2 % on that
branch, which the residual's bf16 rounding and the MLP's two quantizers carry on.
"""

from __future__ import annotations

import numpy as np

from . import fusions, mlp, nvfp4


def attention(q, k, v, causal: bool = False) -> np.ndarray:
    """q [B, N, H, D], k / v [B, P + N, H, D] (values of bf16) -> bf16 [B, N, H, D]; float64 softmax attention.
    With ``causal`` query i sees keys 0..P+i."""
    q = np.asarray(q, dtype=np.float64).transpose(0, 2, 1, 3)
    k = np.asarray(k, dtype=np.float64).transpose(0, 2, 1, 3)
    v = np.asarray(v, dtype=np.float64).transpose(0, 2, 1, 3)
    N, S, D = q.shape[2], k.shape[2], q.shape[3]
    s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(D)
    if causal:
        allow = np.arange(S)[None, :] <= (S - N + np.arange(N))[:, None]
        s = np.where(allow[None, None], s, -np.inf)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = (p @ v).transpose(0, 2, 1, 3)
    return nvfp4.bf16_round(o.astype(np.float32))


def block(x, mod, cos, sin, k_prefix, v_prefix, lin: dict, norm_q, norm_k, heads: int, eps: float,
          causal: bool = False, return_parts: bool = False, attn=attention, acc: str = "f32"):
    """x [B, N, dim] (bf16 values); mod = (shift1, scale1, gate1, shift2, scale2, gate2) each [B, dim];
    k_prefix / v_prefix [B, P, H, D] (P may be 0); lin[name] = (codes [n, k/2], row scales [n, k/16] (e4m3 bytes),
    weight global, input scale) for name in qkv, out, gate_up, down; ``attn(q, k, v, causal)`` -> bf16 values.
    Returns the block output (and, with ``return_parts``, its intermediates). ``acc``: the GEMMs' summation
    ("f32" = the reference's fp32 matmul; "f64" = the exact sums, to measure how far another valid summation order
    moves the block output)."""
    sh1, sc1, g1, sh2, sc2, g2 = [np.asarray(m, dtype=np.float32).reshape(x.shape[0], 1, -1) for m in mod]
    x = np.asarray(x, dtype=np.float32)
    B, N, Dm = x.shape
    a = fusions.adaln(x, sc1, eps, shift=sh1)
    wc, ws, wg, act = lin["qkv"]
    qkv = nvfp4.linear(a.reshape(B * N, Dm), wc, ws, wg, act, acc)
    Dh = qkv.shape[1] // (3 * heads)
    src = qkv.reshape(B, N, 3, heads, Dh)
    q = fusions.rms_rope(src, 0, norm_q, cos, sin, eps)
    k = fusions.rms_rope(src, 1, norm_k, cos, sin, eps)
    v = src[:, :, 2]
    kk = np.concatenate([np.asarray(k_prefix, dtype=np.float32), k], axis=1)
    vv = np.concatenate([np.asarray(v_prefix, dtype=np.float32), v], axis=1)
    o = attn(q, kk, vv, causal)
    wc, ws, wg, act = lin["out"]
    att = nvfp4.linear(o.reshape(B * N, heads * Dh), wc, ws, wg, act, acc).reshape(B, N, Dm)
    x = nvfp4.bf16_round(x + att * g1)
    m = fusions.adaln(x, sc2, eps, shift=sh2)
    gc, gs, gg, gact = lin["gate_up"]
    dc, ds, dg, dact = lin["down"]
    y = mlp.forward(m.reshape(B * N, Dm), gc, gs, gg, dc, ds, dg, gact, dact, acc=acc).reshape(B, N, Dm)
    out = nvfp4.bf16_round(x + y * g2)
    if return_parts:
        return out, dict(a=a, qkv=qkv.reshape(B, N, -1), q=q, k=k, v=v, o=o, att=att, x1=x, m=m, mlp=y)
    return out
