"""Fused NVFP4 MLP pair as the reference's unfused composition -- TEST INFRASTRUCTURE ONLY.

``swiglu_mlp`` (tfimage/linear.py:136-150) runs TensorFold's ``mlp_prompt``; its epilogue rounding is not
available, so the oracle is the unfused reference chain the model falls back to (qwen_image21.py:204-208):
``down(swiglu(gate_up(x)))`` with NVFP4 linears, i.e.

    gate/up  = bf16(deq(quant(x, act_gu)) @ deq(W_gu)^T)                 (linear.py:125-130)
    h        = bf16(bf16(silu(gate)) * up)                                 (kernels.py:80)
    y        = bf16(deq(quant(h, act_down)) @ deq(W_down)^T)

The fused GPU epilogue computes exactly this from its own bf16 gate/up values, so given identical gate/up the
NVFP4 codes and scales of ``h`` are bit-exact; end to end the output is compared by relative L2.
"""

from __future__ import annotations

import numpy as np

from . import fusions, nvfp4


def gate_up(x, gu_codes, gu_sf, g_gu: float, act_x: float, acc: str = "f32") -> np.ndarray:
    return nvfp4.linear(x, gu_codes, gu_sf, g_gu, act_x, acc)


def hidden(gu_bf16) -> np.ndarray:
    return fusions.swiglu(gu_bf16)


def forward(x, gu_codes, gu_sf, g_gu, down_codes, down_sf, g_down, act_x, act_h, return_parts=False,
            acc: str = "f32"):
    gu = gate_up(x, gu_codes, gu_sf, g_gu, act_x, acc)
    h = hidden(gu)
    hc, hs = nvfp4.quantize(h, act_h)
    y = nvfp4.bf16_round(nvfp4.gemm(hc, hs, act_h, down_codes, down_sf, g_down, acc))
    if return_parts:
        return y, dict(gu=gu, h=h, h_codes=hc, h_sf=hs)
    return y
