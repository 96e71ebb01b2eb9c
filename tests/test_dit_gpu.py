"""The synthetic MMDiT (tfimage.mmdit) against the CPU block oracle (oracle/dit.py) at full model width (dim 3072,
24 x 128 heads, SwiGLU 8192) and reduced token counts (256 image tokens after a 64-token text prefix); the same
comparisons at the configs[4] token counts are in test_dit_full_gpu.py.

Stage-wise (the BASELINE bar, rel-L2 <= 2e-3 of the dequantize-then-fp32-matmul chain, quantized codes bit-exact):
every stage of the real block is compared with the oracle fed that stage's actual GPU input -- the quantizers
against the oracle quantizer on the same bf16 rows, each GEMM against the oracle GEMM on the same codes -- and the
block output against the output recomposed from those oracle stages.

End to end (oracle run from x alone): 2e-3, or twice the reference chain's own summation-order spread where that is
larger (the oracle block with fp32 GEMM sums against the same block with exact sums, measured per case; the
distance to the exact-sum oracle is printed, and the 2e-3 bar against it is asserted at the configs[4] token counts,
in test_dit_full_gpu.py): chained NVFP4 requantization turns last-bit differences into code and block-scale
changes, so two correct implementations differ by about that spread. The float64-attention variant is printed for
information only (the reference's attention op is torch SDPA)."""

import numpy as np
import pytest
import torch
from _dit import end_to_end, gpu_block, image_case, sdpa_gpu, stagewise, summation_spread, text_case
from _helpers import f32, rel_l2

from oracle import dit as odit
from tfimage import mmdit

pytestmark = pytest.mark.gpu
TOL = 2e-3
# End to end the GPU block is compared with the fp32-sum oracle; two valid implementations of the chain differ by
# about the oracle's own fp32-vs-exact-sum spread, and the GPU block differs from the oracle in more places than the
# summation order (fp32 operation orders of AdaLN and RMS-RoPE, within one bf16 ulp; the SwiGLU epilogue's
# approximate silu): it may sit up to twice that spread away (measured: 1.0-1.6x).
SPREAD_BAND = 2.0


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    cfg = mmdit.DitConfig(layers=1)
    m = mmdit.SynthMMDiT(cfg, device="cuda", seed=5)
    g = torch.Generator().manual_seed(6)
    ctx = torch.randn((1, 64, cfg.txt_dim), generator=g).cuda()
    noise = torch.randn((1, 64, 16, 16), generator=g).cuda()
    m.calibrate(ctx, noise, steps=2)
    return m, ctx


@pytest.mark.parametrize("stream", ["image", "text"])
def test_block_stagewise(model, dev, stream):
    m, ctx = model
    if stream == "image":
        case, b, causal = image_case(m, ctx, dev), m.img_blocks[0], False
    else:
        case, b, causal = text_case(m, dev), m.txt_blocks[0], True
    r = stagewise(m, b, case, causal)
    for key in ("a_adaln", "m_adaln", "q", "k", "v", "residual1"):
        assert r[key] <= 1e-4, (key, r[key])                   # bf16-rounding-level ops
    for key in ("qkv", "out", "mlp", "block"):
        assert r[key] <= TOL, (key, r[key])
    assert r["attn_sdpa_vs_f64"] <= 5e-3                              # torch SDPA's own bf16 accuracy (not this path)


def test_image_block_end_to_end(model, dev):
    m, ctx = model
    case = image_case(m, ctx, dev)
    e_sdpa = end_to_end(m, m.img_blocks[0], case, False, sdpa_gpu)
    e_f64 = end_to_end(m, m.img_blocks[0], case, False, odit.attention)
    spread, exact = summation_spread(m, m.img_blocks[0], f32(case[0]), case, False, sdpa_gpu)
    y, _, _ = gpu_block(m, m.img_blocks[0], *case, False)
    e_exact = rel_l2(f32(y), exact)
    print(f"end to end: sdpa {e_sdpa:.2e} (exact-sum oracle {e_exact:.2e}; oracle fp32 vs exact sums {spread:.2e}), "
          f"float64 attention {e_f64:.2e}")
    assert e_sdpa <= max(TOL, SPREAD_BAND * spread)


def test_text_block_end_to_end(model, dev):
    m, _ = model
    case = text_case(m, dev)
    e = end_to_end(m, m.txt_blocks[0], case, True, sdpa_gpu)
    spread, exact = summation_spread(m, m.txt_blocks[0], f32(case[0]), case, True, sdpa_gpu)
    y, _, _ = gpu_block(m, m.txt_blocks[0], *case, True)
    e_exact = rel_l2(f32(y), exact)
    print(f"end to end (causal text block): {e:.2e} (exact-sum oracle {e_exact:.2e}; oracle fp32 vs exact sums "
          f"{spread:.2e})")
    assert e <= max(TOL, SPREAD_BAND * spread)


def test_sampler_runs_static_path(model, dev):
    m, ctx = model
    prefix = m.build_prefix(ctx)
    noise = torch.randn((2, 64, 16, 16), generator=torch.Generator().manual_seed(9)).to(dev)
    x = m.sample(noise, prefix, steps=3)
    assert x.shape == noise.shape and torch.isfinite(x).all()
    # two seeds in one batch give the same latents as each seed alone (rows never mix across the batch)
    x0 = m.sample(noise[:1], prefix, steps=3)
    assert rel_l2(f32(x[:1]), f32(x0)) <= 1e-3


def test_fused_residual_block_matches_unfused(model, dev):
    """The block with both gated residuals in GEMM epilogues equals the block with torch addcmul_ (record mode)."""
    m, ctx = model
    x, mod, cos, sin, kp, vp = image_case(m, ctx, dev)
    fused, _, _ = gpu_block(m, m.img_blocks[0], x, mod, cos, sin, kp, vp, False)
    unfused, _, _ = gpu_block(m, m.img_blocks[0], x, mod, cos, sin, kp, vp, False, record={})
    a, b = f32(fused), f32(unfused)
    print(f"fused vs unfused residual: identical {np.mean(a == b):.6f}, rel-L2 {rel_l2(a, b):.2e}")
    assert rel_l2(a, b) <= 1e-4


def test_graph_step_matches_eager(model, dev):
    """A replayed CUDA graph of the forward gives the eager forward's output bit for bit, for new inputs too."""
    m, ctx = model
    prefix = m.build_prefix(ctx)
    g = torch.Generator().manual_seed(12)
    for seed_t in (0.9, 0.3):
        x = torch.randn((1, 64, 16, 16), generator=g).to(torch.bfloat16).to(dev)
        t = torch.full((1,), seed_t, device=dev)
        eager = m.forward(x, t, prefix, {})
        replay = m.step_graph(x, t, prefix)
        torch.cuda.synchronize()
        assert torch.equal(eager, replay)
    noise = torch.randn((1, 64, 16, 16), generator=g).to(dev)
    assert torch.equal(m.sample(noise, prefix, steps=3), m.sample(noise, prefix, steps=3, graph=True))


def test_persistent_prefix_kv_matches_shared_buffer(model, dev):
    """Per-block key / value buffers (prefix rows written once) give the shared-buffer path's output bit for bit,
    eager and from a step graph, and pick up a prefix rebuilt in place (new prompt) before the next replay."""
    m, ctx = model
    prefix = m.build_prefix(ctx)
    g = torch.Generator().manual_seed(21)
    x = torch.randn((2, 64, 16, 16), generator=g).to(torch.bfloat16).to(dev)
    t = torch.tensor([0.8, 0.4], device=dev)
    per_block: dict = {}
    y1 = m.forward(x, t, prefix, per_block)
    assert per_block["kv"] is not None and len(per_block["kv"]) == m.cfg.layers
    m.kv_budget = 0
    try:
        shared: dict = {}
        y0 = m.forward(x, t, prefix, shared)
        assert shared["kv"] is None
    finally:
        m.kv_budget = None
    assert torch.equal(y0, y1)
    assert torch.equal(m.forward(x, t, prefix, per_block), y1)          # second step: no prefix copies
    yg = m.step_graph(x, t, prefix).clone()
    assert torch.equal(yg, y1)
    ctx2 = torch.randn(ctx.shape, generator=g).to(dev)
    m.build_prefix(ctx2, into=prefix)                                    # new prompt into the same buffers
    y2 = m.forward(x, t, prefix, per_block)
    assert not torch.equal(y2, y1)
    assert torch.equal(y2, m.forward(x, t, m.build_prefix(ctx2), {}))
    assert torch.equal(m.step_graph(x, t, prefix), y2)
