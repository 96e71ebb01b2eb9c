"""configs[4] sizes: blocks of the synthetic MMDiT at full width (dim 3072, 24 x 128 heads, SwiGLU 8192) and full
token counts -- an image block on 4096 image rows (a 64 x 64 latent grid) attending to the 256-row kept prompt
prefix, and a text block on the 256-row prompt (causal) -- against the CPU block oracle (oracle/dit.py), and a
4-block stretch of the step.

* stage-wise: every stage against the oracle fed that stage's GPU input (quantized codes and
  scales bit-exact, GEMM and block outputs within rel-L2 2e-3 of the dequantize-then-fp32-matmul chain);
* end to end: the oracle block run from x alone, with the rel-L2 of every intermediate printed (attribution);
* step: x through 4 image blocks, each GPU block output against the oracle block fed the same (GPU) input, and
  against the oracle chain run from the first block's input alone.

End to end the 2e-3 bar applies against the reference arithmetic with exact GEMM sums; against the reference's fp32
sums the bound is 2e-3 or twice their own spread around the exact sums, whichever is larger. The spread is measured
per case: the oracle block with its fp32 GEMM sums (the reference's dequantize-then-fp32-matmul) against the same
block with exact float64 sums. Every NVFP4 requantization turns a last-bit difference of its input into a code or
block-scale change of a few percent of that element, and the block chains five of them (qkv input, out input, MLP
input, hidden, and the attention's bf16 output feeding the out projection), so the end-to-end rel-L2 between two
correct implementations sits at the spread, about 2-3e-3 per block, however the sums are ordered."""

import pytest
import torch
from _dit import end_to_end, gpu_block, image_case, oracle_block, sdpa_gpu, stagewise, summation_spread, text_case
from _helpers import f32, rel_l2

from tfimage import mmdit

pytestmark = pytest.mark.gpu
TOL = 2e-3
# the GPU block differs from the fp32-sum oracle in more places than the summation order (fp32 operation orders of
# AdaLN and RMS-RoPE, within one bf16 ulp; the SwiGLU epilogue's approximate silu): up to twice that spread
SPREAD_BAND = 2.0


@pytest.fixture(scope="module")
def full():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    cfg = mmdit.DitConfig(layers=4)
    m = mmdit.SynthMMDiT(cfg, device="cuda", seed=25)
    g = torch.Generator().manual_seed(26)
    ctx = torch.randn((1, 256, cfg.txt_dim), generator=g).cuda()
    noise = torch.randn((1, 64, 64, 64), generator=g).cuda()
    m.calibrate(ctx, noise, steps=2)
    return m, ctx, m.build_prefix(ctx)


def _case(m, ctx, prefix, dev, stream):
    if stream == "image":
        return image_case(m, ctx, dev, hw=64, seed=27, prefix=prefix), m.img_blocks[0], False
    return text_case(m, dev, n=256, seed=28), m.txt_blocks[0], True


@pytest.mark.parametrize("stream", ["image", "text"])
def test_full_size_block_stagewise(full, dev, stream):
    m, ctx, prefix = full
    case, b, causal = _case(m, ctx, prefix, dev, stream)
    r = stagewise(m, b, case, causal)
    for key in ("a_adaln", "m_adaln", "q", "k", "v", "residual1"):
        assert r[key] <= 1e-4, (key, r[key])                   # bf16-rounding-level ops
    for key in ("qkv", "out", "mlp", "block"):
        assert r[key] <= TOL, (key, r[key])


@pytest.mark.parametrize("stream", ["image", "text"])
def test_full_size_block_end_to_end(full, dev, stream):
    m, ctx, prefix = full
    case, b, causal = _case(m, ctx, prefix, dev, stream)
    e, parts = end_to_end(m, b, case, causal, sdpa_gpu, attribution=True)
    spread, exact = summation_spread(m, b, f32(case[0]), case, causal, sdpa_gpu)
    y, _, _ = gpu_block(m, b, *case, causal)
    e_exact = rel_l2(f32(y), exact)
    print(f"{stream} block end to end {e:.2e} (to the exact-sum oracle {e_exact:.2e}; oracle fp32 vs exact sums: "
          f"{spread:.2e}); per intermediate:", {k: f"{v:.2e}" for k, v in parts.items()})
    assert e_exact <= TOL                      # the reference arithmetic with exact sums: the 2e-3 bar
    assert e <= max(TOL, SPREAD_BAND * spread)  # the reference's own fp32 sums: their spread around the exact one


def test_full_size_four_block_step(full, dev):
    m, ctx, prefix = full
    x0, mod, cos, sin, _, _ = image_case(m, ctx, dev, hw=64, seed=29, prefix=prefix)
    gx, ox, ox64 = x0, f32(x0), f32(x0)
    forced, forced_exact, forced_spread, free, free_spread = [], [], [], [], []
    for i, b in enumerate(m.img_blocks):
        kpre, vpre = prefix.kv[i]
        case = (gx, mod, cos, sin, kpre, vpre)
        y, _, _ = gpu_block(m, b, gx, mod, cos, sin, kpre, vpre, False)
        r32 = oracle_block(m, b, f32(gx), case, False, sdpa_gpu)
        r64 = oracle_block(m, b, f32(gx), case, False, sdpa_gpu, acc="f64")
        forced.append(rel_l2(f32(y), r32))
        forced_exact.append(rel_l2(f32(y), r64))
        forced_spread.append(rel_l2(r64, r32))
        ox = oracle_block(m, b, ox, case, False, sdpa_gpu)
        ox64 = oracle_block(m, b, ox64, case, False, sdpa_gpu, acc="f64")
        free.append(rel_l2(f32(y), ox))
        free_spread.append(rel_l2(ox64, ox))
        gx = y
    print("per block, oracle fed the GPU input:", [f"{v:.2e}" for v in forced], "exact-sum oracle:",
          [f"{v:.2e}" for v in forced_exact], "its fp32 vs exact sums:", [f"{v:.2e}" for v in forced_spread])
    print("after each block, oracle chain from x0 alone:", [f"{v:.2e}" for v in free],
          "its fp32 vs exact sums:", [f"{v:.2e}" for v in free_spread])
    for f, fe, sp in zip(forced, forced_exact, forced_spread):
        assert fe <= TOL, fe
        assert f <= max(TOL, SPREAD_BAND * sp), (f, sp)
    assert free[-1] <= max(TOL, SPREAD_BAND * free_spread[-1]), (free[-1], free_spread[-1])
