"""Fused elementwise kernels against the oracle (fp32 math: within one bf16 ulp; NVFP4 codes bit-exact)."""

import numpy as np
import pytest
import torch
from _helpers import bf16_cpu, f32, u8, ulp_bf16

from oracle import fusions as ofu
from oracle import nvfp4 as onv
from tfimage import kernels as K

pytestmark = pytest.mark.gpu
GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def within_ulp(y, ref, n=1, atol=1e-7):
    return (np.abs(y - ref) <= n * ulp_bf16(ref) + atol).all()


@pytest.mark.parametrize("B,N,D", [(2, 37, 256), (1, 4352, 3072), (2, 300, 4096), (2, 64, 512), (3, 50, 768),
                                   (1, 129, 1536), (1, 40, 8192)])
def test_adaln_matches_oracle(dev, B, N, D):
    x = bf16_cpu((B, N, D), seed=N, scale=3)
    g = torch.Generator().manual_seed(D)
    s = torch.randn(B, 1, D, generator=g) * 0.1
    sh = torch.randn(B, 1, D, generator=g) * 0.1
    y = K.adaln(x.to(dev), s.to(dev), 1e-6)
    assert within_ulp(f32(y), ofu.adaln(x.float().numpy(), s.numpy(), 1e-6))
    y2 = K.adaln(x.to(dev), s.to(dev), 1e-6, shift=sh.to(dev))
    assert within_ulp(f32(y2), ofu.adaln(x.float().numpy(), s.numpy(), 1e-6, shift=sh.numpy()))


def test_adaln_reference_fixture(dev):
    z = np.load(GOLD / "fusions.npz")
    for tag in ("a", "b"):
        x = torch.from_numpy(z[f"adaln_{tag}_x"].view(np.int16)).view(torch.bfloat16)
        y = K.adaln(x.to(dev), torch.from_numpy(z[f"adaln_{tag}_s"]).to(dev), 1e-6)
        ref = onv.bf16_from_bits(z[f"adaln_{tag}_y"])      # round-toward-zero fixture: one ulp of slack
        assert within_ulp(f32(y), ref)


@pytest.mark.parametrize("B,N,D", [(1, 4352 - 5, 3072), (1, 300, 768), (3, 45, 768), (40, 7, 256), (2, 1000, 8192)])
def test_adaln_fused_quant_bit_exact(dev, B, N, D):
    """AdaLN(+shift) then NVFP4 quantize, in one pass; codes/scales equal the oracle quantizer applied
    to the kernel's own bf16 result (and padded scale rows are zero), also with several batch elements (each with
    its own modulation; row ranges that do not divide evenly) and the widest D."""
    x = bf16_cpu((B, N, D), seed=61)
    g = torch.Generator().manual_seed(62)
    s, sh = torch.randn(B, 1, D, generator=g) * 0.1, torch.randn(B, 1, D, generator=g) * 0.1
    out = torch.empty((B, N, D), dtype=torch.bfloat16, device=dev)
    act = 0.004
    q = K.adaln(x.to(dev), s.to(dev), 1e-6, out=out, shift=sh.to(dev), quant=act)
    yb = f32(out).reshape(B * N, D)
    assert within_ulp(yb, ofu.adaln(x.float().numpy(), s.numpy(), 1e-6, shift=sh.numpy()).reshape(B * N, D))
    rc, rs = onv.quantize(yb, act)
    np.testing.assert_array_equal(u8(q.codes), rc)
    np.testing.assert_array_equal(u8(q.sf), onv.sf_tile(rs))


def rope_inputs(N_img_hw=(64, 64), n_txt=256):
    ids = np.concatenate([ofu.text_ids(n_txt), ofu.image_ids(*N_img_hw, n_txt, N_img_hw)])
    return ofu.rope_table(ids)


@pytest.mark.parametrize("B,N,H", [(2, 9, 4), (1, 4352, 24)])
def test_rms_rope_q_and_k_into_slice(dev, B, N, H):
    """per-head RMSNorm on Q/K [4352, 24, 128] + 3-axis RoPE (16/56/56) over a 64x64 grid + 256 text
    positions; k written behind P prefix rows of a larger buffer, prefix untouched (tools/check_kernels.py:15-17)."""
    D, P = 128, 7
    qkv = bf16_cpu((B, N, 3, H, D), seed=N + H)
    g = torch.Generator().manual_seed(71)
    w = torch.randn(D, generator=g) * 0.05 + 1
    cos, sin = rope_inputs() if N == 4352 else ofu.rope_table(ofu.text_ids(N))
    qkvd = qkv.to(dev)
    q = torch.empty((B, N, H, D), dtype=torch.bfloat16, device=dev)
    kbuf = torch.zeros((B, P + N, H, D), dtype=torch.bfloat16, device=dev)
    cs, sn = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    K.rms_rope(qkvd, 0, w.to(dev), cs, sn, 1e-6, q)
    K.rms_rope(qkvd, 1, w.to(dev), cs, sn, 1e-6, kbuf[:, P:])
    for part, got in ((0, f32(q)), (1, f32(kbuf[:, P:]))):
        ref = ofu.rms_rope(qkv.float().numpy(), part, w.numpy(), cos, sin, 1e-6)
        # fp32 rotation: outputs near zero come from cancelling O(1) terms, so allow 1 ulp plus 2^-20 absolute
        assert within_ulp(got, ref, atol=2.0 ** -20)
        assert (got == ref).mean() > 0.99
    assert float(kbuf[:, :P].abs().max()) == 0.0


def test_rms_rope_reference_fixture(dev):
    z = np.load(GOLD / "fusions.npz")
    qkv = torch.from_numpy(z["rr_qkv"].view(np.int16)).view(torch.bfloat16).to(dev)
    P = int(z["rr_prefix"])
    B, N, _, H, D = qkv.shape
    buf = torch.zeros((B, P + N, H, D), dtype=torch.bfloat16, device=dev)
    K.rms_rope(qkv, 1, torch.from_numpy(z["rr_w"]).to(dev), torch.from_numpy(z["rr_cos"]).to(dev),
               torch.from_numpy(z["rr_sin"]).to(dev), 1e-6, buf[:, P:])
    assert within_ulp(f32(buf), onv.bf16_from_bits(z["rr_kbuf"]))


@pytest.mark.parametrize("M,F", [(6, 160), (4352, 8192)])
def test_swiglu_matches_oracle(dev, M, F):
    """Bit-exact: silu is correctly rounded to bf16 on both sides (the fp32 fast path, with an fp64 recompute near
    a bf16 rounding midpoint and for large |g|)."""
    gu = bf16_cpu((M, 2 * F), seed=F, scale=2)
    g = gu[:, :F].reshape(-1)
    ramp = torch.linspace(-95.0, 40.0, min(g.numel(), 1 << 16)).to(torch.bfloat16)
    g[:ramp.numel()] = ramp                                   # the whole range, the fp32 overflow zone included
    gu[:, :F] = g.view(M, F)
    y = f32(K.swiglu(gu.to(dev)))
    ref = ofu.swiglu(gu.float().numpy())
    np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("B,N,H", [(1, 4352, 24), (2, 77, 3)])
def test_rms_rope_qkv_matches_per_part_kernel(dev, B, N, H):
    """tfb_rms_rope_qkv (q, k and the v copy in one pass) equals rms_rope per part bit for bit, writes k / v behind a
    kept prefix without touching it, and v is the exact copy."""
    D, P = 128, 5
    qkv = bf16_cpu((B, N, 3, H, D), seed=N + 3).to(dev)
    g = torch.Generator().manual_seed(72)
    wq, wk = (torch.randn(D, generator=g) * 0.05 + 1).to(dev), (torch.randn(D, generator=g) * 0.05 + 1).to(dev)
    cos, sin = ofu.rope_table(np.concatenate([ofu.text_ids(P), ofu.image_ids(1, N, P, (1, N))])[P:])
    cs, sn = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    q_ref = torch.empty((B, N, H, D), dtype=torch.bfloat16, device=dev)
    k_ref = torch.empty_like(q_ref)
    K.rms_rope(qkv, 0, wq, cs, sn, 1e-6, q_ref)
    K.rms_rope(qkv, 1, wk, cs, sn, 1e-6, k_ref)
    q = torch.empty_like(q_ref)
    kbuf = torch.full((B, P + N, H, D), 7.0, dtype=torch.bfloat16, device=dev)
    vbuf = torch.full_like(kbuf, -3.0)
    K.rms_rope_qkv(qkv, wq, wk, cs, sn, 1e-6, q, kbuf[:, P:], vbuf[:, P:])
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref) and torch.equal(kbuf[:, P:], k_ref)
    assert torch.equal(vbuf[:, P:], qkv[:, :, 2])
    assert bool((kbuf[:, :P] == 7.0).all()) and bool((vbuf[:, :P] == -3.0).all())


@pytest.mark.parametrize("B,N,H", [(1, 4096, 24), (2, 96, 24), (3, 64, 5)])
def test_qkv_gemm_with_rms_rope_epilogue_matches_two_steps(dev, B, N, H):
    """tfb_gemm_nvfp4_qkv (the qkv GEMM with q / k RMSNorm + RoPE and the v copy in its epilogue) equals the qkv GEMM
    followed by tfb_rms_rope_qkv bit for bit, writes k / v behind a kept prefix without touching it; odd head counts
    put q / k / v boundaries inside a 256-column tile."""
    from tfimage import linear as L

    D, P, Kd = 128, 64, 3072
    x = bf16_cpu((B * N, Kd), seed=B * N + H).to(dev)
    g = torch.Generator().manual_seed(73)
    lin = L.Nvfp4Linear((torch.randn(3 * H * D, Kd, generator=g) * 0.02).to(torch.bfloat16).to(dev),
                        act=float(x.float().abs().max()) / 2688)
    wq, wk = (torch.randn(D, generator=g) * 0.05 + 1).to(dev), (torch.randn(D, generator=g) * 0.05 + 1).to(dev)
    cos, sin = ofu.rope_table(np.concatenate([ofu.text_ids(P), ofu.image_ids(1, N, P, (1, N))])[P:])
    cs, sn = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    qkv = lin(x).view(B, N, 3, H, D)
    q_ref = torch.empty((B, N, H, D), dtype=torch.bfloat16, device=dev)
    kb_ref = torch.full((B, P + N, H, D), 7.0, dtype=torch.bfloat16, device=dev)
    vb_ref = torch.full_like(kb_ref, -3.0)
    K.rms_rope_qkv(qkv, wq, wk, cs, sn, 1e-6, q_ref, kb_ref[:, P:], vb_ref[:, P:])
    q = torch.empty_like(q_ref)
    kbuf = torch.full_like(kb_ref, 7.0)
    vbuf = torch.full_like(kb_ref, -3.0)
    assert K.qkv_rms_rope(lin, x.view(B, N, Kd), wq, wk, cs, sn, 1e-6, q, kbuf[:, P:], vbuf[:, P:])
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref)
    assert torch.equal(kbuf, kb_ref) and torch.equal(vbuf, vb_ref)
