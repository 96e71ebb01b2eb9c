"""tcgen05 GEMMs against the oracle's dequantize-then-fp32-matmul (rel-L2 <= 2e-3 NVFP4, <= 1e-3 FP8)."""

import numpy as np
import pytest
import torch
from _helpers import bf16_cpu, f32, quant_weight, rel_l2, u8, ulp_bf16

from oracle import fp8 as ofp8
from oracle import fusions as ofu
from oracle import nvfp4 as onv
from tfimage import _lib
from tfimage import linear as L

pytestmark = pytest.mark.gpu
TOL_NVFP4 = 2e-3   # GEMM outputs within rel-L2 2e-3 of dequant -> fp32 matmul
TOL_FP8 = 1e-3


def nvfp4_case(dev, M, N, K, seed):
    x = bf16_cpu((M, K), seed=seed, outliers=8)
    w = bf16_cpu((N, K), seed=seed + 1, scale=0.02)
    wc, ws, gw = quant_weight(w)
    ga = onv.dynamic_act_global(float(x.float().abs().max()))
    xc, xs = onv.quantize(x.float().numpy(), ga)
    ref = onv.bf16_round(onv.gemm(xc, xs, ga, wc, ws, gw))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
    y = _lib.gemm_nvfp4(t(xc), t(onv.sf_tile(xs)), t(wc), t(onv.sf_tile(ws)), M, N, K, ga * gw)
    return f32(y), ref


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (1, 32, 128), (300, 320, 384), (1000, 1024, 640)])
def test_gemm_nvfp4_shapes(dev, M, N, K):
    y, ref = nvfp4_case(dev, M, N, K, seed=M + N + K)
    assert rel_l2(y, ref) <= TOL_NVFP4
    assert np.isfinite(y).all()


def test_gemm_nvfp4_config0(dev):
    """X [4096, 3072] (8 outlier channels x20) x W [3072, 3072] N(0, 0.02)."""
    y, ref = nvfp4_case(dev, 4096, 3072, 3072, seed=0)
    assert rel_l2(y, ref) <= TOL_NVFP4
    assert (y == ref).mean() > 0.9            # most outputs round to the same bf16


def test_gemm_nvfp4_repeatable(dev):
    y1, _ = nvfp4_case(dev, 512, 512, 512, seed=3)
    y2, _ = nvfp4_case(dev, 512, 512, 512, seed=3)
    np.testing.assert_array_equal(y1, y2)


@pytest.mark.parametrize("M,per_channel", [(4968, False), (4968, True), (77, True)])
def test_gemm_fp8_config3(dev, M, per_channel):
    """ragged M = 4712 + 256 = 4968, K = N = 3072; per-tensor act, tensor-wise or per-channel W."""
    K = N = 3072 if M > 100 else 256
    x = bf16_cpu((M, K), seed=M, outliers=8)
    w = bf16_cpu((N, K), seed=M + 1, scale=0.02)
    w8, ws = ofp8.weight(w.float().numpy(), per_channel)
    xd = x.to(dev)
    a = _lib.fp8_act_scale(xd)
    q = _lib.quant_fp8(xd, a)
    y = _lib.gemm_fp8(q, torch.from_numpy(w8).to(dev), M, N, K, a, torch.from_numpy(np.atleast_1d(ws)).to(dev))
    ref = ofp8.gemm(u8(q), float(a), w8, ws)
    assert rel_l2(f32(y), ref) <= TOL_FP8


def _fp8_case(dev, M, N, K, per_channel, seed):
    x = bf16_cpu((M, K), seed=seed, outliers=8 if K >= 64 else 0)
    w = bf16_cpu((N, K), seed=seed + 1, scale=0.02)
    w8, ws = ofp8.weight(w.float().numpy(), per_channel)
    xd = x.to(dev)
    a = _lib.fp8_act_scale(xd)
    q = _lib.quant_fp8(xd, a)
    y = _lib.gemm_fp8(q, torch.from_numpy(w8).to(dev), M, N, K, a, torch.from_numpy(np.atleast_1d(ws)).to(dev))
    np.testing.assert_array_equal(u8(q), ofp8.quantize(x.float().numpy(), float(a)))
    return f32(y), ofp8.gemm(u8(q), float(a), w8, ws)


@pytest.mark.parametrize("N,K", [(16384, 3072), (3072, 8192)])
def test_gemm_fp8_config3_mlp_shapes(dev, N, K):
    """configs[3] on the MLP shapes: gate/up [16384, 3072] and down [3072, 8192] at the ragged M = 4968."""
    y, ref = _fp8_case(dev, 4968, N, K, True, seed=N + K)
    assert rel_l2(y, ref) <= TOL_FP8
    assert np.isfinite(y).all()


@pytest.mark.parametrize("M,N,K", [(77, 48, 80), (300, 272, 1040), (129, 16, 16), (513, 400, 3088)])
def test_gemm_fp8_reference_envelope(dev, M, N, K):
    """Shapes with K % 128 != 0 or N % 32 != 0 that the reference's make() sends to FP8 (linear.py:159: K and N
    multiples of 16): the K tail and the last N rows come from TMA's zero fill."""
    for per_channel in (False, True):
        y, ref = _fp8_case(dev, M, N, K, per_channel, seed=M + N + K)
        assert rel_l2(y, ref) <= TOL_FP8, (per_channel, rel_l2(y, ref))


def test_make_dispatch_matches_reference_rule(dev):
    """make("nvfp4" | "fp8", w) returns the reference's backend for every shape (linear.py:153-161): NVFP4 for
    k % 128 == 0 and n % 64 == 0, else FP8 for k % 16 == 0 and n % 16 == 0, else bf16; each layer runs."""
    shapes = [(256, 256), (192, 384), (96, 256), (48, 80), (272, 1040), (16, 16), (40, 64), (64, 72), (3072, 3072)]
    for kind in ("nvfp4", "fp8"):
        for n, k in shapes:
            if kind == "nvfp4" and k % 128 == 0 and n % 64 == 0:
                want = "nvfp4"
            elif k % 16 == 0 and n % 16 == 0:
                want = "fp8"
            else:
                want = "bf16"
            w = bf16_cpu((n, k), seed=n * k, scale=0.02).to(dev)
            lin = L.make(kind, w)
            assert lin.kind == want, (kind, n, k, lin.kind)
            x = bf16_cpu((33, k), seed=n + k).to(dev)
            y = lin(x)
            ref = x.float() @ w.float().T
            assert y.shape == (33, n) and rel_l2(f32(y), f32(ref)) < 0.2


@pytest.mark.parametrize("M,K,F", [(300, 256, 256), (4352, 3072, 8192)])
def test_swiglu_epilogue_given_gate_up(dev, M, K, F):
    """The SwiGLU -> NVFP4 epilogue from the kernel's own bf16 gate/up, at a small shape and at configs[1]
    (4352 x 8192 = 35.7 M hidden values):
    * its NVFP4 quantizer is bit-exact: codes and tiled scales equal the oracle quantizer applied to its bf16 h;
    * its h = bf16(bf16(silu(g)) * u) uses the hardware exp2 / reciprocal approximations for silu, so h differs
      from the correctly rounded value (the oracle; the standalone SwiGLU kernel matches it bit for bit) only where
      the approximation lands within a few fp32 ulp of a bf16 rounding midpoint -- none of the 35.7 M values at
      configs[1] -- each by one bf16 ulp; differences of h and of the resulting NVFP4 codes and scales are counted.
    At the small shape gate/up also match the dequant matmul (at configs[1] the end-to-end MLP test covers that)."""
    x = bf16_cpu((M, K), seed=11 + M)
    w = bf16_cpu((2 * F, K), seed=12 + M, scale=0.05 if M < 1000 else 0.02)
    wc, ws, gw = quant_weight(w)
    ga = onv.dynamic_act_global(float(x.float().abs().max()))
    xc, xs = onv.quantize(x.float().numpy(), ga)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
    gu = torch.empty((M, 2 * F), dtype=torch.bfloat16, device=dev)
    hb = torch.empty((M, F), dtype=torch.bfloat16, device=dev)
    act_h = 0.002
    hc, hs = _lib.gemm_nvfp4_swiglu(t(xc), t(onv.sf_tile(xs)), t(wc), t(onv.sf_tile(ws)), M, F, K, ga * gw, act_h,
                                    gu_out=gu, h_out=hb)
    if M < 1000:
        gu_ref = onv.bf16_round(onv.gemm(xc, xs, ga, wc, ws, gw))
        assert rel_l2(f32(gu), gu_ref) <= TOL_NVFP4
    h = f32(hb)
    rc, rs = onv.quantize(h, act_h)                           # the quantizer, on the kernel's own h: bit-exact
    np.testing.assert_array_equal(u8(hc), rc)
    np.testing.assert_array_equal(u8(hs), onv.sf_tile(rs))
    h_exact = ofu.swiglu(f32(gu))                             # correctly rounded silu, given the same gate/up
    diff = h != h_exact
    assert (np.abs(h - h_exact) <= ulp_bf16(h_exact) * 1.0001 + 1e-30).all()
    ec, es = onv.quantize(h_exact, act_h)
    code_diff = np.mean(u8(hc) != ec)
    scale_diff = np.mean(rs != es)
    print(f"h values off the correctly rounded silu: {diff.sum()} of {h.size} ({diff.mean():.2e}); NVFP4 code bytes "
          f"differing {code_diff:.2e}, block scales differing {scale_diff:.2e}")
    assert diff.mean() <= 1e-5 and code_diff <= 1e-5 and scale_diff <= 1e-5   # measured: 0 of 35.7 M


def test_fused_mlp_config1(dev):
    """X [4352, 3072] N(0,1); W_gu [16384, 3072], W_down [3072, 8192] N(0, 0.02); down.act from the
    oracle's SwiGLU output with calibrate's 4x margin."""
    M, K, F = 4352, 3072, 8192
    x = bf16_cpu((M, K), seed=21)
    wgu = bf16_cpu((2 * F, K), seed=22, scale=0.02)
    wd = bf16_cpu((K, F), seed=23, scale=0.02)
    guc, gus, ggu = quant_weight(wgu)
    dc, ds, gd = quant_weight(wd)
    ax = onv.dynamic_act_global(float(x.float().abs().max()))
    gu_ref = onv.bf16_round(onv.gemm(*onv.quantize(x.float().numpy(), ax), ax, guc, gus, ggu))
    h_ref = ofu.swiglu(gu_ref)
    act_h = 4 * float(np.abs(h_ref).max()) / (6 * 448)
    y_ref = onv.bf16_round(onv.gemm(*onv.quantize(h_ref, act_h), act_h, dc, ds, gd))
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
    y = _lib.mlp_nvfp4(x.to(dev), F, ax, t(guc), t(onv.sf_tile(gus)), ggu, t(dc), t(onv.sf_tile(ds)), gd, act_h)
    assert rel_l2(f32(y), y_ref) <= TOL_NVFP4


# ----------------------------------------------------------------------------------------- API-level (linear.py)
def test_nvfp4_linear_dynamic_and_static(dev):
    M, N, K = 333, 384, 512
    w = bf16_cpu((N, K), seed=31, scale=0.02)
    x = bf16_cpu((M, K), seed=32, outliers=4)
    lin = L.Nvfp4Linear(w.to(dev))
    wc, ws, gw = quant_weight(w)
    np.testing.assert_array_equal(u8(lin.lin.codes), wc)          # nvfp4_weight through the GPU quantizer
    np.testing.assert_array_equal(u8(lin.lin.scales()), ws)
    assert lin.lin.scale == gw
    y = lin(x.to(dev))
    a = onv.dynamic_act_global(float(x.float().abs().max()))
    assert lin.amax == a and lin.lin.act == a
    assert rel_l2(f32(y), onv.linear(x.float().numpy(), wc, ws, gw, a)) <= TOL_NVFP4
    lin.set_act(0.02)
    y2 = lin(x.to(dev))
    assert rel_l2(f32(y2), onv.linear(x.float().numpy(), wc, ws, gw, 0.02)) <= TOL_NVFP4


def test_swiglu_mlp_api_and_fallback_contract(dev):
    M, K, F = 256, 256, 384
    gu = L.Nvfp4Linear(bf16_cpu((2 * F, K), seed=41, scale=0.05).to(dev))
    down = L.Nvfp4Linear(bf16_cpu((K, F), seed=42, scale=0.05).to(dev))
    x = bf16_cpu((M, K), seed=43).to(dev)
    assert L.swiglu_mlp(gu, down, x) is None                         # dynamic layers: caller falls back
    gu.set_act(0.004)
    down.set_act(0.001)
    y = L.swiglu_mlp(gu, down, x)
    from tfimage import kernels as K
    ref = down(K.swiglu(gu(x)))                                       # the unfused chain the model falls back to
    assert rel_l2(f32(y), f32(ref)) <= TOL_NVFP4


def test_fp8_linear_api(dev):
    """Fp8Linear end to end: the weight conversion (the reference's torch expressions with tensor divisors, exact on
    the GPU too) gives the oracle's w8 bytes and scales bit for bit; the activation quantizer and GEMM are checked
    against the oracle on the layer's own w8/ws."""
    w = bf16_cpu((256, 384), seed=51, scale=0.02)
    x = bf16_cpu((100, 384), seed=52)
    for act, pc in ((None, False), (0.05, False), (None, True)):
        lin = L.Fp8Linear(w.to(dev), act, per_channel=pc)
        w8_ref, ws_ref = ofp8.weight(w.float().numpy(), pc)
        np.testing.assert_array_equal(u8(lin.w8), w8_ref)
        np.testing.assert_array_equal(lin.ws.cpu().numpy(), ws_ref)
        y = lin(x.to(dev))
        ref = ofp8.linear(x.float().numpy(), u8(lin.w8), lin.ws.cpu().numpy(), act)
        assert rel_l2(f32(y), ref) <= TOL_FP8


def test_single_cta_kernels_for_large_m():
    """For M > 128 the GEMMs run on CTA pairs; TFB_CTA_GROUP=1 (read once per process) selects the single-CTA
    kernels instead. Re-run the shape, FP8 and SwiGLU-epilogue tests in a child process with it set."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    env = dict(os.environ, TFB_CTA_GROUP="1")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", str(here / "test_gemm_gpu.py"), "-q", "-m", "gpu", "-p", "no:cacheprovider",
         "-k", "gemm_nvfp4_shapes or gemm_fp8_config3 or swiglu_epilogue or fused_mlp"],
        cwd=here.parent, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout


@pytest.mark.parametrize("M,N,K,batches", [(300, 3072, 512, 3), (77, 256, 256, 1), (4096, 3072, 3072, 1)])
def test_gemm_nvfp4_gated_residual_epilogue(dev, M, N, K, batches):
    """tfb_gemm_nvfp4_resid: x += gate[b] * linear(a) inside the GEMM epilogue, against the unfused GEMM followed by
    torch's addcmul_ (the reference block, qwen_image21.py:213-215) and against the oracle."""
    x = bf16_cpu((M, K), seed=M + 5, outliers=4)
    w = bf16_cpu((N, K), seed=N + 6, scale=0.02)
    xc, xs = onv.quantize(x.float().numpy(), ga := onv.dynamic_act_global(float(x.float().abs().max())))
    wc, ws, gw = quant_weight(w)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
    res = bf16_cpu((M, N), seed=M + 7, scale=4.0).to(dev)
    rows = M // batches
    gate = (bf16_cpu((batches, N), seed=M + 8, scale=0.3)).to(dev)
    y = _lib.gemm_nvfp4(t(xc), t(onv.sf_tile(xs)), t(wc), t(onv.sf_tile(ws)), M, N, K, ga * gw)
    ref = res.clone().view(batches, rows, N).addcmul_(y.view(batches, rows, N), gate.view(batches, 1, N)).view(M, N)
    fused = res.clone()
    _lib.gemm_nvfp4_resid(t(xc), t(onv.sf_tile(xs)), t(wc), t(onv.sf_tile(ws)), M, N, K, ga * gw, fused, gate, rows)
    torch.cuda.synchronize()
    a, b = f32(fused), f32(ref)
    assert (a == b).mean() >= 0.9999
    assert np.all(np.abs(a - b) <= ulp_bf16(b) + 1e-30)
    y_or = onv.bf16_round(onv.gemm(xc, xs, ga, wc, ws, gw))
    g_rows = np.repeat(f32(gate), rows, axis=0)
    oracle = onv.bf16_round(f32(res) + y_or * g_rows)
    assert rel_l2(a - f32(res), oracle - f32(res)) <= TOL_NVFP4


def test_swiglu_mlp_gated_residual(dev):
    M, K, F = 256, 512, 384
    gu = L.Nvfp4Linear(bf16_cpu((2 * F, K), seed=61, scale=0.05).to(dev), act=0.004)
    down = L.Nvfp4Linear(bf16_cpu((K, F), seed=62, scale=0.05).to(dev), act=0.001)
    x = bf16_cpu((2, M // 2, K), seed=63).to(dev)
    res = bf16_cpu((2, M // 2, K), seed=64, scale=3.0).to(dev)
    gate = bf16_cpu((2, 1, K), seed=65, scale=0.5).to(dev)
    y = L.swiglu_mlp(gu, down, x.view(M, K))
    ref = res.clone().addcmul_(y.view(2, M // 2, K), gate)
    out = res.clone()
    assert L.swiglu_mlp(gu, down, x.view(M, K), residual=(out, gate)) is out
    assert (f32(out) == f32(ref)).mean() >= 0.9999


def test_swiglu_mlp_host_streams_rows_bit_identically(dev):
    """swiglu_mlp_host (pinned rows in chunks, copies overlapped) equals one swiglu_mlp call on the device."""
    M, K, F = 1000, 512, 384
    gu = L.Nvfp4Linear(bf16_cpu((2 * F, K), seed=91, scale=0.05).to(dev), act=0.003)
    down = L.Nvfp4Linear(bf16_cpu((K, F), seed=92, scale=0.05).to(dev), act=0.002)
    x = bf16_cpu((M, K), seed=93)
    ref = L.swiglu_mlp(gu, down, x.to(dev)).cpu()
    xp = x.pin_memory()
    for chunks, graph in ((1, False), (3, False), (8, False), (3, True), (8, True)):
        y = torch.full((M, K), float("nan"), dtype=torch.bfloat16).pin_memory()
        for _ in range(2 if graph else 1):       # graph: capture on the first call, replay on the second
            y.fill_(float("nan"))
            out = L.swiglu_mlp_host(gu, down, xp, y, chunks=chunks, graph=graph)
            torch.cuda.synchronize()
            assert out is y and torch.equal(y, ref), (chunks, graph)
    # a replay reads the host buffer's current contents
    x2 = bf16_cpu((M, K), seed=94)
    xp.copy_(x2)
    y = torch.empty((M, K), dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        L.swiglu_mlp_host(gu, down, xp, y, chunks=8, graph=True)
    torch.cuda.synchronize()
    assert torch.equal(y, L.swiglu_mlp(gu, down, x2.to(dev)).cpu())
