"""Shared pieces of the DiT parity tests: block inputs at any token count, the GPU block in record mode, the
stage-wise comparison (every stage against the oracle fed that stage's GPU input) and the end-to-end comparison
(the oracle block run from x alone) with its per-intermediate attribution."""

import numpy as np
import torch
from _helpers import f32, rel_l2, u8

from oracle import dit as odit
from oracle import fusions, nvfp4
from tfimage import mmdit


def lin_tuple(lin):
    w = lin.lin
    return (w.codes.cpu().numpy(), w.scales().view(torch.uint8).cpu().numpy(), w.scale, w.act)


def weights(b):
    return {n: lin_tuple(getattr(b, n)) for n in ("qkv", "out", "gate_up", "down")}


def sdpa_gpu(q, k, v, causal):
    """The reference's attention (torch SDPA, bf16) on the oracle's own q, k, v."""
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).cuda().transpose(1, 2)  # noqa: E731
    return f32(mmdit._sdpa(t(q), t(k), t(v), causal).transpose(1, 2))


def image_case(m, ctx, dev, hw=16, seed=7, t=0.7, prefix=None):
    """Block inputs of the image stream: x [1, hw*hw, dim] N(0,1), the step's modulation at timestep t, the RoPE
    table of the image ids behind the prompt, and the first image block's kept prefix keys / values."""
    cfg = m.cfg
    prefix = m.build_prefix(ctx) if prefix is None else prefix
    x = (torch.randn((1, hw * hw, cfg.dim), generator=torch.Generator().manual_seed(seed))).to(torch.bfloat16)
    mod = m._mod(m._temb(torch.tensor([t], device=dev)), m.mod_img)
    cos, sin = mmdit.rope_table(mmdit.image_ids(hw, hw, prefix.next_pos, dev), cfg)
    return x.to(dev), mod, cos, sin, prefix.kv[0][0], prefix.kv[0][1]


def text_case(m, dev, n=64, seed=8):
    """Block inputs of the text stream (the prompt prefix pass: t = 0 modulation, causal, no earlier prefix)."""
    cfg = m.cfg
    x = (torch.randn((1, n, cfg.dim), generator=torch.Generator().manual_seed(seed))).to(torch.bfloat16).to(dev)
    mod = m._mod(m._temb(torch.zeros((1,), device=dev)), m.mod_txt)
    cos, sin = mmdit.rope_table(mmdit.text_ids(n, dev), cfg)
    empty = torch.empty((1, 0, cfg.heads, cfg.head_dim), dtype=torch.bfloat16, device=dev)
    return x, mod, cos, sin, empty, empty


def gpu_block(m, b, x, mod, cos, sin, kpre, vpre, causal, record=None):
    cfg = m.cfg
    B, N, _ = x.shape
    P = kpre.shape[1]
    kbuf = torch.empty((B, P + N, cfg.heads, cfg.head_dim), dtype=torch.bfloat16, device=x.device)
    vbuf = torch.empty_like(kbuf)
    kbuf[:, :P] = kpre
    vbuf[:, :P] = vpre
    y = m._block(b, x.clone(), mod, cos, sin, kbuf, vbuf, causal=causal, record=record)
    torch.cuda.synchronize()
    return y, kbuf, vbuf


def oracle_block(m, b, x_np, case, causal, attn, parts=False, acc="f32"):
    _, mod, cos, sin, kpre, vpre = case
    B = x_np.shape[0]
    return odit.block(x_np, [f32(t.reshape(B, -1)) for t in mod], cos.cpu().numpy(), sin.cpu().numpy(), f32(kpre),
                      f32(vpre), weights(b), b.norm_q.cpu().numpy(), b.norm_k.cpu().numpy(), m.cfg.heads, m.cfg.eps,
                      causal=causal, attn=attn, return_parts=parts, acc=acc)


def summation_spread(m, b, x_np, case, causal, attn):
    """(rel-L2 between the oracle block with the reference's fp32 GEMM sums and the same block with exact (float64)
    sums from the same input, the exact-sum block output): the first is how far an equally valid summation order
    moves the block output through the chain of NVFP4 requantizations -- the floor under any end-to-end comparison
    with the fp32 oracle; the second is the reference arithmetic without summation error."""
    exact = oracle_block(m, b, x_np, case, causal, attn, acc="f64")
    return rel_l2(oracle_block(m, b, x_np, case, causal, attn), exact), exact


def end_to_end(m, b, case, causal, attn, attribution=False):
    """rel-L2 of the GPU block output against the oracle block run from the same x; with ``attribution`` also the
    rel-L2 of each intermediate (GPU record mode against the oracle's own chain)."""
    x, mod, cos, sin, kpre, vpre = case
    y, _, _ = gpu_block(m, b, x, mod, cos, sin, kpre, vpre, causal)
    if not attribution:
        return rel_l2(f32(y), oracle_block(m, b, f32(x), case, causal, attn))
    ref, parts = oracle_block(m, b, f32(x), case, causal, attn, parts=True)
    rec: dict = {}
    yr, kbuf, vbuf = gpu_block(m, b, x, mod, cos, sin, kpre, vpre, causal, record=rec)
    P = kpre.shape[1]
    B, N, _ = x.shape
    att = {
        "a": rel_l2(f32(rec["a_in"].out), parts["a"]),
        "qkv": rel_l2(f32(rec["qkv"]).reshape(B, N, -1), parts["qkv"]),
        "q": rel_l2(f32(rec["q"]), parts["q"]), "k": rel_l2(f32(kbuf[:, P:]), parts["k"]),
        "v": rel_l2(f32(vbuf[:, P:]), parts["v"]), "o": rel_l2(f32(rec["o"]), parts["o"]),
        "att": rel_l2(f32(rec["att"]), parts["att"]), "x1": rel_l2(f32(rec["x1"]), parts["x1"]),
        "m": rel_l2(f32(rec["m_in"].out), parts["m"]), "mlp": rel_l2(f32(rec["mlp"]), parts["mlp"]),
        "out": rel_l2(f32(yr), ref), "out_fused": rel_l2(f32(y), ref),
        "a_codes_equal": float(np.mean(u8(rec["a_in"].codes) == nvfp4.quantize(parts["a"].reshape(B * N, -1),
                                                                                 rec["a_in"].act)[0])),
    }
    return att["out_fused"], att


def stagewise(m, b, case, causal):
    """Each stage of the GPU block against the oracle on that stage's GPU input; returns the rel-L2 per stage
    (NVFP4 codes and scales of both quantizer stages are asserted bit-exact on the way)."""
    x, mod, cos, sin, kpre, vpre = case
    eps = m.cfg.eps
    B, N, D = x.shape
    sh1, sc1, g1, sh2, sc2, g2 = [f32(t.reshape(B, 1, -1)) for t in mod]
    rec: dict = {}
    y, kbuf, vbuf = gpu_block(m, b, x, mod, cos, sin, kpre, vpre, causal, record=rec)
    P = kpre.shape[1]
    r = {}

    def quant_stage(tag, act, bf_in, adaln_ref):
        r[tag + "_adaln"] = rel_l2(f32(bf_in), adaln_ref)
        c_ref, s_ref = nvfp4.quantize(f32(bf_in).reshape(B * N, D), act.act)
        assert np.array_equal(u8(act.codes), c_ref), f"{tag}: NVFP4 codes differ from the oracle quantizer"
        assert np.array_equal(u8(act.sf), nvfp4.sf_tile(s_ref)), f"{tag}: NVFP4 scales differ"
        return act

    def gemm_stage(act, lin):
        wc, ws, wg, _ = lin_tuple(lin)
        sf = nvfp4.sf_untile(u8(act.sf), act.m, act.k)
        return nvfp4.bf16_round(nvfp4.gemm(u8(act.codes), sf, act.act, wc, ws, wg))

    a = quant_stage("a", rec["a_in"], rec["a_in"].out, fusions.adaln(f32(x), sc1, eps, shift=sh1))
    r["qkv"] = rel_l2(f32(rec["qkv"]).reshape(B * N, -1), gemm_stage(a, b.qkv))
    src = f32(rec["qkv"])
    r["q"] = rel_l2(f32(rec["q"]), fusions.rms_rope(src, 0, f32(b.norm_q), f32(cos), f32(sin), eps))
    r["k"] = rel_l2(f32(kbuf[:, P:]), fusions.rms_rope(src, 1, f32(b.norm_k), f32(cos), f32(sin), eps))
    r["v"] = rel_l2(f32(vbuf[:, P:]), src[:, :, 2])
    r["attn_sdpa_vs_f64"] = rel_l2(f32(rec["o"]), odit.attention(f32(rec["q"]), f32(kbuf), f32(vbuf), causal))
    wc, ws, wg, act_out = lin_tuple(b.out)
    r["out"] = rel_l2(f32(rec["att"]).reshape(B * N, -1),
                      nvfp4.linear(f32(rec["o"]).reshape(B * N, -1), wc, ws, wg, act_out))
    x1_ref = nvfp4.bf16_round(f32(rec["x_in"]) + f32(rec["att"]) * g1)
    r["residual1"] = rel_l2(f32(rec["x1"]), x1_ref)
    mq = quant_stage("m", rec["m_in"], rec["m_in"].out, fusions.adaln(f32(rec["x1"]), sc2, eps, shift=sh2))
    dc, ds, dg, dact = lin_tuple(b.down)
    gu = gemm_stage(mq, b.gate_up)
    hc, hs = nvfp4.quantize(fusions.swiglu(gu), dact)
    y_ref = nvfp4.bf16_round(nvfp4.gemm(hc, hs, dact, dc, ds, dg)).reshape(B, N, D)
    r["mlp"] = rel_l2(f32(rec["mlp"]), y_ref)
    r["block"] = rel_l2(f32(y), nvfp4.bf16_round(f32(rec["x1"]) + y_ref * g2))
    print({k: f"{v:.2e}" for k, v in r.items()})
    return r
