"""Child process of tests/test_dropin_gpu.py (a separate interpreter, so that its ``tfimage`` is the assembled
package: the reference's own qwen_image21.py / calibrate.py / sampling.py on this build's linear.py / kernels.py).

    python _dropin_child.py <package root> <repository root> <result json> <scratch dir>

Builds a reduced Qwen-Image DiT with the reference's QwenImage21 class and "nvfp4" linears from ``make``, runs the
reference's calibrate() (dynamic scales, the unfused MLP fallback, then static scales), runs forward() twice through
the kept-prefix path, round-trips the model through store.save / store.load, and runs the same reference model with
oracle-backed linears and fusions (the checker) on the same weights and static scales."""

import json
import sys
from pathlib import Path

pkg_root, repo_root, out_path, scratch = sys.argv[1:5]
sys.path.insert(0, pkg_root)
sys.path.insert(1, repo_root)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import tfimage  # noqa: E402
from tfimage import calibrate as cal  # noqa: E402
from tfimage import kernels as K  # noqa: E402
from tfimage import linear as L  # noqa: E402
from tfimage import qwen_image21 as qi  # noqa: E402
from tfimage import store  # noqa: E402

from oracle import fusions as ofu  # noqa: E402  (the checker only)
from oracle import nvfp4 as onv  # noqa: E402

assert Path(tfimage.__file__).parent == Path(pkg_root) / "tfimage", tfimage.__file__
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
cfg = qi.Config(layers=2, dim=256, heads=2, head_dim=128, mlp=512, in_ch=64)
TXT = 512


def weights(seed: int) -> dict:
    """The checkpoint tensor names QwenImage21.__init__ reads (qwen_image21.py:96-123), seeded, bf16 on the CPU."""
    g = torch.Generator().manual_seed(seed)
    D, F, C = cfg.dim, cfg.mlp, cfg.in_ch
    r = lambda *s, std=0.05: (torch.randn(s, generator=g) * std).to(torch.bfloat16)   # noqa: E731
    w = {"img_in.weight": r(D, C, std=0.2), "txt_in.text_norm.weight": r(TXT, std=0.1),
         "txt_in.in_layer.weight": r(D, TXT), "txt_in.out_layer.weight": r(D, D, std=0.1),
         "time_text_embed.timestep_embedder.linear_1.weight": r(D, 256), "time_text_embed.timestep_embedder."
         "linear_2.weight": r(D, D, std=0.1), "modulation.1.weight": r(4 * D, D, std=0.1),
         "norm_out.linear.weight": r(D, D, std=0.1), "proj_out.weight": r(C, D, std=0.1)}
    for i in range(cfg.layers):
        p = f"transformer_blocks.{i}."
        for n in ("to_q", "to_k", "to_v"):
            w[p + f"attn.{n}.weight"] = r(D, D)
        w[p + "attn.to_out.0.weight"] = r(D, D)
        w[p + "img_mlp.gate_layer.weight"] = r(F, D)
        w[p + "img_mlp.proj.weight"] = r(F, D)
        w[p + "img_mlp.out.weight"] = r(D, F)
        w[p + "attn.norm_q.weight"] = (1 + r(cfg.head_dim, std=0.05).float()).to(torch.bfloat16)
        w[p + "attn.norm_k.weight"] = (1 + r(cfg.head_dim, std=0.05).float()).to(torch.bfloat16)
    return w


W = weights(3)
g = torch.Generator().manual_seed(4)
ctx = torch.randn((1, 16, TXT), generator=g).to(torch.bfloat16)
x = torch.randn((1, cfg.in_ch, 8, 8), generator=g).to(torch.bfloat16).to(dev)
t = torch.tensor([0.6], device=dev)
res: dict = {}

# ------------------------------------------------------------------ the reference model on this build's API
model = qi.QwenImage21(dict(W), "nvfp4", dev, cfg)
lins = dict(model.linears())
res["kinds"] = sorted({type(lin).__name__ for lin in lins.values()})
res["dynamic_before"] = all(lin.dynamic for lin in lins.values())
acts = cal.calibrate(model, [ctx.to(dev)], steps=3, sizes=((8, 8),), log=lambda *a: None)
res["static_after"] = not any(lin.dynamic for lin in lins.values()) and all(v > 0 for v in acts.values())
res["fused_mlp"] = L.swiglu_mlp(model.blocks[0].gate_up, model.blocks[0].down,
                                torch.zeros((4, cfg.dim), dtype=torch.bfloat16, device=dev)) is not None
y = model(x, t, ctx)
y2 = model(x, t, ctx)                                   # same prompt: the kept prefix is reused
res["prefix_reused"] = len(model.prefixes) == 1
res["repeat_equal"] = bool(torch.equal(y, y2))
res["finite"] = bool(torch.isfinite(y.float()).all())
res["shape"] = list(y.shape)

# ------------------------------------------------------------------ engine store round trip
path = Path(scratch) / "engine.safetensors"
store.save(model, path)
loaded = store.load(path, dev)
res["store_equal"] = bool(torch.equal(loaded(x, t, ctx), y))
res["store_cfg"] = loaded.cfg == cfg


# ------------------------------------------------------------------ the checker: same model, oracle arithmetic
class OracleNvfp4(L.Linear):
    """NVFP4 linear as the reference's CPU path: quantize (oracle), dequantize, fp32 matmul, bf16."""

    kind = "nvfp4"
    acc = "f32"                                        # "f64": the same products summed exactly

    def __init__(self, w, act):
        a = w.float().cpu().numpy()
        self.gw = onv.weight_global(np.abs(a).max())
        self.wc, self.ws = onv.quantize(a, self.gw)
        self.act, self.n, self.k = float(act), w.shape[0], w.shape[1]

    def __call__(self, xin):
        out = onv.linear(xin.float().cpu().numpy(), self.wc, self.ws, self.gw, self.act, OracleNvfp4.acc)
        return torch.from_numpy(out).to(torch.bfloat16).to(xin.device)


def o_adaln(xin, scale, eps, out=None):
    B, N, D = xin.shape
    yv = ofu.adaln(xin.float().cpu().numpy(), scale.float().reshape(B, D).cpu().numpy(), eps)
    return torch.from_numpy(yv).to(torch.bfloat16).to(xin.device)


def o_rms_rope(src, part, w, cos, sin, eps, dst):
    yv = ofu.rms_rope(src.float().cpu().numpy(), part, w.float().cpu().numpy(), cos.cpu().numpy(),
                      sin.cpu().numpy(), eps)
    dst.copy_(torch.from_numpy(yv).to(torch.bfloat16))


def o_swiglu(gu):
    return torch.from_numpy(ofu.swiglu(gu.float().cpu().numpy())).to(torch.bfloat16).to(gu.device)


L.make = lambda kind, w, act=None: OracleNvfp4(w, act)
L.swiglu_mlp = lambda *a, **k: None
K.adaln, K.rms_rope, K.swiglu = o_adaln, o_rms_rope, o_swiglu
checker = qi.QwenImage21(dict(W), "nvfp4", dev, cfg, acts=acts)
yr = checker(x, t, ctx)
OracleNvfp4.acc = "f64"
checker.drop_prefixes()
yr64 = checker(x, t, ctx)


def rel(u, v):
    u, v = u.float().cpu().numpy().astype(np.float64), v.float().cpu().numpy().astype(np.float64)
    return float(np.linalg.norm(u - v) / np.linalg.norm(v))


res["rel_l2"] = rel(y, yr)
res["checker_fp32_vs_exact_sums"] = rel(yr64, yr)
res["rel_l2_vs_exact_sums"] = rel(y, yr64)
res["equal_frac"] = float(np.mean(y.float().cpu().numpy() == yr.float().cpu().numpy()))
res["equal_frac_vs_exact_sums"] = float(np.mean(y.float().cpu().numpy() == yr64.float().cpu().numpy()))
Path(out_path).write_text(json.dumps(res))
print(json.dumps(res))
