"""Generate the golden fixtures in this folder by running the reference's own code on CPU.

Usage (needs a checkout of the reference ``tfimage`` project; it is not needed afterwards)::

    python tests/golden/make_golden.py --reference <path to the reference checkout>

What each file pins:
  * ``nvfp4_decode.npz`` -- the reference's ``deq`` (tools/gemm_tf.py:21-24, extracted from the source with ``ast``
    and executed; the rest of that script needs TensorFold and is not run) on seeded codes/scales: LUT, nibble
    order, scale broadcast and global multiply;
  * ``fusions.npz`` -- ``tfimage.kernels.adaln`` / ``rms_rope`` / ``swiglu`` (kernels.py:14-92), run on CPU by
    Triton's interpreter, plus ``_rope_table`` / ``_image_ids`` (qwen_image21.py:63-72,164-169);
  * ``fp8.npz`` -- ``tfimage.linear.Fp8Linear`` (linear.py:70-102) on CPU: ``w8``, ``ws``, the e4m3 activations
    it hands to ``torch._scaled_mm`` (captured by wrapping that call) and its bf16 output, dynamic and static act;
  * ``gguf.npz`` -- ``tfimage.gguf_load.dequantize`` (gguf_load.py:17-86) on CPU for Q8_0 / Q4_K / Q5_K / Q6_K
    blocks made by ``oracle.gguf.random_blocks``: the fp32 values and the bf16 output.
bf16 tensors are stored as uint16 bit patterns.
"""

from __future__ import annotations

import argparse
import ast
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bits(t):
    import torch
    return t.detach().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def extract_deq(ref: Path):
    src = (ref / "tools" / "gemm_tf.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "deq")
    import torch
    ns = {"torch": torch}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "gemm_tf.deq", "exec"), ns)
    return ns["deq"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["gguf"], help="regenerate one fixture only")
    args = ap.parse_args()
    ref = Path(args.reference).resolve()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(ref))
    import torch
    if args.only == "gguf":
        return make_gguf()
    from tfimage import kernels as K
    from tfimage import linear as L
    from tfimage.qwen_image21 import Config, QwenImage21, _rope_table

    # ---------------------------------------------------------------- NVFP4 decode side
    deq = extract_deq(ref)
    g = torch.Generator().manual_seed(11)
    codes = torch.randint(0, 256, (16, 32), generator=g, dtype=torch.uint8)
    scales = torch.randint(0, 0x7F, (16, 4), generator=g, dtype=torch.uint8)       # finite positive e4m3
    gl = 0.0123
    out = deq(codes, scales, gl)
    np.savez_compressed(HERE / "nvfp4_decode.npz", codes=codes.numpy(), scales=scales.numpy(), g=np.float64(gl),
                        out=out.numpy().astype(np.float32))

    # ---------------------------------------------------------------- fusions
    torch.manual_seed(0)
    fx = {}
    for tag, (B, N, D) in {"a": (2, 37, 256), "b": (1, 6, 3072)}.items():
        x = (torch.randn(B, N, D) * 3).to(torch.bfloat16)
        s = torch.randn(B, 1, D) * 0.2
        fx[f"adaln_{tag}_x"], fx[f"adaln_{tag}_s"] = bits(x), s.numpy()
        fx[f"adaln_{tag}_y"] = bits(K.adaln(x, s, 1e-6))
    B, N, H, Dh, P = 2, 9, 4, 128, 3
    qkv = torch.randn(B, N, 3, H, Dh).to(torch.bfloat16)
    w = torch.rand(Dh) + 0.5
    cfg = Config()
    ids = torch.stack([torch.arange(N).float()] * 3, -1)
    cos, sin = _rope_table(ids, cfg)
    buf = torch.zeros(B, P + N, H, Dh, dtype=torch.bfloat16)
    K.rms_rope(qkv, 1, w, cos, sin, 1e-6, buf[:, P:])
    q = torch.empty(B, N, H, Dh, dtype=torch.bfloat16)
    K.rms_rope(qkv, 0, w, cos, sin, 1e-6, q)
    fx.update(rr_qkv=bits(qkv), rr_w=w.numpy(), rr_cos=cos.numpy(), rr_sin=sin.numpy(), rr_kbuf=bits(buf),
              rr_q=bits(q), rr_prefix=np.int64(P))
    gu = (torch.randn(6, 2 * 160) * 2).to(torch.bfloat16)
    fx.update(sw_gu=bits(gu), sw_y=bits(K.swiglu(gu)))
    # RoPE table on a small image grid behind 16 text positions (3-axis ids, axes 16/56/56)
    model = QwenImage21.__new__(QwenImage21)
    model.device = torch.device("cpu")
    img = model._image_ids(8, 6, 16, (8, 6))
    txt = torch.arange(16, dtype=torch.float32)[:, None].expand(16, 3)
    allids = torch.cat([txt, img])
    c2, s2 = _rope_table(allids, cfg)
    fx.update(rope_ids=allids.numpy(), rope_cos=c2.numpy(), rope_sin=s2.numpy())
    np.savez_compressed(HERE / "fusions.npz", **fx)

    # ---------------------------------------------------------------- FP8 W8A8
    torch.manual_seed(1)
    w = torch.randn(48, 64) * 0.02
    x = torch.randn(10, 64).to(torch.bfloat16)
    x[:, 5] *= 20
    captured = {}
    real = torch._scaled_mm

    def spy(a, b, **kw):
        captured["xq"] = a.view(torch.uint8).clone()
        return real(a, b, **kw)

    fp = {}
    for tag, act in (("dyn", None), ("static", 0.05)):
        lin = L.Fp8Linear(w, act)
        torch._scaled_mm = spy
        try:
            y = lin(x)
        finally:
            torch._scaled_mm = real
        fp[f"{tag}_xq"] = captured["xq"][: x.shape[0]].numpy()
        fp[f"{tag}_y"] = bits(y)
        fp[f"{tag}_w8"] = lin.w8.view(torch.uint8).numpy()
        fp[f"{tag}_ws"] = lin.ws.reshape(1).numpy()
    fp.update(w=w.numpy(), x=bits(x), static_act=np.float32(0.05))
    np.savez_compressed(HERE / "fp8.npz", **fp)
    make_gguf()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


def make_gguf():
    import torch
    from tfimage import gguf_load

    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.gguf import TYPES, random_blocks

    out = {}
    for i, kind in enumerate(TYPES):
        vals, nbytes, _ = TYPES[kind]
        raw = random_blocks(kind, 24, 100 + i)
        shape = (len(raw) // nbytes * vals // 64, 64)
        out[f"{kind}_raw"] = raw
        out[f"{kind}_f32"] = gguf_load.dequantize(kind, raw, shape, "cpu", torch.float32).numpy()
        out[f"{kind}_bf16"] = bits(gguf_load.dequantize(kind, raw, shape, "cpu", torch.bfloat16))
    np.savez_compressed(HERE / "gguf.npz", **out)


if __name__ == "__main__":
    main()
