"""Converted engines on disk for this build's weight layout (the interface of the reference's tfimage/store.py).

A converted engine is one safetensors file: the small bf16 tensors of the model, per block the RMS-norm weights and
the four linears, and a JSON ``tfimage`` metadata entry with the format number and each linear's kind and scalars.
Same file structure, names and cache key as the reference store (store.py:19-124); what changes is the content of an
NVFP4 linear's ``bs`` tensor, so ``FORMAT`` is bumped and engines converted for the reference's TensorFold layout
are converted again instead of being misread.

Format 2, per NVFP4 linear ``<prefix>``:

* ``<prefix>words`` int32 [N, K/8]: the E2M1 codes, 8 per word, even element in the lowest nibble (byte view =
  codes [N, K/2], two per byte, low nibble first -- the reference's nibble order);
* ``<prefix>bs`` uint8 [ceil(N/128) * K/64 * 512]: the E4M3 block scales in the GEMM's tiled layout: 512-byte
  chunks [ceil(N/128)][K/64][512], row r / scale j of a chunk at (r%32)*16 + ((r%128)/32)*4 + (j%4), rows past N
  zero (``linear.sf_tile``; ``Fp4Linear.scales()`` gives back the row-major [N, K/16] view);
* metadata ``scale`` (the weight global g), ``n``, ``k``, ``act`` (static input scale, or null = dynamic), ``tile``.

FP8 and bf16 linears are stored as in format 1.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import torch

from . import linear as L

SMALL = ("img_in", "txt_norm", "txt_in1", "txt_in2", "t1", "t2", "mod", "norm_out", "proj_out")
FORMAT = 2


def cache_dir() -> Path:
    base = os.environ.get("TFIMAGE_CACHE") or os.path.join(os.environ.get("LOCALAPPDATA", str(Path.home())), "tfimage")
    path = Path(base)
    path.mkdir(parents=True, exist_ok=True)
    return path


def key(source: str | Path, spec: str) -> str:
    """Cache name for (source file, precision spec): path, size, mtime, spec and FORMAT (store.py:28-33)."""
    st = os.stat(source)
    raw = f"{Path(source).resolve()}|{st.st_size}|{st.st_mtime_ns}|{spec}|{FORMAT}"
    return f"{Path(source).stem}-{spec.replace(':', '_').replace(',', '_').replace('=', '-')}-" \
           f"{hashlib.sha1(raw.encode()).hexdigest()[:10]}"


def linear_tensors(prefix: str, lin: L.Linear) -> tuple[dict, dict]:
    """A linear's tensors (names under ``prefix``) and its metadata entry."""
    if isinstance(lin, L.Nvfp4Linear):
        f = lin.lin
        return ({prefix + "words": f.words, prefix + "bs": f.bs},
                {"kind": "nvfp4", "scale": f.scale, "n": f.n, "k": f.k, "act": None if lin.dynamic else f.act,
                 "tile": lin.tile})
    if isinstance(lin, L.Fp8Linear):
        return ({prefix + "w8": lin.w8.view(torch.uint8), prefix + "ws": lin.ws.reshape(-1)},
                {"kind": "fp8", "n": lin.n, "k": lin.k, "act": lin.act, "per_channel": lin.ws.numel() > 1})
    return {prefix + "w": lin.w}, {"kind": "bf16", "n": lin.n, "k": lin.k}


def linear_load(t: dict, prefix: str, m: dict, device) -> L.Linear:
    """The linear ``linear_tensors`` stored, on ``device``."""
    if m["kind"] == "nvfp4":
        words, bs = t[prefix + "words"].to(device), t[prefix + "bs"].to(device)
        expect = (m["n"] + 127) // 128 * (m["k"] // 64) * 512
        if tuple(words.shape) != (m["n"], m["k"] // 8) or bs.numel() != expect:
            raise ValueError(f"{prefix}: NVFP4 tensors do not match n={m['n']} k={m['k']} (format {FORMAT})")
        lin = L.Nvfp4Linear.from_fp4(L.Fp4Linear(words, bs, m["scale"], m["n"], m["k"],
                                                 act=m["act"] if m["act"] is not None else 1.0), tile=m.get("tile", 12))
        lin.dynamic = m["act"] is None
        return lin
    if m["kind"] == "fp8":
        lin = L.Fp8Linear.__new__(L.Fp8Linear)
        lin.w8 = t[prefix + "w8"].to(device).view(torch.float8_e4m3fn)
        ws = t[prefix + "ws"].to(device)
        lin.ws = ws if m.get("per_channel") else ws.reshape(())
        lin.n, lin.k, lin.act, lin._a, lin._a_val = m["n"], m["k"], m["act"], None, None
        return lin
    return L.Bf16Linear(t[prefix + "w"].to(device))


def save_linears(path: str | Path, linears: dict, extra: dict | None = None, meta: dict | None = None) -> None:
    """Named linears (+ extra plain tensors) to one safetensors file, written atomically."""
    from safetensors.torch import save_file

    tensors = {k: v for k, v in (extra or {}).items()}
    info = {"format": FORMAT, "linears": {}, **(meta or {})}
    for name, lin in linears.items():
        t, m = linear_tensors(f"{name}.", lin)
        tensors.update(t)
        info["linears"][name] = m
    path = Path(path)
    tmp = path.with_suffix(".tmp")
    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()}, str(tmp),
              metadata={"tfimage": json.dumps(info)})
    os.replace(tmp, path)


def read(path: str | Path) -> tuple[dict, dict]:
    """(tensors on the CPU, metadata) of a stored file; refuses other formats."""
    from safetensors import safe_open
    from safetensors.torch import load_file

    with safe_open(str(path), "pt") as f:
        info = json.loads(f.metadata()["tfimage"])
    if info.get("format") != FORMAT:
        raise ValueError(f"{path}: engine format {info.get('format')} (this build reads format {FORMAT}); convert it "
                         "again")
    return load_file(str(path), device="cpu"), info


def load_linears(path: str | Path, device="cuda") -> tuple[dict, dict, dict]:
    """(named linears on ``device``, the other tensors (CPU), metadata) of a ``save_linears`` file."""
    t, info = read(path)
    lins = {name: linear_load(t, f"{name}.", m, device) for name, m in info["linears"].items()}
    owned = {k for name in lins for k in t if k.startswith(name + ".")}
    return lins, {k: v for k, v in t.items() if k not in owned}, info


# ----------------------------------------------------------------------- the reference DiT (qwen_image21.QwenImage21)
def save(model, path: Path) -> None:
    """A converted QwenImage21 (store.py:52-63): SMALL tensors, per block norm_q / norm_k and the four linears."""
    extra = {name: getattr(model, name) for name in SMALL}
    lins = {}
    for i, b in enumerate(model.blocks):
        extra[f"{i}.norm_q"], extra[f"{i}.norm_k"] = b.norm_q, b.norm_k
        for proj in ("qkv", "out", "gate_up", "down"):
            lins[f"{i}.{proj}"] = getattr(b, proj)
    save_linears(path, lins, extra, {"kind": model.kind})


def load(path: Path, device="cuda"):
    """The QwenImage21 ``save`` stored (store.py:84-101); the model class is the reference's own module."""
    from .qwen_image21 import Block, Config, QwenImage21

    lins, t, info = load_linears(path, device)
    model = QwenImage21.__new__(QwenImage21)
    model.cfg, model.kind, model.device, model.prefix = Config(), info["kind"], torch.device(device), None
    model.prefixes = []
    for name in SMALL:
        setattr(model, name, t[name].to(device))
    model.blocks = [Block(*(lins[f"{i}.{p}"] for p in ("qkv", "out", "gate_up", "down")), t[f"{i}.norm_q"].to(device),
                          t[f"{i}.norm_k"].to(device)) for i in range(model.cfg.layers)]
    return model


def load_or_convert(source: str | Path, spec: str, device="cuda", log=print):
    """The converted engine for ``source`` at ``spec``: from the cache, or converted now and cached
    (store.py:104-124)."""
    from .qwen_image21 import QwenImage21

    path = cache_dir() / (key(source, spec) + ".safetensors")
    if path.is_file():
        log(f"[tfimage] loading converted {path.name}")
        return load(path, device)
    log(f"[tfimage] converting {Path(source).name} to {spec} (once; cached at {path})")
    model = QwenImage21.from_gguf(source, spec, device)
    contexts = cache_dir() / "calib_contexts.pt"
    if any(lin.kind == "nvfp4" for _, lin in model.linears()):
        if contexts.is_file():
            from .calibrate import calibrate

            calibrate(model, torch.load(contexts), log=log)
        else:
            log(f"[tfimage] no {contexts}: NVFP4 inputs are scaled per call (a host sync each); run "
                "bench/comfy_dump_contexts.py to calibrate")
    save(model, path)
    return model
