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
def _model_modules():
    """(QwenImage21 module, calibrate module) of the reference DiT, which live beside this file when the reference's
    qwen_image21.py, calibrate.py and sampling.py are placed in this package (the model code itself is not part of
    this build: it runs unchanged on this package's linear / kernels)."""
    try:
        from . import calibrate, qwen_image21
    except ImportError as e:
        raise ImportError("tfimage.store needs the reference DiT modules qwen_image21.py, calibrate.py and "
                          "sampling.py inside the tfimage package (copy them from the reference checkout); "
                          f"import failed: {e}") from e
    return qwen_image21, calibrate


def save(model, path: Path) -> None:
    """A converted QwenImage21 (store.py:52-63): SMALL tensors, per block norm_q / norm_k and the four linears; the
    model's Config goes into the metadata (so models of other sizes load back with their own shapes)."""
    import dataclasses

    extra = {name: getattr(model, name) for name in SMALL}
    lins = {}
    for i, b in enumerate(model.blocks):
        extra[f"{i}.norm_q"], extra[f"{i}.norm_k"] = b.norm_q, b.norm_k
        for proj in ("qkv", "out", "gate_up", "down"):
            lins[f"{i}.{proj}"] = getattr(b, proj)
    meta = {"kind": model.kind}
    cfg = getattr(model, "cfg", None)
    if dataclasses.is_dataclass(cfg):
        meta["config"] = dataclasses.asdict(cfg)
    save_linears(path, lins, extra, meta)


def load(path: Path, device="cuda"):
    """The QwenImage21 ``save`` stored (store.py:84-101), rebuilt around the reference's own model class; without a
    stored Config (engines written by other tools) the reference's default Config is assumed."""
    qi, _ = _model_modules()
    lins, t, info = load_linears(path, device)
    fields = info.get("config")
    cfg = qi.Config(**{k: tuple(v) if isinstance(v, list) else v for k, v in fields.items()}) if fields else qi.Config()
    model = qi.QwenImage21.__new__(qi.QwenImage21)
    model.cfg, model.kind, model.device, model.prefix = cfg, info["kind"], torch.device(device), None
    model.prefixes = []
    for name in SMALL:
        setattr(model, name, t[name].to(device))
    model.blocks = [qi.Block(*(lins[f"{i}.{p}"] for p in ("qkv", "out", "gate_up", "down")),
                             t[f"{i}.norm_q"].to(device), t[f"{i}.norm_k"].to(device)) for i in range(cfg.layers)]
    return model


def load_or_convert(source: str | Path, spec: str, device="cuda", log=print):
    """The engine of GGUF file ``source`` at precision ``spec`` (store.py:103-124): a conversion already in the cache
    is loaded; otherwise the file is converted now, its NVFP4 input scales calibrated when the calibration contexts
    file is in the cache (else they stay dynamic, measured on every call), and the result stored for next time."""
    qi, cal = _model_modules()
    target = cache_dir() / f"{key(source, spec)}.safetensors"
    if target.is_file():
        log(f"[tfimage] engine {target.name} found in the cache")
        return load(target, device)
    log(f"[tfimage] first use of {Path(source).name} at {spec}: converting, then caching it as {target}")
    model = qi.QwenImage21.from_gguf(source, spec, device)
    if any(lin.kind == "nvfp4" for _, lin in model.linears()):
        contexts = cache_dir() / "calib_contexts.pt"
        if not contexts.is_file():
            log(f"[tfimage] {contexts} is missing, so NVFP4 input scales stay dynamic (one host sync per linear "
                "call); dump calibration contexts first to make them static")
        else:
            cal.calibrate(model, torch.load(contexts), log=log)
    save(model, target)
    return model
