"""Converted-engine store (tfimage/store.py, format 2): linears and plain tensors round-trip bit for bit through one
safetensors file; other formats are refused; on the GPU a reloaded NVFP4 layer computes exactly what the original
did."""

import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from tfimage import linear as L
from tfimage import store


def _nvfp4(n, k, seed, act=0.01):
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)
    scales = torch.randint(0x20, 0x48, (n, k // 16), dtype=torch.uint8, generator=g)
    lin = L.Nvfp4Linear.from_fp4(L.Fp4Linear.from_checkpoint(codes, scales, 0.0123, act=act if act else 1.0), tile=13)
    lin.dynamic = act is None
    return lin


def _check_same(a, b):
    assert type(a) is type(b) and (a.n, a.k) == (b.n, b.k)
    if isinstance(a, L.Nvfp4Linear):
        assert torch.equal(a.lin.words, b.lin.words) and torch.equal(a.lin.bs, b.lin.bs)
        assert (a.lin.scale, a.dynamic, a.tile) == (b.lin.scale, b.dynamic, b.tile)
        if not a.dynamic:
            assert a.lin.act == b.lin.act
    elif isinstance(a, L.Fp8Linear):
        assert torch.equal(a.w8.view(torch.uint8), b.w8.view(torch.uint8)) and torch.equal(a.ws, b.ws)
        assert a.act == b.act
    else:
        assert torch.equal(a.w, b.w)


def test_linears_round_trip(tmp_path):
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(96, 256, generator=g) * 0.02).to(torch.bfloat16)
    lins = {"a.qkv": _nvfp4(300, 256, 1), "a.out": _nvfp4(128, 384, 2, act=None),
            "b.fp8": L.Fp8Linear(w, 0.05, per_channel=True), "b.fp8t": L.Fp8Linear(w, None),
            "c.bf16": L.Bf16Linear(w)}
    extra = {"img_in": torch.randn(8, 4, generator=g), "0.norm_q": torch.ones(128)}
    path = tmp_path / "engine.safetensors"
    store.save_linears(path, lins, extra, {"kind": "nvfp4"})
    back, t, info = store.load_linears(path, device="cpu")
    assert info["format"] == store.FORMAT == 2 and info["kind"] == "nvfp4"
    assert set(back) == set(lins)
    for name in lins:
        _check_same(lins[name], back[name])
    assert set(t) == set(extra) and all(torch.equal(t[k], extra[k]) for k in extra)
    # the tiled scales read back as the same row-major view
    assert torch.equal(back["a.qkv"].lin.scales().view(torch.uint8), lins["a.qkv"].lin.scales().view(torch.uint8))


def test_other_formats_are_refused(tmp_path):
    from safetensors.torch import save_file

    path = tmp_path / "old.safetensors"
    save_file({"x": torch.zeros(1)}, str(path), metadata={"tfimage": json.dumps({"format": 1, "linears": {}})})
    with pytest.raises(ValueError, match="format 1"):
        store.read(path)


def test_model_save_layout(tmp_path):
    """store.save writes the reference model's structure (SMALL tensors, per-block norms and four linears)."""
    blocks = [SimpleNamespace(qkv=_nvfp4(384, 128, 10 + i), out=_nvfp4(128, 128, 20 + i), gate_up=_nvfp4(256, 128, 30 + i),
                              down=_nvfp4(128, 128, 40 + i), norm_q=torch.ones(128), norm_k=torch.ones(128) * 2)
              for i in range(2)]
    model = SimpleNamespace(kind="nvfp4", blocks=blocks, **{name: torch.full((2, 2), float(i)) for i, name in
                                                           enumerate(store.SMALL)})
    path = tmp_path / "m.safetensors"
    store.save(model, path)
    lins, t, info = store.load_linears(path, device="cpu")
    assert sorted(lins) == sorted(f"{i}.{p}" for i in range(2) for p in ("qkv", "out", "gate_up", "down"))
    for i, b in enumerate(blocks):
        for p in ("qkv", "out", "gate_up", "down"):
            _check_same(getattr(b, p), lins[f"{i}.{p}"])
        assert torch.equal(t[f"{i}.norm_k"], b.norm_k)
    assert all(torch.equal(t[name], getattr(model, name)) for name in store.SMALL)


def test_key_includes_format(tmp_path, monkeypatch):
    f = tmp_path / "w.gguf"
    f.write_bytes(b"x")
    k2 = store.key(f, "nvfp4")
    monkeypatch.setattr(store, "FORMAT", 1)
    assert store.key(f, "nvfp4") != k2


@pytest.mark.gpu
def test_reloaded_nvfp4_layer_is_identical(tmp_path, dev):
    from _helpers import bf16_cpu

    w = bf16_cpu((384, 512), seed=9, scale=0.02).to(dev)
    lin = L.Nvfp4Linear(w, act=0.003)
    path = tmp_path / "one.safetensors"
    store.save_linears(path, {"l": lin})
    back = store.load_linears(path, device=dev)[0]["l"]
    x = bf16_cpu((200, 512), seed=10).to(dev)
    assert torch.equal(lin(x), back(x))
    assert np.array_equal(lin.lin.bs.cpu().numpy(), back.lin.bs.cpu().numpy())


def test_model_level_functions_name_the_missing_reference_modules(tmp_path):
    """store.load / load_or_convert build the reference's QwenImage21; without its modules in the package the
    error says what to install."""
    with pytest.raises(ImportError, match="qwen_image21.py"):
        store.load(tmp_path / "missing.safetensors", device="cpu")
