"""The C-ABI library and the host-side logic, without a GPU (no compute entry point is called here)."""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nvfp4 as onv
from tfimage import _lib, ext, linear as L

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "tfb.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(tfb_\w+)\s*\(", text, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    syms = header_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SIGNATURES), "the ctypes table must mirror include/tfb.h"


def test_pure_helpers():
    lib = _lib.load()
    assert lib.tfb_version() == 100
    assert lib.tfb_sf_tiled_bytes(300, 3072) == 3 * 48 * 512
    assert lib.tfb_sf_tiled_bytes(128, 100) == -1
    assert isinstance(lib.tfb_last_error(), bytes)


def test_use_prebuilt_returns_library_folder(tmp_path):
    assert (ext.use_prebuilt() / _lib.LIB_NAME).is_file()
    with pytest.raises(_lib.TfbError):
        _lib.load(tmp_path)          # an empty folder: no silent fallback


def test_sf_tile_matches_oracle_layout():
    rng = np.random.default_rng(0)
    s = rng.integers(0, 127, (300, 24), dtype=np.uint8)
    t = L.sf_tile(torch.from_numpy(s))
    np.testing.assert_array_equal(t.numpy(), onv.sf_tile(s))
    np.testing.assert_array_equal(L.sf_untile(t, 300, 384).numpy(), s)


def test_fp4linear_container_roundtrip_and_tiles():
    rng = np.random.default_rng(1)
    codes = torch.from_numpy(rng.integers(0, 256, (256, 64), dtype=np.uint8))
    scales = torch.from_numpy(rng.integers(0, 127, (256, 8), dtype=np.uint8)).view(torch.float8_e4m3fn)
    lin = L.Fp4Linear.from_checkpoint(codes, scales, 0.01, act=0.5)
    assert (lin.n, lin.k, lin.act, lin.scale) == (256, 128, 0.5, 0.01)
    assert lin.words.dtype == torch.int32 and lin.words.shape == (256, 16)
    assert torch.equal(lin.codes, codes)
    assert torch.equal(lin.scales().view(torch.uint8), scales.view(torch.uint8))
    half = lin.tiles(2, 4)                  # rows 128..255
    assert half.n == 128 and torch.equal(half.codes, codes[128:])
    assert torch.equal(half.scales().view(torch.uint8), scales.view(torch.uint8)[128:])


def test_make_dispatch_without_gpu():
    w = torch.randn(256, 384) * 0.02
    assert isinstance(L.make("fp8", w), L.Fp8Linear)
    assert isinstance(L.make("nvfp4", w), L.Fp8Linear)       # no sm_100 here: nvfp4 falls back like the reference
    assert isinstance(L.make("fp8", torch.randn(256, 200)), L.Bf16Linear)
    assert isinstance(L.make("bf16", w), L.Bf16Linear)
    assert not L.nvfp4_supported() or torch.cuda.is_available()


def test_fp8_weight_conversion_matches_reference_fixture():
    z = np.load(ROOT / "tests" / "golden" / "fp8.npz")
    lin = L.Fp8Linear(torch.from_numpy(z["w"]))
    np.testing.assert_array_equal(lin.w8.view(torch.uint8).numpy(), z["dyn_w8"])
    np.testing.assert_array_equal(lin.ws.reshape(1).numpy(), z["dyn_ws"])


def test_ops_refuse_cpu_tensors():
    with pytest.raises(_lib.TfbError):
        _lib.quant_nvfp4(torch.zeros(4, 64, dtype=torch.bfloat16), 1.0)


def test_gguf_block_table_and_host_checks():
    from oracle import gguf as og
    from tfimage import gguf_load

    lib = _lib.load()
    for kind, (vals, nbytes, type_id) in og.TYPES.items():
        assert _lib.GGUF_TYPES[kind] == type_id
        assert _lib.gguf_block(kind) == (vals, nbytes)
    assert lib.tfb_gguf_block_bytes(2, None) == -1                    # Q4_0: not decoded here
    assert set(gguf_load.DECODERS) == {"Q8_0", "Q6_K", "Q5_K", "Q4_K"}
    f16 = np.arange(6, dtype=np.float16)
    y = gguf_load.dequantize("F16", f16, (2, 3), "cpu", torch.float32)  # pass-through types are a cast
    assert torch.equal(y, torch.arange(6, dtype=torch.float32).view(2, 3))
    with pytest.raises(ValueError, match="IQ4_XS"):
        gguf_load.dequantize("IQ4_XS", np.zeros(136, np.uint8), (256,), "cpu")
    with pytest.raises(_lib.TfbError, match="no CPU path"):
        gguf_load.dequantize("Q4_K", og.random_blocks("Q4_K", 1, 0), (256,), "cpu")


def test_tp_layout():
    n, off = _lib.tp_layout(2, 4096, 3072)
    x, recv, fp, fx, ep = off
    assert x == 0 and recv == 4096 * 3072 * 2                   # x: the replicated residual stream
    assert ep > fx and n == ep + 256                            # the device epoch word
    assert fp - recv == 1 * 2048 * 3072 * 2                     # one receive slot of a 2048-row chunk
    tiles = (2048 // 128) * (3072 // 256)
    assert fx - fp == -(-tiles * 4 // 256) * 256 and ep >= fx + 2 * tiles * 4
    assert all(o % 256 == 0 for o in off)
    n8, off8 = _lib.tp_layout(8, 4100, 3072)                    # chunks rounded up to whole 256-row tiles
    assert off8[2] - off8[1] == 7 * 768 * 3072 * 2
    with pytest.raises(_lib.TfbError):
        _lib.tp_layout(1, 4096, 3072)
    with pytest.raises(_lib.TfbError):
        _lib.tp_layout(9, 4096, 3072)
    assert ctypes_sizeof_comm() == 4 + 4 + 8 * 8 + 8 + 8


def ctypes_sizeof_comm():
    import ctypes

    return ctypes.sizeof(_lib.TpComm)
