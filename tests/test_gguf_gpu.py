"""GGUF block decode on the GPU (tfb_gguf_dequant through tfimage.gguf_load) against the CPU oracle (oracle/gguf.py,
pinned to the reference's decoders and to gguf-py): bit-exact in f32, f16 and bf16, for every decoded type, on
ragged block counts (partial last tile), a full-size weight, the reference's golden blocks and a GGUF file."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gguf as og
from tfimage import _lib, gguf_load

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
OUT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return t.view(torch.int32 if t.element_size() == 4 else torch.int16).numpy().reshape(-1)


def _oracle_bits(kind, raw, out) -> np.ndarray:
    y = og.dequantize(kind, raw, out)
    if out == "f32":
        return y.view(np.int32)
    if out == "bf16":
        return (y.view(np.uint32) >> 16).astype(np.uint16).view(np.int16)
    return y.astype(np.float16).view(np.int16)


@pytest.mark.parametrize("out", list(OUT))
@pytest.mark.parametrize("kind", list(og.TYPES))
@pytest.mark.parametrize("n_blocks", [1, 7, 8, 9, 65, 1000, 4099])
def test_decode_matches_oracle(dev, kind, out, n_blocks):
    vals, nbytes, _ = og.TYPES[kind]
    raw = og.random_blocks(kind, n_blocks, 1000 * n_blocks + len(kind))
    y = gguf_load.dequantize(kind, raw, (n_blocks * vals,), dev, OUT[out])
    assert y.dtype == OUT[out] and y.shape == (n_blocks * vals,)
    np.testing.assert_array_equal(_bits(y), _oracle_bits(kind, raw, out))


@pytest.mark.parametrize("kind", list(og.TYPES))
def test_decode_matches_reference_golden(dev, kind):
    z = np.load(GOLD / "gguf.npz")
    raw = z[f"{kind}_raw"]
    shape = z[f"{kind}_f32"].shape
    y32 = gguf_load.dequantize(kind, raw, shape, dev, torch.float32)
    np.testing.assert_array_equal(_bits(y32), z[f"{kind}_f32"].reshape(-1).view(np.int32))
    yb = gguf_load.dequantize(kind, raw, shape, dev, torch.bfloat16)
    np.testing.assert_array_equal(_bits(yb), z[f"{kind}_bf16"].reshape(-1).view(np.int16))


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K"])
def test_full_size_weight(dev, kind):
    """A [3072, 8192] weight (the down projection's shape): every value bit-exact in bf16."""
    vals, nbytes, _ = og.TYPES[kind]
    n = 3072 * 8192
    raw = og.random_blocks(kind, n // vals, 3)
    y = gguf_load.dequantize(kind, raw, (3072, 8192), dev, torch.bfloat16)
    np.testing.assert_array_equal(_bits(y), _oracle_bits(kind, raw, "bf16"))


def test_decoders_table_returns_block_rows(dev):
    raw = og.random_blocks("Q5_K", 5, 9)
    y = gguf_load.DECODERS["Q5_K"](torch.from_numpy(raw).to(dev))
    assert y.shape == (5, 256) and y.dtype == torch.float32
    np.testing.assert_array_equal(_bits(y), _oracle_bits("Q5_K", raw, "f32"))


def test_other_output_dtype_goes_through_f32(dev):
    raw = og.random_blocks("Q8_0", 4, 2)
    y = gguf_load.dequantize("Q8_0", raw, (4, 32), dev, torch.float64)
    np.testing.assert_array_equal(y.cpu().numpy().reshape(-1), og.dequantize("Q8_0", raw).astype(np.float64))


def test_gguf_file_roundtrip(dev, tmp_path):
    """tensors(path) on a GGUF file holding every decoded type plus F16 / F32: names, torch-order shapes and values
    as gguf-py decodes them."""
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize as gq

    path = tmp_path / "m.gguf"
    w = gguf.GGUFWriter(str(path), arch="tfimage-test")
    want = {}
    for i, kind in enumerate(og.TYPES):
        vals, nbytes, _ = og.TYPES[kind]
        rows, per_row = 6, 2 * (256 // vals)             # 6 rows x 512 values
        raw = og.random_blocks(kind, rows * per_row, 50 + i).reshape(rows, per_row * nbytes)
        w.add_tensor(f"blk.{kind}", raw, raw_dtype=getattr(T, kind))
        want[f"blk.{kind}"] = gq(raw, getattr(T, kind)).astype(np.float32).reshape(rows, 512)
    f16 = (np.random.default_rng(0).standard_normal((3, 40)) * 0.1).astype(np.float16)
    f32 = np.random.default_rng(1).standard_normal((5,)).astype(np.float32)
    w.add_tensor("norm.f16", f16)
    w.add_tensor("norm.f32", f32)
    want["norm.f16"], want["norm.f32"] = f16.astype(np.float32), f32
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    got = dict(gguf_load.tensors(path, dev, torch.float32))
    assert sorted(got) == sorted(want)
    for name, ref in want.items():
        assert tuple(got[name].shape) == ref.shape, name
        np.testing.assert_array_equal(got[name].cpu().numpy(), ref, err_msg=name)


def test_bad_inputs_are_refused_before_launch(dev):
    raw = torch.from_numpy(og.random_blocks("Q4_K", 3, 0)).to(dev)
    out = torch.empty(3 * 256, dtype=torch.bfloat16, device=dev)
    with pytest.raises(_lib.TfbError, match="BAD_ALIGN"):
        _lib.check(_lib.load().tfb_gguf_dequant(12, raw.data_ptr() + 1, 256, out.data_ptr(), 2, None))
    with pytest.raises(_lib.TfbError, match="BAD_SHAPE"):
        _lib.check(_lib.load().tfb_gguf_dequant(12, raw.data_ptr(), 300, out.data_ptr(), 2, None))
    with pytest.raises(_lib.TfbError, match="BAD_ARG"):
        _lib.check(_lib.load().tfb_gguf_dequant(2, raw.data_ptr(), 256, out.data_ptr(), 2, None))
    with pytest.raises(_lib.TfbError, match="BAD_ARG"):
        _lib.check(_lib.load().tfb_gguf_dequant(12, raw.data_ptr(), 256, out.data_ptr(), 7, None))
    _lib.check(_lib.load().tfb_gguf_dequant(12, raw.data_ptr(), 0, out.data_ptr(), 2, None))   # empty: no launch
    with pytest.raises(ValueError, match="Q2_K"):
        gguf_load.dequantize("Q2_K", np.zeros(84, np.uint8), (256,), dev)
