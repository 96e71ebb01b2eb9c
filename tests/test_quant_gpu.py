"""GPU quantizers against the oracle: NVFP4 codes/scales and FP8 bytes bit for bit."""

import numpy as np
import pytest
import torch
from _helpers import bf16_cpu, f32, u8

from oracle import fp8 as ofp8
from oracle import nvfp4 as onv
from tfimage import _lib

pytestmark = pytest.mark.gpu
GOLD = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def tie_rows():
    """Rows whose scaled values land exactly on every E2M1 rounding midpoint and on saturation.

    With g = 1/8: inv6g = 4/3, a block amax of 0.75 gives scale 1.0 and multiplier 1 / (1 * 1/8) = 8, so an
    element e/8 maps to e exactly."""
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0]
    blk = [6.0] + mids                                            # element 0 is the amax (6 / 8 = 0.75)
    row = np.array(blk + [-v for v in blk], dtype=np.float32) / 8
    return np.tile(row, (4, 4)), 1.0 / 8


@pytest.mark.parametrize("M,K", [(1, 64), (300, 192), (77, 448), (4096, 3072), (20000, 1344)])
@pytest.mark.parametrize("layout", [_lib.SF_ROWS, _lib.SF_TILED])
def test_quant_nvfp4_bit_exact(dev, M, K, layout):
    x = bf16_cpu((M, K), seed=M + K, outliers=8)
    g = onv.dynamic_act_global(float(x.float().abs().max()))
    codes, sf = _lib.quant_nvfp4(x.to(dev), g, layout)
    rc, rs = onv.quantize(x.float().numpy(), g)
    np.testing.assert_array_equal(u8(codes), rc)
    if layout == _lib.SF_ROWS:
        np.testing.assert_array_equal(u8(sf), rs)
    else:
        np.testing.assert_array_equal(u8(sf), onv.sf_tile(rs))       # padded rows included (zero)


@pytest.mark.parametrize("M,K", [(130, 80), (33, 336), (5, 16)])
def test_quant_nvfp4_rows_layout_ragged_segments(dev, M, K):
    """Row-major scales for K a multiple of 16 only: the last 256-element segment of each row is partial."""
    x = bf16_cpu((M, K), seed=3 * M + K, outliers=2)
    g = onv.dynamic_act_global(float(x.float().abs().max()))
    codes, sf = _lib.quant_nvfp4(x.to(dev), g, _lib.SF_ROWS)
    rc, rs = onv.quantize(x.float().numpy(), g)
    np.testing.assert_array_equal(u8(codes), rc)
    np.testing.assert_array_equal(u8(sf), rs)


def test_quant_nvfp4_rounding_midpoints(dev):
    xs, g = tie_rows()
    x = torch.from_numpy(xs).to(torch.bfloat16)
    assert torch.equal(x.float(), torch.from_numpy(xs))             # all exactly representable
    codes, sf = _lib.quant_nvfp4(x.to(dev), g, _lib.SF_ROWS)
    rc, rs = onv.quantize(xs, g)
    np.testing.assert_array_equal(u8(sf), rs)
    np.testing.assert_array_equal(u8(codes), rc)
    assert (rs == 0x38).all()                                       # scale 1.0


def test_quant_nvfp4_zero_blocks_tiny_and_huge(dev):
    x = torch.zeros(8, 128)
    x[1, :16] = -1e-30                 # negative values flushing to -0
    x[2, 16:32] = 3.0e38               # saturates the block scale
    x[3] = torch.linspace(-1e-5, 1e-5, 128)
    x = x.to(torch.bfloat16)
    for g in (1.0, 1e-9):
        codes, sf = _lib.quant_nvfp4(x.to(dev), g, _lib.SF_ROWS)
        rc, rs = onv.quantize(x.float().numpy(), g)
        np.testing.assert_array_equal(u8(codes), rc)
        np.testing.assert_array_equal(u8(sf), rs)


def test_quant_nvfp4_strided_rows(dev):
    base = bf16_cpu((64, 512), seed=5).to(dev)
    x = base[:, 128:384]                                            # ldx = 512
    g = 0.01
    codes, sf = _lib.quant_nvfp4(x, g, _lib.SF_ROWS)
    rc, rs = onv.quantize(f32(x), g)
    np.testing.assert_array_equal(u8(codes), rc)
    np.testing.assert_array_equal(u8(sf), rs)


def test_quant_nvfp4_rejects_bad_shapes(dev):
    x = torch.zeros(4, 96, dtype=torch.bfloat16, device=dev)
    with pytest.raises(_lib.TfbError, match="BAD_SHAPE"):
        _lib.quant_nvfp4(x, 1.0, _lib.SF_TILED)                     # tiled needs K % 64
    with pytest.raises(_lib.TfbError, match="BAD_ARG"):
        _lib.quant_nvfp4(torch.zeros(4, 64, dtype=torch.bfloat16, device=dev), 0.0)


@pytest.mark.parametrize("tag", ["dyn", "static"])
def test_quant_fp8_matches_reference_fixture(dev, tag):
    z = np.load(GOLD / "fp8.npz")
    x = torch.from_numpy(z["x"].view(np.int16)).view(torch.bfloat16).to(dev)
    if tag == "dyn":
        a = _lib.fp8_act_scale(x)
        assert float(a) == float(ofp8.act_scale(onv.bf16_from_bits(z["x"])))
    else:
        a = torch.tensor(float(z["static_act"]), device=dev)
    q = _lib.quant_fp8(x, a)
    np.testing.assert_array_equal(u8(q), z[f"{tag}_xq"])


def test_quant_fp8_large_ragged(dev):
    x = bf16_cpu((4968, 3072), seed=7, outliers=8)
    xd = x.to(dev)
    a = _lib.fp8_act_scale(xd)
    q = _lib.quant_fp8(xd, a)
    np.testing.assert_array_equal(u8(q), ofp8.quantize(x.float().numpy(), float(a)))


def test_absmax(dev):
    for n in (1, 7, 8, 1000, 4096 * 3072 + 5):
        x = bf16_cpu((n,), seed=n)
        assert float(_lib.absmax(x.to(dev))) == float(x.float().abs().max())
