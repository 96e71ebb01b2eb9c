"""The CPU oracle against the reference's golden fixtures and known answers (no GPU)."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8, fusions, mlp, nvfp4
from oracle import gguf as ogguf

GOLD = Path(__file__).resolve().parent / "golden"


def ulp_bf16(v):
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


# ------------------------------------------------------------------------------------------------- NVFP4 side
def test_decode_matches_reference_deq():
    z = np.load(GOLD / "nvfp4_decode.npz")
    out = nvfp4.dequantize(z["codes"], z["scales"], float(z["g"]))
    np.testing.assert_array_equal(out, z["out"])


def test_lut_pinned():
    # tools/gemm_tf.py:22 -- the sign lives in bit 3
    assert nvfp4.E2M1_LUT.tolist() == [0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6]
    assert np.signbit(nvfp4.E2M1_LUT[8])


def test_e4m3_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    v = np.concatenate([
        (rng.standard_normal(100000) * np.exp2(rng.integers(-14, 10, 100000))).astype(np.float32),
        np.arange(0, 470, 1 / 64, dtype=np.float32),
        np.array([0, -0.0, 2 ** -9, 2 ** -10, 3 * 2 ** -11, 448, 449, 463.9, 464, 1e9], np.float32)])
    t = torch.from_numpy(np.clip(v, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(nvfp4.e4m3_encode(v), t)
    # satfinite: anything past 448 saturates
    assert nvfp4.e4m3_encode(np.float32(1e30)) == 0x7E
    assert nvfp4.e4m3_encode(np.float32(np.inf)) == 0x7E


def test_e2m1_round_to_nearest_even():
    grid = np.array([0, .5, 1, 1.5, 2, 3, 4, 6])
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-8, 8, 20000).astype(np.float32),
                        np.array([.25, .75, 1.25, 1.75, 2.5, 3.5, 5, -.25, -5, 6.5, 1e9, -0.0], np.float32)])
    a = np.minimum(np.abs(x).astype(np.float64), 6.0)
    d = np.abs(a[:, None] - grid[None])
    ref = []
    for row in d:
        c = np.nonzero(row == row.min())[0]
        ref.append(c[np.argmin(c % 2)])          # ties go to the even code (even mantissa)
    ref = np.array(ref) | (np.signbit(x).astype(np.int64) << 3)
    np.testing.assert_array_equal(nvfp4.e2m1_encode(x), ref)


def test_e2m1_lut_matches_format_definition():
    # E2M1: sign bit 3, exponent bits 2..1 (bias 1), mantissa bit 0; exponent 0 is subnormal (m * 0.5).
    # torch cannot decode float4_e2m1fn_x2 on the CPU, so the LUT is derived from the bit layout instead.
    ref = []
    for c in range(16):
        s, e, m = c >> 3, (c >> 1) & 3, c & 1
        v = m * 0.5 if e == 0 else 2.0 ** (e - 1) * (1 + m / 2)
        ref.append(-v if s else v)
    np.testing.assert_array_equal(nvfp4.E2M1_LUT, np.array(ref, dtype=np.float32))
    assert np.signbit(nvfp4.E2M1_LUT[8]) and not np.signbit(nvfp4.E2M1_LUT[0])
    # every code round-trips through the encoder (the -0 code included)
    np.testing.assert_array_equal(nvfp4.e2m1_encode(nvfp4.E2M1_LUT), np.arange(16))


def test_e4m3_table_matches_torch_float8():
    # the oracle's E4M3 decode against torch's float8_e4m3fn for all 256 bytes (0x7f / 0xff are NaN in both)
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(nvfp4.E4M3_TABLE, t)


def test_quantize_properties():
    rng = np.random.default_rng(2)
    x = nvfp4.bf16_round(rng.standard_normal((64, 256)).astype(np.float32))
    x[:, 7] *= 20
    g = nvfp4.dynamic_act_global(np.abs(x).max())
    c, s = nvfp4.quantize(x, g)
    assert c.shape == (64, 128) and s.shape == (64, 16)
    d = nvfp4.dequantize(c, s, g)
    # every block's max element maps to within one E4M3 step of 6 * scale
    rel = np.linalg.norm(d - x) / np.linalg.norm(x)
    assert rel < 0.15
    # idempotence: re-quantizing the dequantized tensor under the same global reproduces the codes and scales
    c2, s2 = nvfp4.quantize(d, g)
    np.testing.assert_array_equal(s2, s)
    np.testing.assert_array_equal(nvfp4.dequantize(c2, s2, g), d)


def test_quantize_zero_block_and_negative_zero():
    x = np.zeros((2, 32), np.float32)
    x[1, 16:] = -1e-30                     # rounds to -0 under a large global
    c, s = nvfp4.quantize(x, 1.0)
    assert (s == 0).all()
    assert (c[0] == 0).all()
    assert (c[1, 8:] == 0x88).all()        # "-0" codes: sign kept, magnitude zero


def test_sf_tile_roundtrip_and_layout():
    rng = np.random.default_rng(3)
    s = rng.integers(0, 127, (300, 24), dtype=np.uint8)
    t = nvfp4.sf_tile(s)
    assert t.size == 384 * 24
    np.testing.assert_array_equal(nvfp4.sf_untile(t, 300, 24 * 16), s)
    # row 37, scale 5: group 0, chunk 1, offset (37 % 32) * 16 + (37 // 32) * 4 + 1
    assert t[1 * 512 + 5 * 16 + 1 * 4 + 1] == s[37, 5]
    g2 = t.reshape(3, 6, 512)[2].reshape(6, 32, 4, 4)       # group 2 = rows 256..383: [chunk][r % 32][r // 32][j]
    assert (g2[:, :, 2:, :] == 0).all() and (g2[:, 12:, 1, :] == 0).all()     # padded rows 300..383 are zero


def test_gemm_oracle_matches_float_reference():
    rng = np.random.default_rng(4)
    x = nvfp4.bf16_round(rng.standard_normal((32, 128)).astype(np.float32))
    w = nvfp4.bf16_round((rng.standard_normal((48, 128)) * 0.02).astype(np.float32))
    gw = nvfp4.weight_global(np.abs(w).max())
    wc, ws = nvfp4.quantize(w, gw)
    ga = nvfp4.dynamic_act_global(np.abs(x).max())
    y = nvfp4.linear(x, wc, ws, gw, ga)
    ref = x @ w.T
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 0.2      # NVFP4 quantization error, not a parity bar


# ----------------------------------------------------------------------------------------------- fusions side
def test_adaln_matches_reference_triton():
    z = np.load(GOLD / "fusions.npz")
    for tag in ("a", "b"):
        x = nvfp4.bf16_from_bits(z[f"adaln_{tag}_x"])
        ref = nvfp4.bf16_from_bits(z[f"adaln_{tag}_y"])
        # the fixtures come from Triton's CPU interpreter, which rounds toward zero on the bf16 store: the oracle
        # with the same rounding reproduces them bit for bit; with round-to-nearest it is within one bf16 ulp
        np.testing.assert_array_equal(fusions.adaln(x, z[f"adaln_{tag}_s"], 1e-6, rounding="rz"), ref)
        y = fusions.adaln(x, z[f"adaln_{tag}_s"], 1e-6)
        assert (np.abs(y - ref) <= ulp_bf16(ref) + 1e-6).all()


def test_rms_rope_matches_reference_triton():
    z = np.load(GOLD / "fusions.npz")
    qkv = nvfp4.bf16_from_bits(z["rr_qkv"])
    P = int(z["rr_prefix"])
    for part, ref in ((1, nvfp4.bf16_from_bits(z["rr_kbuf"])[:, P:]), (0, nvfp4.bf16_from_bits(z["rr_q"]))):
        yz = fusions.rms_rope(qkv, part, z["rr_w"], z["rr_cos"], z["rr_sin"], 1e-6, rounding="rz")
        assert (yz == ref).mean() > 0.999 and (np.abs(yz - ref) <= ulp_bf16(ref)).all()
        y = fusions.rms_rope(qkv, part, z["rr_w"], z["rr_cos"], z["rr_sin"], 1e-6)
        assert (np.abs(y - ref) <= ulp_bf16(ref) + 1e-6).all()
    assert (z["rr_kbuf"][:, :P] == 0).all()         # the reference leaves prefix rows untouched


def test_swiglu_matches_reference_triton():
    # bit-exact under the interpreter's round-toward-zero stores (the silu intermediate is rounded too, so the
    # round-to-nearest oracle can differ from these fixtures by more than one ulp)
    z = np.load(GOLD / "fusions.npz")
    ref = nvfp4.bf16_from_bits(z["sw_y"])
    np.testing.assert_array_equal(fusions.swiglu(nvfp4.bf16_from_bits(z["sw_gu"]), rounding="rz"), ref)


def test_rope_table_matches_reference():
    z = np.load(GOLD / "fusions.npz")
    ids = np.concatenate([fusions.text_ids(16), fusions.image_ids(8, 6, 16, (8, 6))])
    np.testing.assert_array_equal(ids, z["rope_ids"])
    c, s = fusions.rope_table(ids)
    np.testing.assert_array_equal(c, z["rope_cos"])
    np.testing.assert_array_equal(s, z["rope_sin"])


# ---------------------------------------------------------------------------------------------------- FP8 side
@pytest.mark.parametrize("tag", ["dyn", "static"])
def test_fp8_matches_reference_fp8linear(tag):
    z = np.load(GOLD / "fp8.npz")
    w8, ws = fp8.weight(z["w"])
    np.testing.assert_array_equal(w8, z[f"{tag}_w8"])
    np.testing.assert_array_equal(np.atleast_1d(ws), z[f"{tag}_ws"])
    x = nvfp4.bf16_from_bits(z["x"])
    a = fp8.act_scale(x) if tag == "dyn" else np.float32(z["static_act"])
    xq = fp8.quantize(x, a)
    np.testing.assert_array_equal(xq, z[f"{tag}_xq"])
    y = fp8.gemm(xq, a, w8, ws)
    ref = nvfp4.bf16_from_bits(z[f"{tag}_y"])
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-3


def test_fp8_per_channel_reduces_to_tensorwise_on_uniform_rows():
    w = np.tile(np.linspace(-1, 1, 64, dtype=np.float32), (8, 1))
    w8a, sa = fp8.weight(w)
    w8b, sb = fp8.weight(w, per_channel=True)
    np.testing.assert_array_equal(w8a, w8b)
    np.testing.assert_array_equal(np.full(8, sa), sb)


def test_mlp_oracle_composition():
    rng = np.random.default_rng(5)
    M, K, F = 16, 64, 64
    x = nvfp4.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    wgu = nvfp4.bf16_round((rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32))
    wd = nvfp4.bf16_round((rng.standard_normal((K, F)) * 0.05).astype(np.float32))
    ggu, gd = nvfp4.weight_global(np.abs(wgu).max()), nvfp4.weight_global(np.abs(wd).max())
    guc, gus = nvfp4.quantize(wgu, ggu)
    dc, ds = nvfp4.quantize(wd, gd)
    ax = nvfp4.dynamic_act_global(np.abs(x).max())
    y, parts = mlp.forward(x, guc, gus, ggu, dc, ds, gd, ax, 0.01, return_parts=True)
    assert y.shape == (M, K) and parts["h_codes"].shape == (M, F // 2)
    np.testing.assert_array_equal(parts["h"], fusions.swiglu(parts["gu"]))


@pytest.mark.parametrize("kind", list(ogguf.TYPES))
def test_gguf_decoders_match_reference(kind):
    """oracle.gguf against the reference's own decoders (gguf_load.py:17-86, run on CPU): fp32 and bf16, bit-exact."""
    z = np.load(GOLD / "gguf.npz")
    raw = z[f"{kind}_raw"]
    y = ogguf.dequantize(kind, raw)
    assert np.array_equal(y.view(np.uint32), z[f"{kind}_f32"].reshape(-1).view(np.uint32))
    yb = ogguf.dequantize(kind, raw, "bf16")
    assert np.array_equal((yb.view(np.uint32) >> 16).astype(np.uint16), z[f"{kind}_bf16"].reshape(-1))


@pytest.mark.parametrize("kind", list(ogguf.TYPES))
def test_gguf_decoders_match_gguf_py(kind):
    """oracle.gguf against gguf-py 0.19.0's numpy decoders (ggml's block formats), bit-exact in fp32, on blocks
    with every byte value in the code / scale fields."""
    quants = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType

    vals, nbytes, type_id = ogguf.TYPES[kind]
    assert int(getattr(GGMLQuantizationType, kind)) == type_id
    raw = ogguf.random_blocks(kind, 2000, 7)
    ref = quants.dequantize(raw.reshape(-1, nbytes), getattr(GGMLQuantizationType, kind)).reshape(-1)
    y = ogguf.dequantize(kind, raw)
    assert y.size == raw.size // nbytes * vals
    assert np.array_equal(y.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_gguf_f16_output_and_bad_length():
    raw = ogguf.random_blocks("Q4_K", 3, 1)
    y = ogguf.dequantize("Q4_K", raw)
    assert np.array_equal(ogguf.dequantize("Q4_K", raw, "f16"), y.astype(np.float16).astype(np.float32))
    with pytest.raises(ValueError):
        ogguf.dequantize("Q4_K", raw[:-1])


def test_bf16_round_f64_is_a_single_correct_rounding():
    # bf16 neighbours and their midpoint are exact in float64, so the correctly rounded result is decidable exactly
    rng = np.random.default_rng(11)
    x = rng.standard_normal(20000) * np.exp2(rng.integers(-30, 30, 20000))
    # values that double rounding gets wrong: a bf16 midpoint nudged by less than half an fp32 ulp
    lo = nvfp4.bf16_round(rng.standard_normal(2000).astype(np.float32)).astype(np.float64)
    mid = lo + np.abs(lo) * 2.0 ** -8
    x = np.concatenate([x, mid + np.abs(mid) * 2.0 ** -30, mid - np.abs(mid) * 2.0 ** -30, mid])
    got = nvfp4.bf16_round_f64(x).astype(np.float64)
    # exact: the bf16 values on either side of x -- its float64 pattern truncated to 8 significand bits (toward
    # zero), and that plus one bf16 step (away from zero) -- then the nearer one, ties to the even pattern
    low = np.uint64((1 << 45) - 1)
    bits = x.view(np.uint64)
    down_bits = bits & ~low
    down = down_bits.view(np.float64)
    up = (down_bits + np.uint64(1 << 45)).view(np.float64)
    even = ((down_bits >> np.uint64(45)) & np.uint64(1)) == 0
    dd, du = np.abs(x - down), np.abs(up - x)          # exact: both neighbours are within 2^8 ulps of x
    ref = np.where(dd < du, down, np.where(dd > du, up, np.where(even, down, up)))
    np.testing.assert_array_equal(got, ref)


def test_silu_bf16_rne_is_correctly_rounded_and_near_the_reference_formula():
    # (below g = -88.7 the fp32 formula's e^-g overflows and it returns -0, while the exact silu is still a normal
    # bf16 down to g = -94; the comparison with the formula therefore stops at -85)
    g = nvfp4.bf16_round(np.linspace(-85, 30, 200001).astype(np.float32))
    exact = fusions.silu_bf16(g)                        # float64, one rounding
    ref_fp32 = fusions.silu_bf16(g, rounding="rz")      # the reference formula in fp32 (truncated)
    ulp = ulp_bf16(exact)
    assert np.all(np.abs(exact - ref_fp32) <= ulp * 1.0001)
    assert fusions.silu_bf16(np.float32(-90.0)) < 0     # -90 e^-90 = -7.4e-38: representable, not -0
    # against an independent float64 evaluation with the single rounding
    sel = np.abs(g) < 20
    e64 = g[sel].astype(np.float64) / (1.0 + np.exp(-g[sel].astype(np.float64)))
    np.testing.assert_array_equal(exact[sel], nvfp4.bf16_round_f64(e64))


def test_gemm_oracle_exact_sums_option():
    # float64 summation of the same products: equal to the fp32 result up to fp32 summation error
    rng = np.random.default_rng(12)
    x = nvfp4.bf16_round(rng.standard_normal((64, 512)).astype(np.float32))
    w = nvfp4.bf16_round((rng.standard_normal((96, 512)) * 0.02).astype(np.float32))
    gw = nvfp4.weight_global(np.abs(w).max())
    wc, ws = nvfp4.quantize(w, gw)
    ga = nvfp4.dynamic_act_global(np.abs(x).max())
    xc, xs = nvfp4.quantize(x, ga)
    a, b = nvfp4.gemm(xc, xs, ga, wc, ws, gw), nvfp4.gemm(xc, xs, ga, wc, ws, gw, acc="f64")
    assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()
