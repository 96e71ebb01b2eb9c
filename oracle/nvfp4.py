"""NVFP4 (E2M1 values, one E4M3 scale per 16 K-elements, fp32 global) CPU restatement -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this module; the product package
never does.

What is pinned against the reference (run in the build container, fixtures in ``tests/golden/``):
  * the decode LUT ``[0, .5, 1, 1.5, 2, 3, 4, 6, -0, -.5, ..., -6]`` with the sign in bit 3
    (``tools/gemm_tf.py:22``), low nibble = even element (``tools/gemm_tf.py:23``), and
    ``dequant = lut[code] * e4m3(scale) * global`` (``tools/gemm_tf.py:24``): :func:`dequantize` is checked
    bit-exactly against the reference's own ``deq`` function;
  * the per-row scale view ``[N, K/16]`` e4m3 that ``nvfp4_weight`` returns (``tfimage/linear.py:30-38``);
  * the global-scale formulas: weights ``max(amax, 1e-12) / (6*448)`` (``tfimage/linear.py:35``), dynamic
    activations ``max(amax, 1e-6) / (6*448)`` (``tfimage/linear.py:127``).

What is NOT pinned ("parity unpinned"): the encoder rounding. The reference calls TensorFold's ``quant4``
(``tfimage/linear.py:36``, ``tools/gemm_tf.py:17,45``), whose source is an absent submodule (TensorFold v0.6.1 @
``17c73e1``). This module therefore states the rounding this build adopts, following the published NVFP4
definition (E2M1 elements, E4M3 block scale per 16, fp32 tensor scale) the way ModelOpt-style quantizers apply it:

    g      = float32(global)
    inv6g  = 1 / (6 * g)                                   (fp32, round-to-nearest-even at each step)
    amax   = max |x_i| over the 16-element block           (exact)
    sf     = e4m3_rne_satfinite(amax * inv6g)              (clamp to 448, then round to nearest even)
    d      = float(sf) * g                                 (fp32 RN)
    inv    = 0 if d == 0 else 1 / d                        (fp32 RN)
    code_i = e2m1_rne_satfinite(x_i * inv)                 (ties to even; |v| > 6 saturates to 6)

The E2M1 sign bit is the sign bit of ``x_i * inv`` (so negative values that round to zero give code 8, "-0").
An all-zero block gets scale 0 and codes 0/8. Inputs are finite; NaN inputs give unspecified codes.
The GPU quantizers (standalone, AdaLN-fused and the SwiGLU GEMM epilogue) are bit-exact against this statement.
"""

from __future__ import annotations

import numpy as np

FP4_MAX, E4M3_MAX = 6.0, 448.0
# tools/gemm_tf.py:22 -- decode LUT, sign in bit 3
E2M1_LUT = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], dtype=np.float32)


# ----------------------------------------------------------------------------------------------- scalar formats
def bf16_round(x) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 values."""
    b = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def bf16_round_f64(x) -> np.ndarray:
    """float64 -> nearest bf16 (ties to even) with one rounding, as fp32 values. The value is first rounded to fp32
    by round-to-odd (toward zero, last bit set if inexact); fp32 keeps 16 more significand bits than bf16, so the
    round-to-nearest-even to bf16 that follows equals a single rounding of the float64 value (rounding to fp32 to
    nearest first could land exactly on a bf16 midpoint and round a second time the wrong way)."""
    x = np.asarray(x, dtype=np.float64)
    f = x.astype(np.float32)
    away = np.abs(f.astype(np.float64)) > np.abs(x)
    f = np.where(away, np.nextafter(f, np.float32(0)), f).astype(np.float32)
    inexact = (f.astype(np.float64) != x).astype(np.uint32)
    return bf16_round((np.ascontiguousarray(f).view(np.uint32) | inexact).view(np.float32)).reshape(np.shape(x))


def bf16_trunc(x) -> np.ndarray:
    """fp32 -> bf16 by rounding toward zero (what Triton's CPU interpreter does on a bf16 store)."""
    b = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32)
    return ((b >> 16) << 16).view(np.float32).reshape(np.shape(x))


def bf16_bits(x) -> np.ndarray:
    """fp32 values (already bf16-representable or not) -> uint16 bf16 bit patterns (RNE)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(u16) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for c in range(256):
        s, e, m = c >> 7, (c >> 3) & 15, c & 7
        if e == 15 and m == 7:
            v = np.nan
        elif e == 0:
            v = m * 2.0 ** -9
        else:
            v = (1 + m / 8) * 2.0 ** (e - 7)
        t[c] = -v if s else v
    return t


E4M3_TABLE = _e4m3_table()


def e4m3_decode(code) -> np.ndarray:
    return E4M3_TABLE[np.asarray(code, dtype=np.uint8)]


def e4m3_encode(v) -> np.ndarray:
    """fp32 -> E4M3 (fn) byte: saturate finite values to +-448, then round to nearest, ties to even."""
    v = np.asarray(v, dtype=np.float32)
    sign = (np.signbit(v).astype(np.uint16) << 7)
    a = np.minimum(np.abs(v).astype(np.float64), E4M3_MAX)
    nan = np.isnan(v)
    a = np.where(nan, 0.0, a)
    _, ex = np.frexp(a)
    e = np.maximum(ex.astype(np.int64) - 1, -6)                  # value = q * 2^(e-3), q in [8,16) for normals
    q = np.rint(a * np.exp2((3 - e).astype(np.float64)))        # exact power-of-two scaling; rint = ties-to-even
    carry = q >= 16
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 8, q)
    mag = ((e + 7) << 3) + (q.astype(np.int64) - 8)             # subnormals (e == -6, q < 8) give mag == q
    mag = np.where(a == 0, 0, mag)
    out = (mag.astype(np.uint16) | sign)
    out = np.where(nan, 0x7F | sign, out)
    return out.astype(np.uint8)


def e2m1_encode(v) -> np.ndarray:
    """fp32 -> 4-bit E2M1 code (0..15): round to nearest on {0,.5,1,1.5,2,3,4,6}, ties to even, saturate at 6."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v)
    mag = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5)
           + (a > 5.0)).astype(np.uint8)
    return (mag | (np.signbit(v).astype(np.uint8) << 3)).astype(np.uint8)


# ------------------------------------------------------------------------------------------------ global scales
def weight_global(amax: float) -> float:
    """tfimage/linear.py:35 -- g = max(amax(W), 1e-12) / (6*448), Python double."""
    return max(float(amax), 1e-12) / (FP4_MAX * E4M3_MAX)


def dynamic_act_global(amax: float) -> float:
    """tfimage/linear.py:127 -- a = max(amax(x), 1e-6) / (6*448), Python double."""
    return max(float(amax), 1e-6) / (FP4_MAX * E4M3_MAX)


# ------------------------------------------------------------------------------------------- quantize / decode
def quantize(x, g: float) -> tuple[np.ndarray, np.ndarray]:
    """x [M, K] (fp32 values; bf16 inputs are exact in fp32) -> (codes uint8 [M, K/2], scales uint8 [M, K/16]).

    The rounding statement is in the module docstring. Codes pack two elements per byte, the even element in the
    low nibble (tools/gemm_tf.py:23)."""
    x = np.asarray(x, dtype=np.float32)
    M, K = x.shape
    assert K % 16 == 0, "K must be a multiple of 16"
    g32 = np.float32(g)
    inv6g = np.float32(1.0) / (np.float32(6.0) * g32)
    blk = x.reshape(M, K // 16, 16)
    amax = np.abs(blk).max(axis=2)
    sf = e4m3_encode((amax * inv6g).astype(np.float32))
    d = (e4m3_decode(sf) * g32).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1.0) / np.where(d == 0, np.float32(1), d)).astype(np.float32)
    v = (blk * inv[..., None]).astype(np.float32)
    c = e2m1_encode(v)
    packed = (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)
    return packed.reshape(M, K // 2), sf


def dequantize(codes, scales, g: float) -> np.ndarray:
    """(codes [M, K/2], e4m3 scale bytes [M, K/16], global) -> fp32 [M, K]; tools/gemm_tf.py:21-24."""
    codes = np.asarray(codes, dtype=np.uint8)
    M = codes.shape[0]
    c = np.stack([codes & 15, codes >> 4], -1).reshape(M, -1)
    s = np.repeat(e4m3_decode(scales), 16, axis=1)
    return (E2M1_LUT[c] * s * np.float32(g)).astype(np.float32)


# ------------------------------------------------------------------------------------------- GEMM scale layout
def sf_tile(sf_rows, rows_pad: int | None = None) -> np.ndarray:
    """Row-major scales [R, K/16] -> the GEMM layout: 512-byte chunks [ceil(R/128)][K/64][512].

    Inside a chunk (128 rows x 4 scales, i.e. 64 K-elements) row r, scale j sits at ``(r % 32) * 16 +
    (r // 32) * 4 + j``: the layout tcgen05.cp.32x128b.warpx4 moves into TMEM for block-scaled MMA. Rows past R
    are zero."""
    sf_rows = np.asarray(sf_rows, dtype=np.uint8)
    R, KS = sf_rows.shape
    assert KS % 4 == 0, "K must be a multiple of 64"
    Rp = rows_pad if rows_pad is not None else -(-R // 128) * 128
    buf = np.zeros((Rp, KS), dtype=np.uint8)
    buf[:R] = sf_rows
    return np.ascontiguousarray(buf.reshape(Rp // 128, 4, 32, KS // 4, 4).transpose(0, 3, 2, 1, 4)).reshape(-1)


def sf_untile(tiled, R: int, K: int) -> np.ndarray:
    KS = K // 16
    Rp = -(-R // 128) * 128
    t = np.asarray(tiled, dtype=np.uint8).reshape(Rp // 128, KS // 4, 32, 4, 4).transpose(0, 3, 2, 1, 4)
    return np.ascontiguousarray(t.reshape(Rp, KS)[:R])


# ---------------------------------------------------------------------------------------------- reference GEMMs
def gemm(a_codes, a_sf, ga: float, b_codes, b_sf, gb: float, acc: str = "f32") -> np.ndarray:
    """The reference's CPU path: dequantize both operands, fp32 matmul (tools/gemm_tf.py:43-44) -> fp32 [M, N].

    ``acc="f64"`` (a measuring aid, not the reference): the same products summed in float64, i.e. the exact result
    up to float64 rounding -- the reference's fp32 result and any other fp32 summation order scatter around it."""
    if acc == "f64":
        A = dequantize(a_codes, a_sf, 1.0).astype(np.float64) * float(ga)
        B = dequantize(b_codes, b_sf, 1.0).astype(np.float64) * float(gb)
        return (A @ B.T).astype(np.float32)
    A = dequantize(a_codes, a_sf, ga)
    B = dequantize(b_codes, b_sf, gb)
    return A @ B.T


def linear(x, b_codes, b_sf, gb: float, act: float, acc: str = "f32") -> np.ndarray:
    """Nvfp4Linear.__call__ (tfimage/linear.py:125-130): quantize x under ``act``, W4A4 GEMM, bf16 output."""
    ac, asf = quantize(x, act)
    return bf16_round(gemm(ac, asf, act, b_codes, b_sf, gb, acc))
