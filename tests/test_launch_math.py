"""Index arithmetic of two launches, restated on the CPU (no GPU involved).

* The qkv GEMM's RMS-RoPE epilogue (`csrc/gemm.cu`, MODE_FP4_QKV) loads each warp's cos / sin rows with no row
  guard. For every row block of the tile grid, CTA of a pair and warp quadrant, the 32 token indices n0 + r that a
  warp reads must stay inside the [ntok, 64] table, and for the rows inside M they must be the rows' own tokens.
  This holds because ntok % 32 == 0, which `tfb_gemm_nvfp4_qkv` requires.
* The RMS-RoPE kernels (`csrc/fusions.cu`) give each half-warp UPT units, hw + k * span (span = the grid's
  half-warps). Every unit of a launch must be taken exactly once.
"""

import numpy as np
import pytest

BM = 128            # rows of one CTA's tile (gemm.cu)


def qkv_warp_rows(B: int, ntok: int, cg: int):
    """(grow0, bb, n0) of every epilogue warp: gemm.cu's row0 = mb * BM * CG + rank * BM, grow0 = row0 + 32 q,
    bb = grow0 / ntok, n0 = grow0 - bb * ntok, over mb < ceil(M / (BM * CG))."""
    M = B * ntok
    num_m = -(-M // (BM * cg))
    for mb in range(num_m):
        for rank in range(cg):
            for q in range(4):
                grow0 = mb * BM * cg + rank * BM + q * 32
                bb = grow0 // ntok
                yield grow0, bb, grow0 - bb * ntok


@pytest.mark.parametrize("B,ntok", [(1, 4096), (1, 256), (2, 4352), (3, 96), (1, 32), (5, 4128), (7, 160)])
@pytest.mark.parametrize("cg", [1, 2])
def test_qkv_epilogue_cos_rows_in_table(B, ntok, cg):
    M = B * ntok
    r = np.arange(32)                                     # (g4 * 4 + u) * 4 + lane / 8 over g4, u, lane
    passes = ((np.arange(2)[:, None, None] * 4 + np.arange(4)[None, :, None]) * 4
              + (np.arange(32)[None, None, :] >> 3)).ravel()
    assert set(passes.tolist()) == set(r.tolist())
    jj = (np.arange(2)[:, None] * 8 + np.arange(8)[None, :]).ravel()
    assert jj.max() * 4 + 3 < 64                          # the float4 column offsets stay inside a table row
    for grow0, bb, n0 in qkv_warp_rows(B, ntok, cg):
        tok = n0 + r
        assert tok.min() >= 0 and tok.max() < ntok, (grow0, n0)
        live = grow0 + r < M
        rows = grow0 + r[live]
        assert np.all(rows // ntok == bb) and np.all(rows % ntok == tok[live])


@pytest.mark.parametrize("units", [1, 15, 16, 17, 255, 256, 257, 4096 * 24, 4352 * 24 + 7])
@pytest.mark.parametrize("upt", [1, 2, 4])
def test_rms_rope_units_taken_once(units, upt):
    threads = -(-units // upt) * 16                       # the launchers' thread count
    grid = -(-threads // 256)
    span = grid * (256 // 16)                             # half-warps in the grid
    u = np.arange(span)[:, None] + np.arange(upt)[None, :] * span
    u = u[u < units]
    assert np.array_equal(np.bincount(u, minlength=units), np.ones(units, dtype=np.int64))
