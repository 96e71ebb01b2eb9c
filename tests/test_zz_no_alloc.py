"""tfb_mlp_nvfp4_static -- the fused NVFP4 MLP pair on the library's static per-device scratch, which allocates no
device memory -- against tfb_mlp_nvfp4 with a caller-owned workspace. Both are called through the C ABI (ctypes),
twice in a row, on the same inputs. The file name keeps it last in collection, so it also runs after every other
GPU test has used the library."""

import ctypes

import pytest
import torch
from _helpers import bf16_cpu, f32, rel_l2

from tfimage import _lib

pytestmark = pytest.mark.gpu


def _case(dev, M, K, F, seed):
    x = bf16_cpu((M, K), seed=seed).to(dev)
    wgu = bf16_cpu((2 * F, K), seed=seed + 1, scale=0.02).to(dev)
    wd = bf16_cpu((K, F), seed=seed + 2, scale=0.02).to(dev)
    g_gu = float(wgu.float().abs().max()) / (6 * 448)
    g_d = float(wd.float().abs().max()) / (6 * 448)
    guc, gus = _lib.quant_nvfp4(wgu, g_gu)          # tiled scales, the GEMM layout
    dc, ds = _lib.quant_nvfp4(wd, g_d)
    act_x = float(x.float().abs().max()) / (6 * 448)
    act_h = 0.004
    return x, guc, gus, g_gu, dc, ds, g_d, act_x, act_h


def _call(name, args, ws=()):
    lib = _lib.load()
    x, guc, gus, g_gu, dc, ds, g_d, act_x, act_h, y, stream = args
    M, K = x.shape
    F = guc.shape[0] // 2
    common = (x.data_ptr(), M, K, F, act_x, guc.data_ptr(), gus.data_ptr(), g_gu, dc.data_ptr(), ds.data_ptr(), g_d,
              act_h, y.data_ptr())
    st = getattr(lib, name)(*common, *[w.data_ptr() for w in ws], stream)
    assert st == 0, f"{name}: status {st}: {lib.tfb_last_error().decode()}"


@pytest.mark.parametrize("M,K,F", [(300, 512, 384), (4352, 3072, 8192)])
def test_static_scratch_mlp_matches_workspace_entry_point(dev, M, K, F):
    x, guc, gus, g_gu, dc, ds, g_d, act_x, act_h = _case(dev, M, K, F, seed=M + K)
    stream = torch.cuda.current_stream().cuda_stream
    y_ws = torch.empty((M, K), dtype=torch.bfloat16, device=dev)
    ws = _lib.mlp_workspace(M, K, F, dev)
    _call("tfb_mlp_nvfp4", (x, guc, gus, g_gu, dc, ds, g_d, act_x, act_h, y_ws, stream), ws)
    outs = []
    for _ in range(2):                                   # two calls in a row on the same scratch
        y = torch.full((M, K), float("nan"), dtype=torch.bfloat16, device=dev)
        _call("tfb_mlp_nvfp4_static", (x, guc, gus, g_gu, dc, ds, g_d, act_x, act_h, y, stream))
        outs.append(y)
    torch.cuda.synchronize()
    ref = f32(y_ws)
    assert torch.isfinite(y_ws.float()).all()
    for i, y in enumerate(outs):
        # Same three kernels, same inputs, same stream: only the scratch location differs, so the outputs must be
        # bit-identical (a scale block read from a neighbouring scratch region would show up here). The rel-L2 is
        # reported only to size a failure.
        assert torch.equal(y, y_ws), f"call {i}: differs from the workspace entry point (rel-L2 {rel_l2(f32(y), ref):.3e})"


def test_static_scratch_rejects_oversized_calls(dev):
    lib = _lib.load()
    M, K, F = 8192, 3072, 8192                           # 53.5 MB of scratch > the 32 MiB array
    st = lib.tfb_mlp_nvfp4_static(None, M, K, F, 1.0, None, None, 1.0, None, None, 1.0, 1.0, None, None)
    assert _lib.STATUS[st] == "BAD_SHAPE"
    msg = lib.tfb_last_error().decode()
    assert "scratch" in msg and str(_lib.MLP_STATIC_SCRATCH_BYTES) in msg
    assert ctypes.sizeof(ctypes.c_void_p) == 8
