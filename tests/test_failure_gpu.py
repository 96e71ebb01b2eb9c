"""Failure detection on the GPU without a GPU fault: a bounded device wait that nothing will ever satisfy runs out,
the kernel records TFB_DEVICE_TIMEOUT in the library's error word and returns, the host reads the status, and the
context stays usable for the next launch.

The wait is tfb_tp_wait's: it holds the stream until every other rank of a tensor-parallel group has stored its x
rows of the current call into this rank's buffer, counted by per-tile counters. Here the "group" is two buffers on
one GPU with no second rank behind the other one, so the counters stay zero and every wait runs to its 1 s limit
(the library's bound on any pipeline or peer wait)."""

import ctypes
import time

import numpy as np
import pytest
import torch
from _helpers import bf16_cpu, f32, quant_weight, rel_l2

from oracle import nvfp4 as onv
from tfimage import _lib

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_the_context_recovers(dev):
    world, M, N = 2, 1024, 256              # rank 1's chunk holds M / 2 rows: two tiles whose x rows never arrive
    nbytes, _ = _lib.tp_layout(world, M, N)
    own = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    silent = torch.zeros(nbytes, dtype=torch.uint8, device=dev)     # stands in for a rank that never signals
    base = (ctypes.c_void_p * _lib.TP_MAX_WORLD)(own.data_ptr(), silent.data_ptr())
    comm = _lib.TpComm(world, 0, base, M, N)
    assert _lib.device_status(reset=True) == 0
    t0 = time.perf_counter()
    _lib.tp_wait(comm, M, N, 1, dev)        # epoch 1: the other chunk's x counters would have to reach 2
    code = _lib.device_status(reset=True)   # synchronizes, reads and clears the error word
    waited = time.perf_counter() - t0
    assert code == 0x304, hex(code)         # the peer-x wait of tfb_tp_wait ran out
    assert 0.5 < waited < 20.0, waited      # ended by the 1 s limit, not by a hang
    assert _lib.device_status(reset=False) == 0
    # the context is intact: a normal NVFP4 GEMM right after matches the oracle
    Mg, Ng, Kg = 256, 256, 256
    x = bf16_cpu((Mg, Kg), seed=5)
    w = bf16_cpu((Ng, Kg), seed=6, scale=0.02)
    wc, ws, gw = quant_weight(w)
    ga = onv.dynamic_act_global(float(x.float().abs().max()))
    xc, xs = onv.quantize(x.float().numpy(), ga)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)   # noqa: E731
    y = _lib.gemm_nvfp4(t(xc), t(onv.sf_tile(xs)), t(wc), t(onv.sf_tile(ws)), Mg, Ng, Kg, ga * gw)
    ref = onv.bf16_round(onv.gemm(xc, xs, ga, wc, ws, gw))
    assert rel_l2(f32(y), ref) <= 2e-3
    assert _lib.device_status(reset=False) == 0
