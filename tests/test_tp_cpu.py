"""Tensor-parallel MLP host logic on the CPU: world sizes 2 and 4 over gloo, each rank running the oracle on its shard
(tfimage.tp's shards of the weight containers), the partial outputs all-reduced. Checks that a rank's NVFP4 SwiGLU
codes / scales are exactly the corresponding columns of the unsharded ones and that the reduced output equals the
unsharded oracle up to the bf16 rounding of the partials."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fusions as ofu
from oracle import nvfp4 as onv
from tfimage import linear as L
from tfimage import tp

M, K, F, D = 96, 256, 512, 256


def _weights():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(M, K, generator=g)).to(torch.bfloat16).float().numpy()
    wgu = (torch.randn(2 * F, K, generator=g) * 0.05).to(torch.bfloat16).float().numpy()
    wd = (torch.randn(D, F, generator=g) * 0.05).to(torch.bfloat16).float().numpy()
    act_x = onv.dynamic_act_global(float(np.abs(x).max()))
    gc, gs = onv.quantize(wgu, g_gu := onv.weight_global(np.abs(wgu).max()))
    dc, ds = onv.quantize(wd, g_d := onv.weight_global(np.abs(wd).max()))
    return x, act_x, (gc, gs, g_gu), (dc, ds, g_d)


def _container(c, s, g, act):
    return L.Fp4Linear.from_checkpoint(torch.from_numpy(c), torch.from_numpy(s), g, act)


def _mlp(x, act_x, gu: L.Fp4Linear, dn: L.Fp4Linear, act_h):
    u8 = lambda t: t.view(torch.uint8).numpy()            # noqa: E731
    gate_up = onv.linear(x, u8(gu.codes), u8(gu.scales()), gu.scale, act_x)
    h = ofu.swiglu(gate_up)
    hc, hs = onv.quantize(h, act_h)
    y = onv.bf16_round(onv.gemm(hc, hs, act_h, u8(dn.codes), u8(dn.scales()), dn.scale))
    return y, hc, hs


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, act_x, (gc, gs, g_gu), (dc, ds, g_d) = _weights()
        gu, dn = _container(gc, gs, g_gu, act_x), _container(dc, ds, g_d, 1.0)
        # down's static input scale: 4 x the amax of the unsharded SwiGLU output (calibrate.py's margin)
        h_full = ofu.swiglu(onv.linear(x, gc, gs, g_gu, act_x))
        act_h = 4 * float(np.abs(h_full).max()) / (6 * 448)
        y_full, hc_full, hs_full = _mlp(x, act_x, gu, dn, act_h)
        y_part, hc, hs = _mlp(x, act_x, tp.shard_gate_up(gu, rank, world), tp.shard_down(dn, rank, world), act_h)
        f = F // world
        assert np.array_equal(hc, hc_full[:, rank * f // 2:(rank + 1) * f // 2]), "h codes differ from unsharded"
        assert np.array_equal(hs, hs_full[:, rank * f // 16:(rank + 1) * f // 16]), "h scales differ from unsharded"
        t = torch.from_numpy(y_part.astype(np.float32))
        dist.all_reduce(t)
        y = onv.bf16_round(t.numpy())
        err = float(np.linalg.norm(y - y_full) / np.linalg.norm(y_full))
        assert err <= 4e-3, err
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as fh:
            fh.write(f"{err:.3e}\n")
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_mlp_shards_over_gloo(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    errs = [float((tmp_path / f"rank{r}.txt").read_text()) for r in range(world)]
    assert len(errs) == world and max(errs) <= 4e-3


def test_shards_reassemble_the_unsharded_containers():
    x, act_x, (gc, gs, g_gu), (dc, ds, g_d) = _weights()
    gu, dn = _container(gc, gs, g_gu, act_x), _container(dc, ds, g_d, 1.0)
    for world in (2, 4):
        sh = [tp.shard_gate_up(gu, r, world) for r in range(world)]
        f = F // world
        gate = torch.cat([s.codes[:f] for s in sh])
        up = torch.cat([s.codes[f:] for s in sh])
        assert torch.equal(torch.cat([gate, up]), gu.codes)
        ds_ = [tp.shard_down(dn, r, world) for r in range(world)]
        assert torch.equal(torch.cat([s.codes for s in ds_], 1), dn.codes)
        assert torch.equal(torch.cat([s.scales().view(torch.uint8) for s in ds_], 1), dn.scales().view(torch.uint8))


def test_p2p_comm_refuses_a_one_rank_group(tmp_path):
    """A peer-memory communicator needs 2 to 8 ranks (TFB_TP_MAX_WORLD): a 1-rank group is refused before any buffer
    is made (no GPU involved)."""
    import socket

    import torch.distributed as dist

    from tfimage import tp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="2 to 8 ranks"):
            tp.P2PComm(4096, 3072)
    finally:
        dist.destroy_process_group()
