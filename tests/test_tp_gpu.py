"""Tensor-parallel MLP on 2 GPUs over NCCL (skipped with fewer GPUs): tfimage.tp.TPMLP at the configs[1] MLP shape
against the unsharded fused pair on the same rank. The partials are reduced in bf16, so the bound is the bf16
rounding of two partial sums (measured on the CPU restatement: ~3e-3)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    from _helpers import bf16_cpu, f32, rel_l2
    from tfimage import linear as L
    from tfimage import tp

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        M, K, F = 4352, 3072, 8192
        x = bf16_cpu((M, K), seed=81).to(dev)
        gu = L.Nvfp4Linear(bf16_cpu((2 * F, K), seed=82, scale=0.02).to(dev), act=float(x.float().abs().max()) / 2688)
        down = L.Nvfp4Linear(bf16_cpu((K, F), seed=83, scale=0.02).to(dev), act=0.0008)
        ref = L.swiglu_mlp(gu, down, x)
        y = tp.TPMLP(gu, down)(x)
        res = bf16_cpu((M, K), seed=84, scale=3.0).to(dev)
        gate = bf16_cpu((1, K), seed=85, scale=0.5).to(dev)
        out = tp.TPMLP(gu, down)(x, residual=(res.clone(), gate))
        torch.cuda.synchronize()
        err = rel_l2(f32(y), f32(ref))
        err_res = rel_l2(f32(out), f32(res.clone().addcmul_(ref, gate)))
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as fh:
            fh.write(f"{err:.3e} {err_res:.3e}\n")
    finally:
        dist.destroy_process_group()


def test_tp_mlp_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        err, err_res = map(float, (tmp_path / f"rank{r}.txt").read_text().split())
        print(f"rank {r}: TP vs unsharded rel-L2 {err:.2e}, with residual {err_res:.2e}")
        assert err <= 5e-3 and err_res <= 2e-3
