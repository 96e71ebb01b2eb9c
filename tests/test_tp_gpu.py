"""Tensor-parallel MLP over the GPUs of the box -- 2, 4 or 8 ranks, the largest power of two available (skipped with
fewer than 2): tfimage.tp.TPMLP at the configs[1] MLP shape against the unsharded fused pair on the same rank, and the
down GEMM with the reduction fused in (peer memory) against the NCCL path and against the partials summed in rank
order. NCCL reduces the bf16 partials in bf16, so against one GPU the bound is the bf16 rounding of the partial sums
(measured on the CPU restatement: ~3e-3 for two ranks; it grows with the number of partials)."""

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

    # NVLS off: a rank that fails mid-test must not leave an NVLink multicast object bound on the others' GPUs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
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


def _world():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return 8 if n >= 8 else 4 if n >= 4 else 2 if n >= 2 else 0


def test_tp_mlp_gpus(tmp_path):
    world = _world()
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        err, err_res = map(float, (tmp_path / f"rank{r}.txt").read_text().split())
        print(f"rank {r} of {world}: TP vs unsharded rel-L2 {err:.2e}, with residual {err_res:.2e}")
        assert err <= (5e-3 if world == 2 else 1e-2) and err_res <= (2e-3 if world == 2 else 4e-3)


def _p2p_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    from _helpers import bf16_cpu, f32, rel_l2
    from tfimage import _lib
    from tfimage import linear as L
    from tfimage import mmdit, tp

    # NVLS off: a rank that fails mid-test must not leave an NVLink multicast object bound on the others' GPUs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    lines = []
    try:
        M, K, F = 4096, 3072, 8192
        x = bf16_cpu((M, K), seed=91).to(dev)
        gu = L.Nvfp4Linear(bf16_cpu((2 * F, K), seed=92, scale=0.02).to(dev), act=float(x.float().abs().max()) / 2688)
        down = L.Nvfp4Linear(bf16_cpu((K, F), seed=93, scale=0.02).to(dev), act=0.0008)
        comm = tp.P2PComm(M, K)
        fused, nccl = tp.TPMLP(gu, down, comm=comm), tp.TPMLP(gu, down)
        ref_full = L.swiglu_mlp(gu, down, x)
        for step in range(3):                       # three calls on one buffer: epochs 1, 2, 3
            res = bf16_cpu((M, K), seed=94 + step, scale=3.0).to(dev)
            gate = bf16_cpu((1, K), seed=97 + step, scale=0.5).to(dev)
            xs = comm.x(M)
            xs.copy_(res)
            fused(x, residual=(xs, gate))
            want = nccl(x, residual=(res.clone(), gate))
            # the fused reduction's arithmetic: the ranks' bf16 partials summed in fp32 in rank order, then bf16
            part = L.swiglu_mlp(nccl.gate_up, nccl.down, x)
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            acc = torch.zeros(part.shape, dtype=torch.float32, device=dev)
            for pr in parts:
                acc += pr.float()
            want_order = res.clone().addcmul_(acc.to(torch.bfloat16), gate)
            torch.cuda.synchronize()
            same = bool(torch.equal(xs, want))
            same_order = bool(torch.equal(xs, want_order))
            err = rel_l2(f32(xs), f32(res.clone().addcmul_(ref_full, gate)))
            # every rank holds the same x
            peer = [torch.empty_like(xs) for _ in range(world)]
            dist.all_gather(peer, xs.clone())
            agree = all(torch.equal(peer[0], p) for p in peer)
            lines.append(f"mlp {int(same)} {int(same_order)} {int(agree)} {err:.3e}")
        assert _lib.device_status() == 0
        comm.close()

        # the DiT step with the MLP split over the ranks: peer-memory reduction == NCCL all-reduce, bit for bit
        cfg = mmdit.DitConfig(layers=2)
        m = mmdit.SynthMMDiT(cfg, device=dev, seed=5)
        g = torch.Generator().manual_seed(6)
        ctx = torch.randn((1, 64, cfg.txt_dim), generator=g).to(dev)
        noise = torch.randn((1, 64, 32, 32), generator=g).to(dev)
        m.calibrate(ctx, noise, steps=1)
        prefix = m.build_prefix(ctx)
        xb = noise.to(torch.bfloat16)
        t = torch.full((1,), 0.6, device=dev)
        single = m.forward(xb, t, prefix, {}).clone()
        m.enable_tp()
        via_nccl = m.forward(xb, t, prefix, {}).clone()
        m.disable_tp()
        m.enable_tp(p2p=True)
        via_p2p = [m.forward(xb, t, prefix, {}).clone() for _ in range(2)]
        via_graph = [m.step_graph(xb, t, prefix).clone() for _ in range(3)]   # capture, then two replays
        m.disable_tp()
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        lines.append(f"dit {int(torch.equal(via_p2p[0], via_nccl))} {int(torch.equal(via_p2p[1], via_p2p[0]))} "
                     f"{rel_l2(f32(via_p2p[0]), f32(single)):.3e} {rel_l2(f32(via_p2p[0]), f32(via_nccl)):.3e}")
        lines.append(f"graph {int(all(torch.equal(g, via_p2p[0]) for g in via_graph))}")
        with open(os.path.join(out_dir, f"p2p{rank}.txt"), "w") as fh:
            fh.write("\n".join(lines) + "\n")
    finally:
        dist.destroy_process_group()


def test_tp_mlp_peer_memory_gpus(tmp_path):
    """The down GEMM with the cross-GPU reduction fused in (tfb_gemm_nvfp4_tp over CUDA IPC peer memory): identical x
    on every rank over repeated calls on one buffer, bit-equal to the partials summed in fp32 in rank order (the
    kernel's arithmetic) plus torch's addcmul_, and -- with two ranks, where that sum is exactly NCCL's -- bit-equal
    to NCCL's bf16 all-reduce + gated residual; the DiT step with the MLP split that way, eager and replayed from a
    captured CUDA graph (bit-equal to each other; with two ranks also to the NCCL-split step)."""
    world = _world()
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_p2p_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        text = (tmp_path / f"p2p{r}.txt").read_text()
        print(f"rank {r} of {world}:\n{text}")
        for line in text.split("\n"):
            if line.startswith("mlp"):
                _, same, same_order, agree, err = line.split()
                assert same_order == "1" and agree == "1" and float(err) <= (2e-3 if world == 2 else 4e-3)
                assert same == "1" or world > 2      # NCCL sums more than two partials in its own order
            elif line.startswith("graph"):
                assert line.split()[1] == "1"        # replayed CUDA graphs of the split step (device epochs)
            elif line.startswith("dit"):
                _, a, b, err, err_nccl = line.split()
                # against one GPU the split step differs by the bf16 rounding of the partials, which the next blocks'
                # NVFP4 requantization amplifies (measured 4.8e-2 with two ranks on this 2-block random-weight model,
                # for the NCCL split as well)
                assert b == "1" and float(err) <= 1e-1 and float(err_nccl) <= 1e-1
                assert a == "1" or world > 2
