"""Benchmark of the NVFP4 quantized-linear hot path on B200 (the fused MLP pair).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = ``tfimage.linear.swiglu_mlp`` on one image's rows: quantize X [4352, 3072] under the gate/up input
scale, gate/up NVFP4 GEMM [16384, 3072] whose epilogue applies SwiGLU and writes NVFP4 rows, down NVFP4 GEMM
[3072, 8192] -> bf16 [4352, 3072]; 657.13 GFLOP. Inputs are resident in HBM; L2 is flushed (a 256 MiB write, then a read of it)
between steps, outside the per-step CUDA events. Under torchrun every rank runs its own image (independent seeds,
no collective: weak scaling) and the result is whole-job TFLOP/s over the max per-rank time.

``e2e`` runs the same public call with the step's input copied from pinned host memory and its output copied back
inside the timed region. ``cpu_baseline`` (rank 0, N=1) and ``--impl reference`` time the reference's torch CPU
path -- oracle quantize, dequantize, fp32 matmul -- restated in ``oracle/`` on a bounded row sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "qwen-image21-tensorfold-rtx_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "NVFP4 linear TFLOP/s (% FP4 peak); DiT step ms @4096 tok; img/s at 1-8 GPU"
M_ROWS, K_DIM, F_DIM = 4352, 3072, 8192
FLOP_GU = 2 * M_ROWS * K_DIM * 2 * F_DIM          # 438.09 GFLOP
FLOP_DOWN = 2 * M_ROWS * F_DIM * K_DIM            # 219.04 GFLOP
FLOP_STEP = FLOP_GU + FLOP_DOWN
# Nominal dense tensor peaks of one B200 (MEASURED_PEAKS.json carries HBM and bf16 figures only, so the FP4 / FP8
# fractions are against these nominal numbers).
FP4_NOMINAL_TFLOPS, FP8_NOMINAL_TFLOPS = 9000.0, 4500.0
# DRAM bytes per gate/up launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of this launch
# (35.89 MB read + 1.70 MB written: 1.05 x its 35.8 MB of algorithmic operand bytes).
TRAFFIC_GU = 37.59e6
WORKLOAD = ("configs[1] fused NVFP4 MLP pair: X bf16 [4352,3072] N(0,1) -> gate/up W [16384,3072] N(0,0.02) with "
            "SwiGLU->NVFP4 epilogue -> down W [3072,8192] N(0,0.02) -> bf16 [4352,3072]")


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, \
            "fallback"


# ------------------------------------------------------------------------------------------------ clock sampling
REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """NVML SM clock + throttle reasons on a background thread: one sample when the region opens, one every ~1 ms,
    one when it closes (a timed region of a few ms still gets several)."""

    def __init__(self, index: int):
        self.index, self.samples, self.reasons, self.max_mhz = index, [], 0, None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:                                   # noqa: BLE001 -- no NVML: report no clocks
            self.nv = None

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:                                   # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.001)

    def __enter__(self):
        if self.nv is not None:
            self._sample()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()
            self._sample()

    def report(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        names = [n for b, n in REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------ CPU baseline
def cpu_reference_setup(seed: int = 0):
    """The reference's CPU path: oracle-quantized weights, dequantized once (a weight cache), as fp32 torch."""
    import numpy as np
    import torch

    from oracle import nvfp4 as onv

    g = torch.Generator().manual_seed(seed)
    wgu = (torch.randn(2 * F_DIM, K_DIM, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    wd = (torch.randn(K_DIM, F_DIM, generator=g) * 0.02).to(torch.bfloat16).float().numpy()
    out = {}
    for name, w in (("gu", wgu), ("down", wd)):
        gw = onv.weight_global(np.abs(w).max())
        c, s = onv.quantize(w, gw)
        out[name] = torch.from_numpy(onv.dequantize(c, s, gw))
    x = torch.randn(M_ROWS, K_DIM, generator=g).to(torch.bfloat16).float().numpy()
    out["x"] = x
    out["act_x"] = onv.dynamic_act_global(np.abs(x).max())
    return out


def cpu_reference_step(st, rows: int, row0: int = 0):
    """quantize+dequantize X rows -> fp32 matmul gate/up -> bf16 -> SwiGLU -> quantize+dequantize under down.act ->
    fp32 matmul down -> bf16 (tools/gemm_tf.py:21-24,43; kernels.py:80)."""
    import numpy as np
    import torch

    from oracle import fusions as ofu
    from oracle import nvfp4 as onv

    xs = st["x"][row0:row0 + rows]
    xd = torch.from_numpy(onv.dequantize(*onv.quantize(xs, st["act_x"]), st["act_x"]))
    gu = onv.bf16_round((xd @ st["gu"].T).numpy())
    h = ofu.swiglu(gu)
    act_h = st.setdefault("act_h", 4 * float(np.abs(h).max()) / (6 * 448))
    hd = torch.from_numpy(onv.dequantize(*onv.quantize(h, act_h), act_h))
    return onv.bf16_round((hd @ st["down"].T).numpy())


def cpu_baseline(budget_s: float = 10.0, rows: int = 64):
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    st = cpu_reference_setup()
    cpu_reference_step(st, rows)                                      # warm-up, sets act_h
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_reference_step(st, rows, row0=(n * rows) % (M_ROWS - rows))
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    flop = FLOP_STEP * rows / M_ROWS
    return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{rows} of the {M_ROWS} rows per step, {n} steps over {budget_s:.0f} s: oracle NVFP4 "
                      f"quantize+dequantize, torch fp32 matmul, SwiGLU, requantize, fp32 matmul (weights "
                      f"dequantized once outside the timing)"}


def cpu_baseline_fusions(budget_s: float = 4.0, rows: int = 256) -> dict:
    """configs[2] on the host cores: the reference's fusions as restated in oracle/ (AdaLN + shift -> bf16 -> NVFP4
    codes + scales; RMSNorm + RoPE of q and k from a qkv row block), on ``rows`` rows per call, reported as GB/s of
    the same algorithmic bytes per row as the GPU legs."""
    import numpy as np
    import torch

    from oracle import fusions as ofu
    from oracle import nvfp4 as onv

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(23)
    D, H, Dh = 3072, 24, 128
    x = onv.bf16_round(rng.standard_normal((1, rows, D)).astype(np.float32))
    sc = (rng.standard_normal((1, 1, D)) * 0.1).astype(np.float32)
    sh = (rng.standard_normal((1, 1, D)) * 0.1).astype(np.float32)
    qkv = onv.bf16_round(rng.standard_normal((1, rows, 3, H, Dh)).astype(np.float32))
    w = (rng.standard_normal(Dh) * 0.05 + 1).astype(np.float32)
    ang = rng.uniform(0, 6.3, (rows, Dh // 2)).astype(np.float32)
    cos, sin = np.cos(ang), np.sin(ang)

    def run(fn):
        fn()
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s / 2:
            fn()
            n += 1
        return (time.perf_counter() - t0) / n

    t_ada = run(lambda: onv.quantize(ofu.adaln(x, sc, 1e-6, shift=sh).reshape(rows, D), 0.004))
    t_rope = run(lambda: (ofu.rms_rope(qkv, 0, w, cos, sin, 1e-6), ofu.rms_rope(qkv, 1, w, cos, sin, 1e-6)))
    ada_bytes = rows * (D * 2 + D // 2 + D // 16)
    rope_bytes = rows * (4 * H * Dh * 2 + 2 * 64 * 8)
    return {"adaln_quant_gbs": ada_bytes / t_ada / 1e9, "rms_rope_q_k_gbs": rope_bytes / t_rope / 1e9,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{rows} rows per call (numpy restatement of kernels.py:14-70 + the NVFP4 quantizer)"}


def cpu_baseline_linears(budget_s: float = 4.0, rows: int = 128) -> dict:
    """configs[0] and configs[3] on the host cores: the reference's CPU linear paths as restated in oracle/ -- NVFP4
    (quantize + dequantize the X rows under the dynamic global, fp32 matmul against the dequantized weight, bf16;
    tools/gemm_tf.py:21-24) and FP8 W8A8 (per-tensor e4m3 activation, per-channel weight scales, fp32 matmul, bf16;
    tfimage/linear.py:86-100) -- on ``rows`` rows per call, weights quantized and dequantized once outside the timing,
    reported as TFLOP/s of those rows."""
    import numpy as np
    import torch

    from oracle import fp8 as ofp8
    from oracle import nvfp4 as onv

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(29)
    K = N = 3072
    x = rng.standard_normal((rows, K)).astype(np.float32)
    x[:, rng.permutation(K)[:8]] *= 20
    x = onv.bf16_round(x)
    w = onv.bf16_round((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    gw = onv.weight_global(float(np.abs(w).max()))
    wd = torch.from_numpy(onv.dequantize(*onv.quantize(w, gw), gw))
    w8, ws = ofp8.weight(w, per_channel=True)
    w8d = torch.from_numpy(onv.e4m3_decode(w8).astype(np.float32))

    def run(fn):
        fn()
        n, t0 = 0, time.perf_counter()
        while n == 0 or time.perf_counter() - t0 < budget_s / 2:
            fn()
            n += 1
        return (time.perf_counter() - t0) / n

    def nvfp4():
        ga = onv.dynamic_act_global(float(np.abs(x).max()))
        xd = torch.from_numpy(onv.dequantize(*onv.quantize(x, ga), ga))
        return onv.bf16_round((xd @ wd.T).numpy())

    def fp8():
        a = ofp8.act_scale(x)
        xq = torch.from_numpy(onv.e4m3_decode(ofp8.quantize(x, a)).astype(np.float32))
        return onv.bf16_round(((xq @ w8d.T) * (float(a) * torch.from_numpy(np.asarray(ws, np.float32)))).numpy())

    flop = 2 * rows * K * N
    return {"c0_nvfp4_tflops": flop / run(nvfp4) / 1e12, "c3_fp8_tflops": flop / run(fp8) / 1e12,
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{rows} of the 4096 (configs[0]) / 4968 (configs[3]) rows per call, [3072, 3072] weight"}


def _sdpa_cpu(q, k, v, causal=False):
    """The reference's attention op (torch SDPA) on the host cores in fp32, for the CPU block timing."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    from oracle import nvfp4 as onv

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).transpose(1, 2)   # noqa: E731
    o = F.scaled_dot_product_attention(t(q), t(k), t(v), is_causal=causal)
    return onv.bf16_round(o.transpose(1, 2).contiguous().numpy())


def cpu_baseline_dit(model, prefix, layers: int) -> dict:
    """configs[4] on the host cores: one image block of the step at full size (4096 image rows attending to the
    256-row kept prefix), the reference's CPU arithmetic as restated in oracle/dit.py (NVFP4 quantize -> dequantize
    -> fp32 matmul per linear, fusions, torch SDPA in fp32), with the model's own NVFP4 weights; the step estimate
    is that block's time x the number of blocks (every image block has the same shapes)."""
    import numpy as np
    import torch

    from oracle import dit as odit
    from tfimage import mmdit

    torch.set_num_threads(os.cpu_count() or 1)
    cfg, dev = model.cfg, model.device
    b = model.img_blocks[0]
    N = 64 * 64
    g = torch.Generator().manual_seed(41)
    x = torch.randn((1, N, cfg.dim), generator=g).to(torch.bfloat16).float().numpy()
    mod = [t.reshape(1, -1).float().cpu().numpy()
           for t in model._mod(model._temb(torch.tensor([0.5], device=dev)), model.mod_img)]
    cos, sin = mmdit.rope_table(mmdit.image_ids(64, 64, prefix.next_pos, dev), cfg)
    cos, sin = cos.cpu().numpy(), sin.cpu().numpy()
    kp, vp = (t.float().cpu().numpy() for t in prefix.kv[0])
    lin = {n: (getattr(b, n).lin.codes.cpu().numpy(), getattr(b, n).lin.scales().view(torch.uint8).cpu().numpy(),
               getattr(b, n).lin.scale, getattr(b, n).lin.act) for n in ("qkv", "out", "gate_up", "down")}
    nq, nk = b.norm_q.cpu().numpy(), b.norm_k.cpu().numpy()
    t0 = time.perf_counter()
    y = odit.block(x, mod, cos, sin, kp, vp, lin, nq, nk, cfg.heads, cfg.eps, attn=_sdpa_cpu)
    block_s = time.perf_counter() - t0
    return {"block_s": block_s, "step_s_estimate": block_s * layers, "img_per_s_estimate": 1.0 / (block_s * layers * 25),
            "cores": torch.get_num_threads(), "kind": "port", "finite": bool(np.isfinite(y).all()),
            "sample": f"one image block timed once ({N} rows + {prefix.length}-row prefix, weight dequantization "
                      f"included); step = {layers} x block, img/s = 1 / (25 steps x step)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    st = cpu_reference_setup()
    t0 = time.perf_counter()
    cpu_reference_step(st, 16)
    probe = max(time.perf_counter() - t0, 1e-3)
    per_row = probe / 16
    rows = int(max(8, min(M_ROWS // 2, (120.0 / max(args.steps + args.warmup, 1)) / per_row)))
    for i in range(args.warmup):
        cpu_reference_step(st, rows, row0=(i * rows) % (M_ROWS - rows))
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        cpu_reference_step(st, rows, row0=(i * rows) % (M_ROWS - rows))
        times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = FLOP_STEP * rows / M_ROWS / dt / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (dequantized nvfp4)", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows_per_step": rows, "M": M_ROWS, "K": K_DIM, "F": F_DIM},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"{rows} of {M_ROWS} rows per step (reference torch CPU dequant-matmul "
                                       f"path restated in oracle/)"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------- configs[0], [2], [3] legs
def l2_flush(buf) -> None:
    """Evict L2 before a timed run: write a buffer larger than L2 (126 MB), then read it back, so the lines left in
    L2 are clean -- after the write alone the timed kernel would first pay for writing ~126 MB of dirty flush data
    back to HBM (it showed up as a 2x slower first kernel of every step)."""
    buf.zero_()
    buf.sum()


def config_legs(dev, fp4_peak: float, fp8_peak: float, hbm_gbs: float) -> dict:
    """The other BASELINE configs measured beside the headline: each kernel timed alone with CUDA events on the
    launching stream, L2 flushed (256 MiB write, then a read of it) before every iteration, median of 20 after 3
    warm-up runs."""
    import numpy as np
    import torch

    from tfimage import _lib
    from tfimage import kernels as Kn
    from tfimage import linear as L
    from tfimage import mmdit

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, it=20):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(it):
            l2_flush(flush)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize(dev)
            ts.append(a.elapsed_time(b))
        return statistics.median(ts) * 1e3                         # us

    def act_input(m, k, seed):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(m, k, generator=g)
        x[:, torch.randperm(k, generator=g)[:8]] *= 20             # 8 outlier channels x20
        return x.to(torch.bfloat16).to(dev)

    out = {}
    # one NVFP4 W4A4 linear, X [4096, 3072], W [3072, 3072]
    M0, K0 = 4096, 3072
    x0 = act_input(M0, K0, 21)
    g = torch.Generator().manual_seed(22)
    lin = L.Nvfp4Linear((torch.randn(K0, K0, generator=g) * 0.02).to(torch.bfloat16).to(dev))
    lin.set_act(float(_lib.absmax(x0)) / (6 * 448))
    q0 = lin.quantize(x0)
    t_gemm, t_quant = timed(lambda: lin(q0)), timed(lambda: lin.quantize(x0))
    t_lin = timed(lambda: lin(x0))             # the reference call: bf16 X -> quantize -> GEMM -> bf16 Y, one stream
    # end to end from pinned host rows: X in, quantize + GEMM, Y out, one after the other on the stream
    x0_host = x0.cpu().pin_memory()
    y0_host = torch.empty((M0, K0), dtype=torch.bfloat16).pin_memory()
    x0_dev = torch.empty_like(x0)

    def e2e0():
        x0_dev.copy_(x0_host, non_blocking=True)
        y0_host.copy_(lin(x0_dev), non_blocking=True)
    t_e2e0 = timed(e2e0)
    flop0 = 2 * M0 * K0 * K0
    qbytes = M0 * K0 * 2 + M0 * K0 // 2 + M0 * K0 // 16
    out["configs[0]"] = {
        "workload": "NVFP4 W4A4 linear: X bf16 [4096, 3072] N(0,1), 8 channels x20; W [3072, 3072] N(0, 0.02)",
        "gemm_us": t_gemm, "gemm_tflops": flop0 / t_gemm / 1e6, "gemm_frac_fp4_peak": flop0 / t_gemm / 1e6 / fp4_peak,
        "quant_us": t_quant, "quant_gbs": qbytes / t_quant / 1e3, "quant_frac_hbm": qbytes / t_quant / 1e3 / hbm_gbs,
        "linear_us": t_lin, "linear_tflops": flop0 / t_lin / 1e6,
        "e2e": {"us": t_e2e0, "tflops": flop0 / t_e2e0 / 1e6, "h2d_bytes": M0 * K0 * 2, "d2h_bytes": M0 * K0 * 2,
                "path": "pinned X -> device copy, Nvfp4Linear (quantize + GEMM), bf16 Y -> pinned host copy, in order"}}
    del x0, lin, q0, x0_host, y0_host, x0_dev

    # AdaLN(+shift) + NVFP4 quantize on x [4352, 3072]; RMSNorm + RoPE of q, k (+ v) from qkv
    M2, D = 4352, 3072
    g = torch.Generator().manual_seed(23)
    x2 = torch.randn(1, M2, D, generator=g).to(torch.bfloat16).to(dev)
    sc = (torch.randn(1, 1, D, generator=g) * 0.1).to(dev)
    sh = (torch.randn(1, 1, D, generator=g) * 0.1).to(dev)
    t_ada = timed(lambda: Kn.adaln(x2, sc, 1e-6, shift=sh, quant=0.004))
    ada_bytes = M2 * D * 2 + M2 * D // 2 + M2 * D // 16
    H, Dh = 24, 128
    qkv = torch.randn(1, M2, 3, H, Dh, generator=g).to(torch.bfloat16).to(dev)
    wq = (torch.randn(Dh, generator=g) * 0.05 + 1).to(dev)
    wk = (torch.randn(Dh, generator=g) * 0.05 + 1).to(dev)
    cfg = mmdit.DitConfig()
    ids = torch.cat([mmdit.text_ids(256, dev), mmdit.image_ids(64, 64, 256, dev)])
    cos, sin = mmdit.rope_table(ids, cfg)
    q = torch.empty(1, M2, H, Dh, dtype=torch.bfloat16, device=dev)
    kb = torch.empty(1, M2 + 256, H, Dh, dtype=torch.bfloat16, device=dev)
    vb = torch.empty_like(kb)
    t_qkv = timed(lambda: Kn.rms_rope_qkv(qkv, wq, wk, cos, sin, 1e-6, q, kb[:, 256:], vb[:, 256:]))
    t_qk = timed(lambda: (Kn.rms_rope(qkv, 0, wq, cos, sin, 1e-6, q), Kn.rms_rope(qkv, 1, wk, cos, sin, 1e-6, kb[:, 256:])))
    plane = M2 * H * Dh * 2
    rope_bytes = M2 * 64 * 8
    out["configs[2]"] = {
        "workload": "AdaLN(+shift)+NVFP4 quantize on x bf16 [4352, 3072] N(0,1), shift/scale N(0, 0.1); RMSNorm(q, k) "
                    "+ 3-axis RoPE (16/56/56, 64x64 grid + 256 text ids) from qkv [4352, 3, 24, 128] N(0,1)",
        "adaln_quant_us": t_ada, "adaln_quant_gbs": ada_bytes / t_ada / 1e3,
        "adaln_quant_frac_hbm": ada_bytes / t_ada / 1e3 / hbm_gbs,
        "rms_rope_qkv_us": t_qkv, "rms_rope_qkv_gbs": (6 * plane + rope_bytes) / t_qkv / 1e3,
        "rms_rope_qkv_frac_hbm": (6 * plane + rope_bytes) / t_qkv / 1e3 / hbm_gbs,
        "rms_rope_q_k_us": t_qk, "rms_rope_q_k_gbs": (4 * plane + 2 * rope_bytes) / t_qk / 1e3,
        "bytes": {"adaln_quant": ada_bytes, "rms_rope_qkv": 6 * plane + rope_bytes,
                  "rms_rope_q_k": 4 * plane + 2 * rope_bytes}}
    del x2, qkv, q, kb, vb

    # FP8 W8A8, per-tensor activation scale, per-channel weight scales, ragged M = 4968
    M3 = 4968
    x3 = act_input(M3, 3072, 24)
    res = {"workload": "FP8 E4M3 W8A8, per-tensor act / per-channel W scales, M = 4968 (4712 image + 256 text)"}
    for name, n, k in (("linear_3072", 3072, 3072), ("gate_up_16384", 16384, 3072), ("down_3072_k8192", 3072, 8192)):
        g = torch.Generator().manual_seed(n + k)
        f8 = L.Fp8Linear((torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(dev), per_channel=True)
        xin = x3 if k == 3072 else act_input(M3, k, 25)
        a = _lib.fp8_act_scale(xin)
        q8 = _lib.quant_fp8(xin, a)
        t8 = timed(lambda: _lib.gemm_fp8(q8, f8.w8.view(torch.uint8), M3, n, k, a, f8.ws))
        fl = 2 * M3 * n * k
        res[name] = {"gemm_us": t8, "tflops": fl / t8 / 1e6, "frac_fp8_peak": fl / t8 / 1e6 / fp8_peak}
    out["configs[3]"] = res

    # GGUF block decode (the checkpoint loader's hot loop): one [16384, 3072] weight per quantized type -> bf16
    rows, cols = 16384, 3072
    res = {"workload": "GGUF Q8_0 / Q4_K / Q5_K / Q6_K weight [16384, 3072] (uniform random code bytes, block scales "
                       "fixed finite f16) decoded to bf16; bytes = raw blocks read + bf16 written"}
    gen = torch.Generator(device=dev).manual_seed(31)
    for kind, scale_cols in (("Q8_0", (0,)), ("Q4_K", (0, 2)), ("Q5_K", (0, 2)), ("Q6_K", (208,))):
        vals, nbytes = _lib.gguf_block(kind)
        raw = torch.randint(0, 256, (rows * cols // vals, nbytes), dtype=torch.uint8, device=dev, generator=gen)
        for c in scale_cols:
            raw[:, c], raw[:, c + 1] = 0x1C, 0x1C                 # f16 0x1C1C = 0.00412
        y = torch.empty(rows * cols, dtype=torch.bfloat16, device=dev)
        t = timed(lambda: _lib.gguf_dequant(kind, raw, y))
        nb = raw.numel() + 2 * y.numel()
        res[kind] = {"us": t, "gbs": nb / t / 1e3, "frac_hbm": nb / t / 1e3 / hbm_gbs, "bytes": nb}
        del raw, y
    out["gguf_decode"] = res
    out["peaks"] = {"fp4_tflops": fp4_peak, "fp8_tflops": fp8_peak, "hbm_gbs": hbm_gbs}
    del flush
    _ = np
    return out


# ------------------------------------------------------------------------------------------------- DiT leg
DIT_SEEDS, DIT_STEPS = 32, 25
DIT_WORKLOAD = ("configs[4] synthetic double-stream MMDiT, NVFP4: 28 blocks, hidden 3072, 24 x 128 heads, SwiGLU "
                "8192, separate image/text weights N(0, 0.02); latent [16, 128, 128] -> 4096 tokens; text [256, 3584] "
                "N(0, 1), K/V prefix-cached once per prompt; 25 Euler steps; 32 seeds split across ranks")


def dit_leg(world: int, rank: int, dev, barrier, reduce_max):
    """single-image DiT step latency at 4096 tokens, and images/s of the 25-step sampler over 32 seeds
    split across the ranks (each rank a full weight replica, no collective on the data path). Returns the numbers
    and (model, prefix, layers) for the CPU block timing."""
    import torch

    from tfimage import mmdit

    model = mmdit.SynthMMDiT(mmdit.DitConfig(), device=dev, seed=0)       # the same weights on every rank
    g = torch.Generator().manual_seed(4)
    ctx = torch.randn((1, 256, 3584), generator=g).to(dev)
    model.calibrate(ctx, torch.randn((1, 64, 64, 64), generator=g).to(dev), steps=2)
    counts = [DIT_SEEDS // world + (r < DIT_SEEDS % world) for r in range(world)]
    first = sum(counts[:rank])
    noise = torch.randn((DIT_SEEDS, 64, 64, 64), generator=torch.Generator().manual_seed(5))[first:first + counts[rank]]
    noise = noise.to(dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)                       # noqa: E731

    # single-image step latency (B = 1, 4096 tokens attending to the 256-token prefix)
    prefix = model.build_prefix(ctx)
    x1 = noise[:1].to(torch.bfloat16)
    t1 = torch.full((1,), 0.5, device=dev)
    work: dict = {}

    def latency(fn):
        for _ in range(3):
            fn()
        barrier()
        lat = [(ev(), ev()) for _ in range(10)]
        for a, b in lat:
            a.record(stream)
            fn()
            b.record(stream)
        barrier()
        return reduce_max(statistics.median(a.elapsed_time(b) for a, b in lat))

    step_ms_eager = latency(lambda: model.forward(x1, t1, prefix, work))
    step_ms = latency(lambda: model.step_graph(x1, t1, prefix))          # one captured forward per step

    # single-image latency with the MLP split over the ranks (NCCL all-reduce of the bf16 down partial per block)
    tp_lat = None
    if world > 1:
        def tp_step_ms(p2p: bool, graph: bool = False) -> float:
            model.enable_tp(p2p=p2p)
            step = (lambda: model.step_graph(x1, t1, prefix)) if graph else (lambda: model.forward(x1, t1, prefix, work))
            for _ in range(3):
                step()
            barrier()
            lat = [(ev(), ev()) for _ in range(10)]
            for a, b in lat:
                a.record(stream)
                step()
                b.record(stream)
            barrier()
            ms = reduce_max(statistics.median(a.elapsed_time(b) for a, b in lat))
            model.disable_tp()
            return ms

        tp_lat = {"world": world, "step_ms": tp_step_ms(True, graph=True), "step_ms_eager": tp_step_ms(True),
                  "step_ms_nccl": tp_step_ms(False),
                  "split": "MLP: gate/up columns (pairs kept local) and down rows over the ranks; attention, qkv, "
                           "out replicated",
                  "collective": "step_ms (one replayed CUDA graph per step; step_ms_eager: launched eagerly): the reduction fused into the down GEMM (tfb_gemm_nvfp4_tp: partial tiles "
                                "sent to their row owner with NVLink peer stores while the GEMM runs, reduced with "
                                "the gated residual in the owner's epilogue, x rows stored into every rank); "
                                "step_ms_nccl: NCCL all-reduce (sum) of the bf16 down partial [4096, 3072] per block"}

    # throughput: this rank's seeds through the whole sampler, the prompt's prefix built inside the timed region
    model.sample(noise, prefix, 1, graph=True)           # captures this batch's step graph (one-time)
    barrier()
    a, b = ev(), ev()
    with ClockSampler(dev.index) as clk:
        a.record(stream)
        prefix = model.build_prefix(ctx, into=prefix)     # the prompt's prefix pass, into the graph's buffers
        lat_out = model.sample(noise, prefix, DIT_STEPS, graph=True)
        b.record(stream)
        barrier()
    sample_s = reduce_max(a.elapsed_time(b)) / 1e3
    ok = bool(torch.isfinite(lat_out).all())
    info = {"workload": DIT_WORKLOAD, "step_ms_at_4096_tokens": step_ms, "step_ms_eager": step_ms_eager,
            "step_batch": 1,
            "img_per_s": DIT_SEEDS / sample_s, "sample_s": sample_s, "seeds": DIT_SEEDS,
            "seeds_per_rank": counts, "steps": DIT_STEPS, "scaling": "strong (32 seeds split across ranks)",
            "parallelism": f"dp{world} (weight replica per rank, no collective)",
            "weights_gb": model.nbytes() / 1e9, "libtfb_launches_per_step": 7 * model.cfg.layers + 1,
            "launches_note": "per image block: AdaLN+quant, qkv GEMM, q/k/v RMS-RoPE, out GEMM (+residual), AdaLN+quant, "
                             "gate/up+SwiGLU GEMM, down GEMM (+residual); plus the final AdaLN. torch adds SDPA per "
                             "block and the embedders; the prefix rows stay in per-block K/V buffers (no copies)",
            "tensor_parallel_latency": tp_lat, "finite": ok, "clocks": clk.report(),
            "timing": "CUDA events on the launching stream, max over ranks; latency = median of 10 steps after 3 "
                      "warm-up, each step one replayed CUDA graph of the forward (eager launches: step_ms_eager); "
                      "throughput = one timed 25-step sampler run (graph steps, prefix pass included) after a "
                      "warm-up step"}
    return info, (model, prefix, model.cfg.layers)


# ------------------------------------------------------------------------------------------------- summary
def summary(line: dict) -> dict:
    """The numbers of every BASELINE config in a few short keys, printed last in the line (a reader that keeps only
    the line's tail still sees them): configs[0] GEMM, configs[2] fusions, configs[3] FP8 GEMMs, configs[4] DiT
    step / images per second / tensor-parallel step, the CPU arms and the host link."""
    def r(v, n=3):
        return None if v is None else round(float(v), n)

    out = {"c1_mlp_tflops": r(line["value"], 1), "c1_gu_frac_fp4": r(line["roofline"]["frac"]),
           "c1_e2e_tflops": r(line["e2e"]["value"], 1)}
    cf = line.get("configs")
    if cf:
        c0, c2, c3 = cf["configs[0]"], cf["configs[2]"], cf["configs[3]"]
        out.update(c0_gemm_us=r(c0["gemm_us"], 2), c0_gemm_tflops=r(c0["gemm_tflops"], 1),
                   c0_frac_fp4=r(c0["gemm_frac_fp4_peak"]), c0_quant_us=r(c0["quant_us"], 2),
                   c0_linear_tflops=r(c0["linear_tflops"], 1), c0_e2e_tflops=r(c0["e2e"]["tflops"], 1),
                   c2_adaln_quant_gbs=r(c2["adaln_quant_gbs"], 0), c2_adaln_quant_frac=r(c2["adaln_quant_frac_hbm"]),
                   c2_rope_qkv_gbs=r(c2["rms_rope_qkv_gbs"], 0), c2_rope_qkv_frac=r(c2["rms_rope_qkv_frac_hbm"]),
                   c3_fp8_tflops=[r(c3[k]["tflops"], 0) for k in ("linear_3072", "gate_up_16384", "down_3072_k8192")],
                   c3_frac_fp8=[r(c3[k]["frac_fp8_peak"]) for k in ("linear_3072", "gate_up_16384", "down_3072_k8192")])
    d = line.get("dit")
    if d:
        out.update(c4_step_ms=r(d["step_ms_at_4096_tokens"]), c4_img_per_s=r(d["img_per_s"]),
                   c4_img_per_s_per_gpu=r(d["img_per_s"] / line["n_gpus"]))
        tp = d.get("tensor_parallel_latency")
        if tp:
            out.update(c4_tp_world=tp["world"], c4_tp_step_ms_fused=r(tp["step_ms"]),
                       c4_tp_step_ms_nccl=r(tp["step_ms_nccl"]))
    cb = line.get("cpu_baseline")
    if cb:
        out["cpu_c1_tflops"] = r(cb["value"], 4)
    if line.get("cpu_baseline_configs2"):
        out["cpu_c2_adaln_quant_gbs"] = r(line["cpu_baseline_configs2"]["adaln_quant_gbs"])
    if line.get("cpu_baseline_configs0_3"):
        out["cpu_c0_tflops"] = r(line["cpu_baseline_configs0_3"]["c0_nvfp4_tflops"], 4)
        out["cpu_c3_fp8_tflops"] = r(line["cpu_baseline_configs0_3"]["c3_fp8_tflops"], 4)
    if line.get("cpu_baseline_configs4"):
        out["cpu_c4_step_s"] = r(line["cpu_baseline_configs4"]["step_s_estimate"], 1)
    hl = line["e2e"].get("host_link", {})
    out.update(link_h2d_gbs=r(hl.get("h2d_gbs_per_rank"), 1), link_both_gbs=r(hl.get("both_gbs_per_rank"), 1))
    out["device_status"] = line.get("device_status")
    return out


# --------------------------------------------------------------------------------------------- profile legs
PROFILE_LEGS = ("gemm0", "fp8_3072", "adaln_quant", "swiglu", "qkv")


def run_profile_leg(name: str, reps: int = 4) -> None:
    """One kernel of one BASELINE config, launched ``reps`` times on cuda:0 with only its own operands allocated
    (a few hundred MB at most), for ncu captures of a single launch:
      gemm0        configs[0] NVFP4 GEMM   X codes [4096, 3072] x W [3072, 3072]
      fp8_3072     configs[3] FP8 GEMM     X e4m3 [4968, 3072] x W [3072, 3072], per-channel W scales
      adaln_quant  configs[2] AdaLN + shift + NVFP4 quantize on x [4352, 3072]
      swiglu       configs[1] gate/up NVFP4 GEMM with the SwiGLU -> NVFP4 epilogue (M 4352, F 8192, K 3072)
      qkv          configs[4] qkv NVFP4 GEMM with q / k RMSNorm + RoPE and the v copy in its epilogue (4096 tokens,
                   24 heads of 128, K 3072)
    Prints one line per launch with its CUDA-event time (for orientation only; never a bench value)."""
    import torch

    from tfimage import _lib
    from tfimage import kernels as Kn
    from tfimage import linear as L

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(77)
    if name == "gemm0":
        x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16).to(dev)
        lin = L.Nvfp4Linear((torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16).to(dev))
        lin.set_act(float(_lib.absmax(x)) / (6 * 448))
        q = lin.quantize(x)
        fn = lambda: lin(q)                                                    # noqa: E731
    elif name == "fp8_3072":
        x = torch.randn(4968, 3072, generator=g).to(torch.bfloat16).to(dev)
        f8 = L.Fp8Linear((torch.randn(3072, 3072, generator=g) * 0.02).to(torch.bfloat16).to(dev), per_channel=True)
        a = _lib.fp8_act_scale(x)
        q8 = _lib.quant_fp8(x, a)
        fn = lambda: _lib.gemm_fp8(q8, f8.w8.view(torch.uint8), 4968, 3072, 3072, a, f8.ws)   # noqa: E731
    elif name == "adaln_quant":
        x = torch.randn(1, 4352, 3072, generator=g).to(torch.bfloat16).to(dev)
        sc = (torch.randn(1, 1, 3072, generator=g) * 0.1).to(dev)
        sh = (torch.randn(1, 1, 3072, generator=g) * 0.1).to(dev)
        fn = lambda: Kn.adaln(x, sc, 1e-6, shift=sh, quant=0.004)               # noqa: E731
    elif name == "swiglu":
        x = torch.randn(4352, 3072, generator=g).to(torch.bfloat16).to(dev)
        gu = L.Nvfp4Linear((torch.randn(2 * 8192, 3072, generator=g) * 0.02).to(torch.bfloat16).to(dev))
        gu.set_act(float(_lib.absmax(x)) / (6 * 448))
        q = gu.quantize(x)
        fn = lambda: _lib.gemm_nvfp4_swiglu(q.codes, q.sf, gu.lin.codes, gu.lin.bs, 4352, 8192, 3072,  # noqa: E731
                                             q.act * gu.lin.scale, 0.004)
    elif name == "qkv":
        x = torch.randn(4096, 3072, generator=g).to(torch.bfloat16).to(dev)
        w = L.Nvfp4Linear((torch.randn(9216, 3072, generator=g) * 0.02).to(torch.bfloat16).to(dev))
        w.set_act(float(_lib.absmax(x)) / (6 * 448))
        q = w.quantize(x)
        qo = torch.empty(1, 4096, 24, 128, dtype=torch.bfloat16, device=dev)
        ko, vo = torch.empty_like(qo), torch.empty_like(qo)
        wq = (torch.randn(128, generator=g) * 0.05 + 1).to(dev)
        wk = (torch.randn(128, generator=g) * 0.05 + 1).to(dev)
        ang = torch.rand(4096, 64, generator=g).to(dev) * 6.28
        cos, sin = torch.cos(ang), torch.sin(ang)
        fn = lambda: _lib.gemm_nvfp4_qkv(q.codes, q.sf, w.lin.codes, w.lin.bs, 1, 4096, 24, 3072,  # noqa: E731
                                         q.act * w.lin.scale, wq, wk, cos, sin, 1e-6, qo, ko, vo)
    else:
        raise SystemExit(f"unknown profile leg {name!r}; one of {PROFILE_LEGS}")
    stream = torch.cuda.current_stream(dev)
    for i in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        print(f"{name} launch {i}: {e0.elapsed_time(e1) * 1e3:.1f} us", flush=True)
    assert _lib.device_status() == 0


# ------------------------------------------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from tfimage import _lib
    from tfimage import kernels as Kn
    from tfimage import linear as L

    # ------------------------------------------------------------------ synthetic model + calibrated scales
    g = torch.Generator().manual_seed(1000 + rank)
    wgu = (torch.randn(2 * F_DIM, K_DIM, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    wd = (torch.randn(K_DIM, F_DIM, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    x_host = torch.randn(M_ROWS, K_DIM, generator=g).to(torch.bfloat16).pin_memory()
    x = x_host.to(dev)
    gate_up, down = L.Nvfp4Linear(wgu), L.Nvfp4Linear(wd)
    del wgu, wd
    gate_up.set_act(float(_lib.absmax(x)) / (6 * 448))             # activation global = amax / (6 * 448)
    h = Kn.swiglu(gate_up(x))
    down.set_act(4 * float(_lib.absmax(h)) / (6 * 448))             # calibrate.py's 4x margin
    del h
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(ev):
        ev[0].record(stream)
        q = gate_up.quantize(x)
        ev[1].record(stream)
        hc, hs = _lib.gemm_nvfp4_swiglu(q.codes, q.sf, gate_up.lin.codes, gate_up.lin.bs, M_ROWS, F_DIM, K_DIM,
                                        q.act * gate_up.lin.scale, down.lin.act)
        ev[2].record(stream)
        y = _lib.gemm_nvfp4(hc, hs, down.lin.codes, down.lin.bs, M_ROWS, K_DIM, F_DIM,
                            down.lin.act * down.lin.scale)
        ev[3].record(stream)
        return y

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def step_call():
        # the public call (linear.swiglu_mlp): the same three kernels back to back, so each next kernel's launch and
        # prologue overlap the previous one's tail (programmatic launch); an event recorded between two kernels
        # would cut that overlap, so a step is timed by one event pair around the call
        return L.swiglu_mlp(gate_up, down, x)

    for _ in range(args.warmup):
        step_call()
        l2_flush(flush)
        step([torch.cuda.Event(enable_timing=True) for _ in range(4)])
        l2_flush(flush)
    step_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    # After a barrier the GPU is idle and the first steps' windows would also hold the host's time to queue their
    # kernels; a ~2 ms GPU sleep ahead of each pass (outside every event window) lets the host queue them first.
    def lead():
        if hasattr(torch.cuda, "_sleep"):                 # torch's spin kernel (cycles); without it: no lead
            torch.cuda._sleep(4_000_000)
    barrier()
    with ClockSampler(local) as clk:
        lead()
        for a, b in step_ev:
            a.record(stream)
            step_call()
            b.record(stream)
            l2_flush(flush)
        barrier()
    # the per-kernel split (and the dominant kernel's roofline): the same K steps again, events between the kernels
    lead()
    for i in range(args.steps):
        step(events[i])
        l2_flush(flush)
    barrier()
    per = [[e[j].elapsed_time(e[j + 1]) for j in range(3)] for e in events]      # ms: quant, gate/up, down
    step_ms = [a.elapsed_time(b) for a, b in step_ev]
    tot = torch.tensor([sum(step_ms), sum(p[1] for p in per)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    ms_step = float(tot[0]) / args.steps
    value = world * FLOP_STEP / (ms_step * 1e-3) / 1e12

    # --------------------------------------------------------------------------------- end to end (host buffers)
    y_host = torch.empty((M_ROWS, K_DIM), dtype=torch.bfloat16).pin_memory()
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(max(3, min(args.steps, 50)))]
    # the public host-buffer call: rows streamed in chunks, copies in both directions overlapped with the MLP
    for _ in range(2):
        L.swiglu_mlp_host(gate_up, down, x_host, y_host, chunks=M_ROWS // 256, graph=True)
    barrier()
    for a, b in e2e_ev:
        l2_flush(flush)
        a.record(stream)
        L.swiglu_mlp_host(gate_up, down, x_host, y_host, chunks=M_ROWS // 256, graph=True)
        b.record(stream)
    barrier()
    e2e_t = torch.tensor([sum(a.elapsed_time(b) for a, b in e2e_ev) / len(e2e_ev)], dtype=torch.float64,
                         device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = world * FLOP_STEP / (float(e2e_t[0]) * 1e-3) / 1e12

    def reduce_max(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    # the host link alone, per rank (every rank at once, max over ranks): the step's 26.7 MB in, out, and both at
    # once on two streams -- what bounds e2e when the copies of all ranks share the host's memory and PCIe
    link = {}
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    y_dev = torch.empty((M_ROWS, K_DIM), dtype=torch.bfloat16, device=dev)
    for name, ops in (("h2d", (("in",),)), ("d2h", (("out",),)), ("both", (("in",), ("out",)))):
        evs = []
        for _ in range(5):
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            # every copy stream forks from the same point before any joins back, so "both" runs the two
            # directions concurrently (joining after each copy would serialise them)
            used = [s_in if kind == "in" else s_out for (kind,) in ops]
            for st_ in used:
                st_.wait_stream(stream)
            for (kind,), st_ in zip(ops, used):
                with torch.cuda.stream(st_):
                    if kind == "in":
                        x.copy_(x_host, non_blocking=True)
                    else:
                        y_host.copy_(y_dev, non_blocking=True)
            for st_ in used:
                stream.wait_stream(st_)
            b.record(stream)
            evs.append((a, b))
        barrier()
        ms = reduce_max(statistics.median(a.elapsed_time(b) for a, b in evs))
        nbytes = x_host.numel() * 2 * len(ops)
        link[name + "_gbs_per_rank"] = nbytes / (ms * 1e-3) / 1e9
    del y_dev

    dit, dit_model = None, None
    if not args.no_dit:
        del flush
        dit, dit_model = dit_leg(world, rank, dev, barrier, reduce_max)
    status = _lib.device_status()

    if rank == 0:
        pk, src = peaks()
        fp4_peak = FP4_NOMINAL_TFLOPS
        gu_ms = statistics.median(p[1] for p in per)
        down_ms = statistics.median(p[2] for p in per)
        q_ms = statistics.median(p[0] for p in per)
        achieved = FLOP_GU / (gu_ms * 1e-3) / 1e12
        e2e_ms = float(e2e_t[0])
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4", "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M_ROWS, "K": K_DIM, "F": F_DIM, "global_batch": world,
                       "rows_per_gpu": M_ROWS, "parallelism": f"dp{world} (independent images, no collective)",
                       "l2": "flushed between steps: 256 MiB write then read back (clean lines) outside the per-step events"},
            "pct_fp4_nominal": value / world / fp4_peak,
            "kernels_ms": {"quant_x": q_ms, "gate_up_swiglu_nvfp4": gu_ms, "down": down_ms},
            "timing": "value / ms_per_step: K steps of the public linear.swiglu_mlp call, one CUDA event pair per "
                      "step; kernels_ms and the roofline: the same K steps again with an event between the kernels "
                      "(those events cut the programmatic-launch overlap, so the three add up to more than a step); each pass "
                      "starts behind a ~2 ms GPU sleep so no window holds host enqueue time",
            "roofline": {"bound": "tensor", "kernel": "gemm_kernel<MODE_FP4_SWIGLU> (gate/up + SwiGLU->NVFP4)",
                         "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s", "frac": achieved / fp4_peak,
                         "traffic": TRAFFIC_GU, "traffic_unit": "bytes per launch",
                         "peak_note": "nominal dense FP4 of one B200 (MEASURED_PEAKS.json has no FP4 figure); "
                                      f"4 x its measured bf16 burst = {4 * pk['bf16_tflops']:.0f} ({src})"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": x_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 2, "ms_per_step": e2e_ms,
                    "copy_gbs_per_rank": (x_host.numel() + y_host.numel()) * 2 / (e2e_ms * 1e-3) / 1e9,
                    "host_link": link},
            "gpu_launches": 3 * args.steps,
            "clocks": clk.report(),
            "device_status": status,
            "dit": dit,
        }
        if not args.no_configs:
            line["configs"] = config_legs(dev, fp4_peak, FP8_NOMINAL_TFLOPS, pk["hbm_gbs"])
            line["configs"]["peaks"]["source"] = (f"FP4 / FP8: nominal dense; HBM: MEASURED_PEAKS.json copy ({src})")
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
            line["cpu_baseline_configs2"] = cpu_baseline_fusions()
            line["cpu_baseline_configs0_3"] = cpu_baseline_linears()
            if dit_model is not None:
                line["cpu_baseline_configs4"] = cpu_baseline_dit(*dit_model)
        line["summary"] = summary(line)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dit", action="store_true", help="skip the configs[4] DiT leg (latency + img/s)")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[0], [2], [3] kernel lines")
    ap.add_argument("--profile-leg", choices=PROFILE_LEGS, help="run one kernel of one config a few times (for ncu)")
    args = ap.parse_args()
    if args.profile_leg:
        run_profile_leg(args.profile_leg)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
