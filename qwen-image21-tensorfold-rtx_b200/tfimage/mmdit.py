"""Synthetic double-stream MMDiT on the tfimage API: the DiT step that the quantized-linear path runs inside.

Shape and dataflow follow the reference DiT (tfimage/qwen_image21.py) at the sizes of the synthetic benchmark model:
28 blocks, hidden 3072, 24 heads x 128, SwiGLU 8192, separate image and text QKV / O / MLP weights, all weights
N(0, 0.02) from a seed (no checkpoint), RMS-norm weights N(1, 0.05). A latent [16, 128, 128] patchified 2 x 2 is
the model input [B, 64, 64, 64] (4096 tokens); the prompt is a [256, 3584] context.

* Prefix (qwen_image21.py:218-255): the text rows run through the text-stream weights once per prompt, modulated at
  t = 0 and attending causally among themselves; every block's keys and values are kept.
* Step (qwen_image21.py:259-299, _block :204-216): only the image rows run. Per block: AdaLN (+ shift) fused with
  the NVFP4 quantizer of the qkv input, qkv GEMM, RMSNorm + RoPE of q and k (k written behind the kept prefix in
  the block's key buffer, v copied beside it), SDPA over [prefix, image], out GEMM, gated residual, AdaLN fused
  with the quantizer of the MLP input, the fused gate/up SwiGLU -> NVFP4 -> down pair, gated residual. Each block
  has its own key / value buffers whose prefix rows are written once per prompt, not copied in every step.
* Sampler: flow-matching Euler on shifted sigmas (sampling.py:12-31).

Linears are ``linear.make(kind, w)`` modules; static input scales come from ``calibrate`` (the reference's
calibrate.py procedure: a dynamic-scale run, then 4 x the largest input scale seen per layer).
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import kernels as K
from . import linear as L


@dataclass(frozen=True)
class DitConfig:
    layers: int = 28
    dim: int = 3072
    heads: int = 24
    head_dim: int = 128
    mlp: int = 8192
    in_ch: int = 64            # 16 latent channels x 2 x 2 patch
    txt_dim: int = 3584
    axes: tuple[int, int, int] = (16, 56, 56)
    theta: float = 10000.0
    eps: float = 1e-6


SHIFT = 0.69                   # sampling.py:7


def sigmas(steps: int, shift: float = SHIFT, table: int = 10000) -> list[float]:
    """Shifted flow-matching sigmas of the "simple" schedule plus a final 0 (sampling.py:12-16)."""
    t = torch.arange(1, table + 1, dtype=torch.float32) / table
    s = math.exp(shift) / (math.exp(shift) + (1 / t - 1))
    stride = table / steps
    return [float(s[-(1 + int(i * stride))]) for i in range(steps)] + [0.0]


def rope_table(ids: torch.Tensor, cfg: DitConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """ids [N, 3] -> cos, sin fp32 [N, head_dim / 2]; per axis the frequencies theta^-(2i/d) in fp64
    (qwen_image21.py:63-72)."""
    parts = []
    for axis, d in enumerate(cfg.axes):
        expo = torch.linspace(0, (d - 2) / d, steps=d // 2, dtype=torch.float64, device=ids.device)
        parts.append(ids[:, axis].to(torch.float64)[:, None] * (1.0 / cfg.theta ** expo)[None])
    a = torch.cat(parts, dim=1)
    return torch.cos(a).float(), torch.sin(a).float()


def image_ids(h: int, w: int, pos: int, device) -> torch.Tensor:
    """[h*w, 3] ids of a target latent grid: (pos, row, col) centred on the grid (qwen_image21.py:164-169)."""
    hh = torch.arange(h, device=device, dtype=torch.float32) - (h - h // 2)
    ww = torch.arange(w, device=device, dtype=torch.float32) - (w - w // 2)
    return torch.stack([torch.full((h, w), float(pos), device=device), hh[:, None].expand(h, w),
                        ww[None, :].expand(h, w)], dim=-1).reshape(-1, 3)


def text_ids(n: int, device) -> torch.Tensor:
    """Sequential positions on all three axes (qwen_image21.py:232)."""
    return torch.arange(n, device=device, dtype=torch.float32)[:, None].expand(n, 3)


@dataclass
class Block:
    qkv: L.Linear
    out: L.Linear
    gate_up: L.Linear
    down: L.Linear
    norm_q: torch.Tensor       # fp32 [head_dim]
    norm_k: torch.Tensor
    tp: object = None          # tp.TPMLP: this rank's MLP shard (single-image latency mode)


_PREFIX_VERSIONS = itertools.count(1)


@dataclass
class Prefix:
    kv: list                   # per block (k, v) [1, P, H, D] bf16
    length: int
    next_pos: int
    version: int = field(default_factory=lambda: next(_PREFIX_VERSIONS))   # new on every (re)build


def _sdpa(q, k, v, causal=False):
    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION],
                     set_priority=True):
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal)


class SynthMMDiT:
    """The synthetic MMDiT with NVFP4 (or ``kind``) linears; weights generated on ``device`` from ``seed``."""

    def __init__(self, cfg: DitConfig = DitConfig(), kind: str = "nvfp4", device="cuda", seed: int = 0):
        self.cfg, self.kind, self.device = cfg, kind, torch.device(device)
        # Per-block key / value buffers that keep the prefix rows across steps (``forward``), used while their total
        # size stays within this many bytes (None: 40 % of the device's memory); larger batches share one buffer.
        self.kv_budget: int | None = None
        g = torch.Generator(device=self.device).manual_seed(seed)
        D = cfg.dim

        def rnd(*shape, std=0.02, mean=0.0):
            t = torch.randn(shape, generator=g, device=self.device, dtype=torch.float32)
            return (t * std + mean).to(torch.bfloat16)

        self.t1, self.t2 = rnd(D, 256), rnd(D, D)                # timestep embedder
        self.mod_img, self.mod_txt = rnd(6 * D, D), rnd(6 * D, D)
        self.img_in, self.proj_out, self.norm_out = rnd(D, cfg.in_ch), rnd(cfg.in_ch, D), rnd(D, D)
        self.txt_norm = (torch.randn((cfg.txt_dim,), generator=g, device=self.device) * 0.05 + 1.0).float()
        self.txt_in1, self.txt_in2 = rnd(D, cfg.txt_dim), rnd(D, D)
        self.img_blocks: list[Block] = []
        self.txt_blocks: list[Block] = []
        H = cfg.heads * cfg.head_dim
        for _ in range(cfg.layers):
            for blocks in (self.img_blocks, self.txt_blocks):
                lin = lambda *s: L.make(kind, rnd(*s))           # noqa: E731  (bf16 copy freed at once)
                blocks.append(Block(lin(3 * H, D), lin(D, H), lin(2 * cfg.mlp, D), lin(D, cfg.mlp),
                                    (torch.randn((cfg.head_dim,), generator=g, device=self.device) * 0.05 + 1).float(),
                                    (torch.randn((cfg.head_dim,), generator=g, device=self.device) * 0.05 + 1).float()))

    # ------------------------------------------------------------------------------------------- pieces
    def linears(self):
        for stream, blocks in (("img", self.img_blocks), ("txt", self.txt_blocks)):
            for i, b in enumerate(blocks):
                for name in ("qkv", "out", "gate_up", "down"):
                    yield f"{stream}.{i}.{name}", getattr(b, name)

    def nbytes(self) -> int:
        return sum(lin.nbytes() for _, lin in self.linears())

    def _temb(self, t: torch.Tensor) -> torch.Tensor:
        """t [B] in [0, 1] -> timestep embedding [B, dim] (sinusoidal 256 -> linear -> silu -> linear)."""
        half = 128
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        args = (t.float() * 1000.0)[:, None] * freqs[None]
        emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)
        return F.linear(F.silu(F.linear(emb, self.t1)), self.t2)

    @staticmethod
    def _mod(temb: torch.Tensor, w: torch.Tensor):
        """-> (shift1, scale1, gate1, shift2, scale2, gate2), each [B, 1, dim]; gates tanh'ed (qwen_image21.py:272).
        Shifts and scales are handed out as fp32 (exact copies of the bf16 values, the AdaLN kernel's input type),
        once per forward rather than converted in each of the 56 AdaLN calls; gates stay bf16."""
        m = F.linear(F.silu(temb), w).unsqueeze(1).chunk(6, dim=-1)
        f = lambda t: t.float().contiguous()     # noqa: E731
        return f(m[0]), f(m[1]), m[2].tanh(), f(m[3]), f(m[4]), m[5].tanh()

    def _block(self, b: Block, x, mod, cos, sin, kbuf, vbuf, causal=False, record: dict | None = None):
        """One block on rows x [B, N, dim] (in place); k / v are written to kbuf / vbuf [B, P + N, H, D] rows P:.
        ``record`` (tests): receives the intermediates; the fused AdaLN + quantize calls then also write their
        bf16 result (the quantizer's input)."""
        sh1, sc1, g1, sh2, sc2, g2 = mod
        cfg = self.cfg
        B, N, _ = x.shape
        H, Dh, eps = cfg.heads, cfg.head_dim, cfg.eps
        P = kbuf.shape[1] - N
        rec = record is not None
        bf = (lambda: torch.empty_like(x)) if rec else (lambda: None)   # noqa: E731
        static = isinstance(b.qkv, L.Nvfp4Linear) and not b.qkv.dynamic
        a_in = K.adaln(x, sc1, eps, shift=sh1, quant=b.qkv if static else None, out=bf() if static else None)
        if not static:
            a_in = a_in.reshape(B * N, -1)
        q = torch.empty((B, N, H, Dh), dtype=torch.bfloat16, device=x.device)
        if rec or not K.qkv_rms_rope(b.qkv, a_in, b.norm_q, b.norm_k, cos, sin, eps, q, kbuf[:, P:], vbuf[:, P:]):
            qkv = b.qkv(a_in).view(B, N, 3, H, Dh)    # record mode keeps the qkv tensor for the tests
            K.rms_rope_qkv(qkv, b.norm_q, b.norm_k, cos, sin, eps, q, kbuf[:, P:], vbuf[:, P:])
        o = _sdpa(q.transpose(1, 2), kbuf.transpose(1, 2), vbuf.transpose(1, 2), causal)
        o = o.transpose(1, 2)
        if rec:                       # the branch output on its own, then torch's addcmul_ (tests)
            a = b.out(o.reshape(B * N, H * Dh)).view(B, N, -1)
            record.update(a_in=a_in, qkv=qkv, q=q, o=o, att=a, x_in=x.clone())   # (rec: qkv set above)
            x.addcmul_(a, g1)
        else:                         # x += g1 * out(o), in the out GEMM's epilogue for NVFP4 layers
            L.gated_residual_(b.out, o.reshape(B * N, H * Dh), x, g1)
        static = isinstance(b.gate_up, L.Nvfp4Linear) and not b.gate_up.dynamic
        m_in = K.adaln(x, sc2, eps, shift=sh2, quant=b.gate_up if static else None, out=bf() if static else None)
        if rec:
            x1 = x.clone()
        if b.tp is not None and static and not rec:
            b.tp(m_in, residual=(x, g2))   # this rank's MLP shard, NCCL all-reduce, then the gated residual
            return x
        if static and not rec and L.swiglu_mlp(b.gate_up, b.down, m_in, residual=(x, g2)) is not None:
            return x                  # x += g2 * down(SwiGLU(gate_up(m))), in the down GEMM's epilogue
        y = L.swiglu_mlp(b.gate_up, b.down, m_in) if static else None
        if y is None:
            h = m_in.reshape(B * N, -1) if not isinstance(m_in, L.Nvfp4Act) else m_in
            y = b.down(K.swiglu(b.gate_up(h)))
        if rec:
            record.update(x1=x1, m_in=m_in, mlp=y.view(B, N, -1))
        x.addcmul_(y.view(B, N, -1), g2)
        return x

    # ------------------------------------------------------------------------------------------- prefix
    @torch.inference_mode()
    def build_prefix(self, context: torch.Tensor, into: Prefix | None = None) -> Prefix:
        """context [1, L, txt_dim] -> the kept per-block text keys / values (t = 0 modulation, causal). ``into``: an
        earlier prefix of the same length whose buffers are overwritten (captured step graphs keep using them)."""
        cfg = self.cfg
        c = context.to(self.device).float()
        c = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + cfg.eps) * self.txt_norm
        x = F.linear(F.gelu(F.linear(c.to(torch.bfloat16), self.txt_in1), approximate="tanh"), self.txt_in2)
        x = x.contiguous()
        B, P, _ = x.shape
        cos, sin = rope_table(text_ids(P, self.device), cfg)
        mod = self._mod(self._temb(torch.zeros((B,), device=self.device)), self.mod_txt)
        if into is not None and (into.length != P or into.kv[0][0].shape[0] != B):
            raise ValueError("build_prefix(into=...): the kept prefix has another length or batch")
        kv = []
        for i, b in enumerate(self.txt_blocks):
            if into is not None:
                k, v = into.kv[i]
            else:
                k = torch.empty((B, P, cfg.heads, cfg.head_dim), dtype=torch.bfloat16, device=self.device)
                v = torch.empty_like(k)
            x = self._block(b, x, mod, cos, sin, k, v, causal=True)
            kv.append((k, v))
        if into is None:
            return Prefix(kv, P, P)
        into.version = next(_PREFIX_VERSIONS)       # step buffers holding the old rows are refilled on next use
        return into

    # ------------------------------------------------------------------------------------------- step
    def _kv_buffers(self, work: dict, B: int, rows: int) -> None:
        """The step's key / value buffers [B, P + N, H, D]: one pair per image block when they fit ``kv_budget``
        (the prefix rows are written once and stay, qwen_image21.py:287-293 copies them in every block of every
        step), else one shared pair that each block refills."""
        cfg = self.cfg
        shape = (B, rows, cfg.heads, cfg.head_dim)
        per_pair = 2 * math.prod(shape) * 2
        budget = self.kv_budget
        if budget is None:
            budget = int(0.4 * torch.cuda.get_device_properties(self.device).total_memory) \
                if self.device.type == "cuda" else 0
        new = lambda: torch.empty(shape, dtype=torch.bfloat16, device=self.device)   # noqa: E731
        if per_pair * len(self.img_blocks) <= budget:
            work.update(kv=[(new(), new()) for _ in self.img_blocks], kv_version=None)
        else:
            work.update(kv=None, kv_shared=(new(), new()))

    def _fill_prefix(self, work: dict, prefix: Prefix) -> None:
        """Copy the prefix rows into the per-block buffers once per prefix version."""
        if work.get("kv") is None or work["kv_version"] == prefix.version:
            return
        P = prefix.length
        for (kb, vb), (pk, pv) in zip(work["kv"], prefix.kv):
            kb[:, :P].copy_(pk.expand(kb.shape[0], -1, -1, -1))
            vb[:, :P].copy_(pv.expand(vb.shape[0], -1, -1, -1))
        work["kv_version"] = prefix.version

    @torch.inference_mode()
    def forward(self, x: torch.Tensor, t: torch.Tensor, prefix: Prefix, work: dict | None = None) -> torch.Tensor:
        """x [B, 64, H, W] bf16, t [B] -> velocity [B, 64, H, W] bf16. ``work`` caches the step's buffers (and,
        with per-block key / value buffers, the prefix rows between steps)."""
        cfg = self.cfg
        B, C, Hh, Ww = x.shape
        N, P = Hh * Ww, prefix.length
        work = {} if work is None else work
        key = (B, Hh, Ww, P)
        if work.get("key") != key:
            self._kv_buffers(work, B, P + N)
            work.update(key=key, rope=rope_table(image_ids(Hh, Ww, prefix.next_pos, self.device), cfg))
        self._fill_prefix(work, prefix)
        cos, sin = work["rope"]
        temb = self._temb(t)
        mod = self._mod(temb, self.mod_img)
        h = F.linear(x.flatten(2).transpose(1, 2), self.img_in)
        comm = self._tp_comm(B * N)
        h = comm.x(B * N).view(B, N, -1).copy_(h) if comm is not None else h.contiguous()
        for i, (b, (pk, pv)) in enumerate(zip(self.img_blocks, prefix.kv)):
            if work["kv"] is not None:
                kbuf, vbuf = work["kv"][i]
            else:
                kbuf, vbuf = work["kv_shared"]
                kbuf[:, :P].copy_(pk.expand(B, -1, -1, -1))
                vbuf[:, :P].copy_(pv.expand(B, -1, -1, -1))
            h = self._block(b, h, mod, cos, sin, kbuf, vbuf)
        h = K.adaln(h, F.linear(F.silu(temb), self.norm_out).unsqueeze(1), cfg.eps)
        out = F.linear(h, self.proj_out)
        return out.transpose(1, 2).reshape(B, C, Hh, Ww)

    __call__ = forward

    @torch.inference_mode()
    def step_graph(self, x: torch.Tensor, t: torch.Tensor, prefix: Prefix) -> torch.Tensor:
        """``forward`` replayed from a CUDA graph: the first call for a (shape, prefix) captures one forward with
        static input / output buffers, later calls copy ``x`` and ``t`` in and replay it (no per-kernel host work,
        no launch gaps). Returns the static output buffer: consume it before the next call."""
        graphs = self.__dict__.setdefault("_graphs", {})
        key = (tuple(x.shape), id(prefix))
        entry = graphs.get(key)
        if entry is not None:
            self._fill_prefix(entry[4], prefix)               # a rebuilt prefix: new rows, outside the graph
        if entry is None:
            xs, ts, work = x.clone(), t.clone(), {}
            self.forward(xs, ts, prefix, work)                   # warm-up: one-time set-up outside the capture
            side = torch.cuda.Stream(x.device)
            side.wait_stream(torch.cuda.current_stream(x.device))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
                out = self.forward(xs, ts, prefix, work)
            torch.cuda.current_stream(x.device).wait_stream(side)
            entry = graphs[key] = (g, xs, ts, out, work, prefix)   # the prefix held: its id stays unique
        g, xs, ts, out = entry[:4]
        xs.copy_(x)
        ts.copy_(t)
        g.replay()
        return out

    @torch.inference_mode()
    def sample(self, noise: torch.Tensor, prefix: Prefix, steps: int = 25, step_events=None,
               graph: bool = False) -> torch.Tensor:
        """Flow-matching Euler from unit-Gaussian noise [B, 64, H, W] (sampling.py:19-31); ``graph``: every step
        replays one captured forward (``step_graph``)."""
        sig = sigmas(steps)
        x = noise.float() * sig[0]
        work: dict = {}
        for i in range(steps):
            t = torch.full((x.shape[0],), sig[i], device=x.device)
            xb = x.to(torch.bfloat16)
            v = (self.step_graph(xb, t, prefix) if graph else self.forward(xb, t, prefix, work)).float()
            x = x + (sig[i + 1] - sig[i]) * v
            if step_events is not None:
                step_events[i].record()
        return x

    def enable_tp(self, group=None, p2p: bool = False) -> None:
        """Single-image latency mode: split every image block's MLP over the ranks of ``group`` (gate/up columns,
        down rows; tp.TPMLP), attention and the other linears replicated. Needs calibrated (static) scales.
        ``p2p``: the reduction runs inside the down GEMM over NVLink peer memory (tp.P2PComm, one per row count,
        made collectively at the first forward), else an NCCL all-reduce follows each MLP."""
        from .tp import TPMLP

        self.__dict__.pop("_graphs", None)           # captured steps of the other mode
        for b in self.img_blocks:
            b.tp = TPMLP(b.gate_up, b.down, group)
        self._tp = {"group": group, "p2p": p2p, "comm": None}

    def disable_tp(self) -> None:
        torch.cuda.synchronize(self.device)
        self.__dict__.pop("_graphs", None)           # graphs that reference the communicator's buffers
        for b in self.img_blocks:
            b.tp = None
        tp = self.__dict__.pop("_tp", None)
        if tp and tp["comm"] is not None:
            tp["comm"].close()

    def _tp_comm(self, rows: int):
        """The P2P communicator for ``rows`` image rows (None unless ``enable_tp(p2p=True)``); the residual stream
        of the step lives in its buffer."""
        from .tp import P2PComm

        tp = self.__dict__.get("_tp")
        if not tp or not tp["p2p"]:
            return None
        comm = tp["comm"]
        if comm is None or comm.max_rows != rows:
            if comm is not None:
                comm.close()
            comm = tp["comm"] = P2PComm(rows, self.cfg.dim, tp["group"], self.device)
            for b in self.img_blocks:
                b.tp.comm = comm
        return comm

    # ------------------------------------------------------------------------------------------- calibration
    @torch.inference_mode()
    def calibrate(self, context: torch.Tensor, noise: torch.Tensor, steps: int = 4, margin: float = 4.0) -> dict:
        """Static NVFP4 input scales (calibrate.py:19-33): run with dynamic scales, keep margin x the largest."""
        lins = [(n, lin) for n, lin in self.linears() if isinstance(lin, L.Nvfp4Linear)]
        for _, lin in lins:
            lin.set_act(None)
            lin.amax = 0.0
        prefix = self.build_prefix(context)
        self.sample(noise, prefix, steps)
        acts = {n: lin.amax * margin for n, lin in lins}
        for n, lin in lins:
            lin.set_act(acts[n])
        return acts
