"""Linear layers for DiT steps on B200: bf16 (reference), FP8 W8A8 and NVFP4 W4A4 on libtfb's tcgen05 GEMMs.

Drop-in for the reference ``tfimage/linear.py`` (same names, arguments and semantics; reference lines cited per
symbol). Activations are quantized under a per-layer input scale ``act``: measured on the fly (``act=None``: the
NVFP4 path reads amax back to the host once per call, exactly like the reference, because calibration consumes
it as a Python float) or fixed from a calibration run (no host sync, CUDA-graph safe). Per-16 NVFP4 block scales
still follow every row's range.

Differences from the reference, all forced by the hardware or by the absent TensorFold library:
  * ``nvfp4_supported`` gates on compute capability 10.0 and on libtfb loading (the reference gates on 12.x);
  * the ``Fp4Linear`` container keeps the reference attribute names but its own layout: ``words`` are the NVFP4
    codes viewed as int32 [N, K/8], ``bs`` the scale bytes in the GEMM's tiled layout;
  * ``make`` dispatches exactly as the reference: NVFP4 needs ``k % 128 == 0 and n % 64 == 0``, FP8
    ``k % 16 == 0 and n % 16 == 0``, other shapes go to bf16;
  * ``Fp8Linear`` optionally takes per-output-channel weight scales (``per_channel=True``).
"""

from __future__ import annotations

from functools import lru_cache

import torch
import torch.nn.functional as F

from . import _lib

FP4_MAX, E4M3_MAX = 6.0, 448.0
# Tile ids the reference passed to TensorFold's prompt GEMM (linear.py:17). They are accepted for API and
# engine-file compatibility; the sm_100a library has one persistent 128x256 tcgen05 tile, used for all of them.
TILES = (0, 1, 2, 12, 13)


@lru_cache(maxsize=1)
def nvfp4_supported() -> bool:
    """linear.py:25-27, for B200: a CUDA device of compute capability 10.0 and a loadable libtfb."""
    if not torch.cuda.is_available() or torch.cuda.get_device_capability() != (10, 0):
        return False
    try:
        _lib.load()
    except OSError:
        return False
    return True


def nvfp4_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """linear.py:30-38: bf16 [N, K] -> (e2m1 codes [N, K/2] uint8, e4m3 scales [N, K/16], global scale)."""
    n, k = w.shape
    g = max(float(w.float().abs().amax()), 1e-12) / (FP4_MAX * E4M3_MAX)
    wb = w.to(torch.bfloat16).contiguous()
    codes, scales = _lib.quant_nvfp4(wb, g, _lib.SF_ROWS)
    return codes, scales.view(torch.float8_e4m3fn), g


# ------------------------------------------------------------------------------------------ scale-layout helpers
def sf_tile(rows: torch.Tensor) -> torch.Tensor:
    """Row-major scale bytes [R, K/16] -> the GEMM's tiled layout [ceil(R/128) * K/64 * 512] (zero-padded rows)."""
    rows = rows.view(torch.uint8)
    R, S = rows.shape
    Rp = (R + 127) // 128 * 128
    if Rp != R:
        rows = torch.cat([rows, rows.new_zeros((Rp - R, S))])
    return rows.reshape(Rp // 128, 4, 32, S // 4, 4).permute(0, 3, 2, 1, 4).reshape(-1).contiguous()


def sf_untile(tiled: torch.Tensor, R: int, K: int) -> torch.Tensor:
    S = K // 16
    Rp = (R + 127) // 128 * 128
    return tiled.view(torch.uint8).reshape(Rp // 128, S // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(Rp, S)[:R]


class Fp4Linear:
    """NVFP4 weight container with the attribute names tfimage's engine store uses (store.py:38-42,66-71).

    ``words``: codes as int32 [N, K/8] (8 E2M1 values per word, even element in the lowest nibble);
    ``bs``: scale bytes, tiled for the GEMM; ``scale``: weight global g; ``act``: input global."""

    def __init__(self, words: torch.Tensor, bs: torch.Tensor, scale: float, n: int, k: int, act: float = 1.0):
        self.words, self.bs, self.scale, self.n, self.k, self.act = words, bs, float(scale), int(n), int(k), float(act)

    @classmethod
    def from_checkpoint(cls, codes: torch.Tensor, scales: torch.Tensor, g: float, act: float = 1.0) -> "Fp4Linear":
        n, half_k = codes.shape
        words = codes.contiguous().view(torch.int32)
        return cls(words, sf_tile(scales.contiguous()), g, n, half_k * 2, act)

    @property
    def codes(self) -> torch.Tensor:
        return self.words.view(torch.uint8)

    def scales(self) -> torch.Tensor:
        """Row-major e4m3 scales [N, K/16] (the nvfp4_weight view)."""
        return sf_untile(self.bs, self.n, self.k).view(torch.float8_e4m3fn)

    def tiles(self, a: int, b: int) -> "Fp4Linear":
        """Rows [64a, 64b) as their own container (the reference's N-tiles of 64 rows)."""
        codes = self.codes[64 * a:64 * b]
        scales = self.scales()[64 * a:64 * b]
        return Fp4Linear.from_checkpoint(codes, scales, self.scale, self.act)


class Nvfp4Act:
    """Activations already quantized under ``act`` (e.g. by the AdaLN fusion): codes [M, K/2] + tiled scales."""

    def __init__(self, codes: torch.Tensor, sf: torch.Tensor, act: float, m: int, k: int):
        self.codes, self.sf, self.act, self.m, self.k = codes, sf, float(act), int(m), int(k)


class Linear:
    """y = x @ W^T for 2-D bf16 rows; ``kind`` names the backend (linear.py:41-52)."""

    kind = "base"
    n: int
    k: int

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def nbytes(self) -> int:
        raise NotImplementedError


class Bf16Linear(Linear):
    """linear.py:55-67 (cuBLAS through F.linear; not a hot-path kernel)."""

    kind = "bf16"

    def __init__(self, w: torch.Tensor):
        self.w = w.to(torch.bfloat16).contiguous()
        self.n, self.k = self.w.shape

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w = self.w if self.w.device == x.device else self.w.to(x.device, non_blocking=True)
        return F.linear(x, w)

    def nbytes(self) -> int:
        return self.w.numel() * 2


class Fp8Linear(Linear):
    """linear.py:70-102: W8A8 e4m3 with one input scale (static or measured on the device) and a tensor-wise --
    or, with ``per_channel=True``, per-output-channel -- weight scale, on libtfb's tcgen05 FP8 GEMM."""

    kind = "fp8"

    def __init__(self, w: torch.Tensor, act: float | None = None, per_channel: bool = False):
        w = w.float()
        self.n, self.k = w.shape
        # the reference's expressions, with the divisor as a tensor so that CUDA divides exactly (a Python-number
        # divisor takes a reciprocal-multiply path there): scales and codes then equal the reference's on the CPU
        e4m3_max = torch.tensor(E4M3_MAX, dtype=torch.float32, device=w.device)
        if per_channel:
            s = (w.abs().amax(dim=1) / e4m3_max).clamp_min(1e-12)
            self.w8 = (w / s[:, None]).to(torch.float8_e4m3fn).contiguous()
            self.ws = s.contiguous()
        else:
            s = (w.abs().amax() / e4m3_max).clamp_min(1e-12)
            self.w8 = (w / s).to(torch.float8_e4m3fn).contiguous()
            self.ws = s.view(()).contiguous()
        self.act = act
        self._a = None
        self._a_val = None

    def _act(self, x: torch.Tensor) -> torch.Tensor:
        if self.act is None:
            return _lib.fp8_act_scale(x)
        if self._a is None or self._a.device != x.device or self._a_val != self.act:
            self._a = torch.tensor(self.act, dtype=torch.float32, device=x.device)
            self._a_val = self.act
        return self._a

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x = x.to(torch.bfloat16)
        if x.stride(-1) != 1:
            x = x.contiguous()
        a = self._act(x)
        w8, ws = self.w8, self.ws
        if w8.device != x.device:
            self.w8, self.ws = w8, ws = w8.to(x.device), ws.to(x.device)
        q = _lib.quant_fp8(x, a)
        return _lib.gemm_fp8(q, w8.view(torch.uint8), x.shape[0], self.n, self.k, a, ws)

    def nbytes(self) -> int:
        return self.w8.numel() + 4 * self.ws.numel()


class Nvfp4Linear(Linear):
    """linear.py:105-133: W4A4 NVFP4 (e2m1 values, e4m3 scale per 16, fp32 global) on libtfb's block-scaled
    tcgen05 GEMM. ``tile`` is kept for API compatibility (see ``TILES``)."""

    kind = "nvfp4"

    def __init__(self, w: torch.Tensor, act: float | None = None, tile: int = 12):
        codes, scales, g = nvfp4_weight(w)
        self.lin = Fp4Linear.from_checkpoint(codes, scales, g, act=act if act is not None else 1.0)
        self.n, self.k = self.lin.n, self.lin.k
        self.dynamic = act is None
        self.tile = tile
        self.amax = 0.0                 # largest input scale seen (calibration)

    @classmethod
    def from_fp4(cls, lin: "Fp4Linear", tile: int = 12) -> "Nvfp4Linear":
        """A static-scale layer around an existing container (e.g. a tensor-parallel shard), no re-quantization."""
        self = cls.__new__(cls)
        self.lin, self.n, self.k, self.dynamic, self.tile, self.amax = lin, lin.n, lin.k, False, tile, 0.0
        return self

    def set_act(self, act: float | None) -> None:
        self.dynamic = act is None
        if act is not None:
            self.lin.act = float(act)

    def quantize(self, x: torch.Tensor) -> Nvfp4Act:
        """Quantize rows under this layer's input scale (measuring it first in dynamic mode, linear.py:126-129)."""
        if self.dynamic:
            a = max(float(_lib.absmax(x)), 1e-6) / (FP4_MAX * E4M3_MAX)
            self.amax = max(self.amax, a)
            self.lin.act = a
        if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
            x = x.to(torch.bfloat16).contiguous()
        codes, sf = _lib.quant_nvfp4(x, self.lin.act, _lib.SF_TILED)
        return Nvfp4Act(codes, sf, self.lin.act, x.shape[0], self.k)

    def __call__(self, x, residual=None) -> torch.Tensor:
        """y = x @ W^T (bf16). ``residual=(res, gate)`` (this build's addition): instead of returning y, update
        ``res`` in place as ``res.addcmul_(y, gate)`` does (qwen_image21.py:213-215) inside the GEMM's epilogue,
        and return ``res``."""
        q = x if isinstance(x, Nvfp4Act) else self.quantize(x)
        lin = self.lin
        if residual is not None:
            res, gate = residual
            r2, g2, rows = _residual_views(res, gate, lin.n)
            _lib.gemm_nvfp4_resid(q.codes, q.sf, lin.codes, lin.bs, q.m, lin.n, lin.k, q.act * lin.scale, r2, g2,
                                  rows)
            return res
        return _lib.gemm_nvfp4(q.codes, q.sf, lin.codes, lin.bs, q.m, lin.n, lin.k, q.act * lin.scale)

    def nbytes(self) -> int:
        return self.lin.words.numel() * 4 + self.lin.bs.numel()


def _residual_views(res: torch.Tensor, gate: torch.Tensor, n: int):
    """res [..., n] bf16 (rows contiguous) and gate [B, 1, n] / [B, n] -> (res rows [M, n], gate rows [B, n], rows
    per gate row); the residual stream is updated in place, so it must be a view the GEMM can write."""
    if res.dtype != torch.bfloat16 or res.shape[-1] != n or res.stride(-1) != 1:
        raise ValueError("residual stream must be bf16 [..., n] with unit column stride")
    r2 = res.view(-1, n)
    g2 = gate.reshape(-1, n)
    if g2.dtype != torch.bfloat16:
        g2 = g2.to(torch.bfloat16)
    if g2.stride(-1) != 1:
        g2 = g2.contiguous()
    if r2.shape[0] % g2.shape[0]:
        raise ValueError("residual rows must split evenly over the gate rows")
    return r2, g2, r2.shape[0] // g2.shape[0]


def gated_residual_(lin: Linear, x, res: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """res.addcmul_(lin(x), gate) -- fused into the GEMM epilogue for static NVFP4 layers, torch otherwise."""
    if isinstance(lin, Nvfp4Linear):
        return lin(x, residual=(res, gate))
    return res.addcmul_(lin(x).view_as(res), gate)


def swiglu_mlp(gate_up: Linear, down: Linear, x: torch.Tensor, residual=None):
    """linear.py:136-150, the fused MLP pair. Two libtfb launches after the input quantizer: the gate/up GEMM
    computes both halves of each hidden column in one 256-wide tile, applies SwiGLU in its epilogue and quantizes
    the result straight to NVFP4 codes + block scales under ``down``'s static input scale; the down GEMM consumes
    those codes. The hidden activations never exist in bf16 in HBM.

    Returns None (and the caller takes the unfused path, as with the reference) unless both layers are NVFP4 with
    static input scales and ``down.k`` equals the hidden width F. The reference also asks F % 64 == 0; the GEMMs here
    need F % 128 == 0, which every NVFP4 ``down`` from ``make`` satisfies (it has k % 128 == 0, and k = F), so the
    fused path is taken for exactly the layer pairs the reference fuses. ``residual=(res, gate)`` (this build's
    addition): the down GEMM adds ``gate * y`` into ``res`` in place (``res.addcmul_(y, gate)``) and ``res`` is
    returned."""

    if not (isinstance(gate_up, Nvfp4Linear) and isinstance(down, Nvfp4Linear)) or gate_up.dynamic or down.dynamic:
        return None
    f = gate_up.n // 2
    if f % 128 or down.k != f:
        return None
    q = x if isinstance(x, Nvfp4Act) else gate_up.quantize(x)
    gu = gate_up.lin
    h_codes, h_sf = _lib.gemm_nvfp4_swiglu(q.codes, q.sf, gu.codes, gu.bs, q.m, f, gu.k, q.act * gu.scale,
                                           down.lin.act)
    h = Nvfp4Act(h_codes, h_sf, down.lin.act, q.m, f)
    return down(h, residual=residual)


_COPY_STREAMS: dict = {}
_HOST_GRAPHS: dict = {}


def _mlp_host_pipeline(gate_up, down, x_host, y_host, xd, chunks: int) -> bool:
    dev = xd.device
    if dev not in _COPY_STREAMS:
        _COPY_STREAMS[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    s_in, s_out = _COPY_STREAMS[dev]
    cur = torch.cuda.current_stream(dev)
    M = x_host.shape[0]
    per = -(-M // chunks)                                         # ceil(M / chunks) rows ...
    step = max(256, -(-per // 256) * 256)                          # ... rounded up to whole 256-row pair tiles
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    for r0 in range(0, M, step):
        r1 = min(M, r0 + step)
        with torch.cuda.stream(s_in):
            xd[r0:r1].copy_(x_host[r0:r1], non_blocking=True)
        cur.wait_stream(s_in)
        y = swiglu_mlp(gate_up, down, xd[r0:r1])
        if y is None:
            return False
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_out):
            y_host[r0:r1].copy_(y, non_blocking=True)
        y.record_stream(s_out)
    cur.wait_stream(s_out)
    return True


def swiglu_mlp_host(gate_up: Linear, down: Linear, x_host: torch.Tensor, y_host: torch.Tensor, chunks: int = 3,
                    graph: bool = False):
    """This build's addition: ``swiglu_mlp`` on host-resident rows, pinned ``x_host`` [M, K] -> ``y_host`` [M, K],
    with the PCIe copies overlapped. The rows go in ``chunks`` pieces: chunk i+1 is copied in while chunk i computes
    and chunk i-1 is copied back, both directions of the link at once. Every op is row-wise, so the result equals one
    ``swiglu_mlp`` call on the whole input. The current stream waits for the last copy (time it with events on it).

    ``graph=True``: the pipeline for these layers, these two host buffers and this shape is captured into a CUDA
    graph on the first call and replayed afterwards (no per-call host work; the caller keeps the buffers and
    refills ``x_host`` in place). Without it each chunk costs three library calls of host time, which starves the
    GPU beyond ~3 chunks. None if the layers cannot take the fused path."""
    if not (isinstance(gate_up, Nvfp4Linear) and isinstance(down, Nvfp4Linear)) or gate_up.dynamic or down.dynamic:
        return None
    dev = gate_up.lin.words.device
    if not graph:
        xd = torch.empty(tuple(x_host.shape), dtype=torch.bfloat16, device=dev)
        return y_host if _mlp_host_pipeline(gate_up, down, x_host, y_host, xd, chunks) else None
    k = (id(gate_up), id(down), x_host.data_ptr(), y_host.data_ptr(), tuple(x_host.shape), chunks, dev)
    entry = _HOST_GRAPHS.get(k)
    if entry is None:
        xd = torch.empty(tuple(x_host.shape), dtype=torch.bfloat16, device=dev)
        if not _mlp_host_pipeline(gate_up, down, x_host, y_host, xd, chunks):   # warm-up: one-time set-up calls
            return None
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            _mlp_host_pipeline(gate_up, down, x_host, y_host, xd, chunks)
        torch.cuda.current_stream(dev).wait_stream(side)
        entry = _HOST_GRAPHS[k] = (g, xd, gate_up, down)
    entry[0].replay()
    return y_host


def make(kind: str, w: torch.Tensor, act: float | None = None) -> Linear:
    """linear.py:153-161: a backend by name for a bf16 [N, K] weight (dims the kernels cannot tile fall back to
    FP8, then bf16, as in the reference)."""

    n, k = w.shape
    if kind == "nvfp4" and nvfp4_supported() and k % 128 == 0 and n % 64 == 0:
        return Nvfp4Linear(w, act)
    if kind in ("nvfp4", "fp8") and k % 16 == 0 and n % 16 == 0:
        return Fp8Linear(w, act)
    return Bf16Linear(w)
