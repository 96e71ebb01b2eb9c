"""Tensor-parallel fused MLP over NCCL: the single-image latency mode of the DiT step (this build's addition).

One image cannot be split by seed, so for the step latency the MLP -- two thirds of a block's linear FLOPs -- is
split over G ranks while attention, qkv and out stay replicated:

* gate/up is column-split with the pairs kept local: rank r holds gate rows [rF/G, (r+1)F/G) and the same up rows,
  so its SwiGLU epilogue sees matching gate/up columns;
* down is split along K (its input columns) to match;
* each rank's fused pair yields a partial down output (bf16 [M, dim]); an NCCL all-reduce (sum) over NVLink adds the
  G partials; the gated residual follows.

With a ``P2PComm`` the reduction is fused into the down GEMM instead (tfb_gemm_nvfp4_tp): the residual stream lives
in a buffer every rank maps over CUDA IPC; each rank owns one chunk of the rows, sends the partial tiles of the
other chunks to their owners with peer stores while its GEMM still runs, adds the received partials and the gated
residual for its own chunk in the epilogue and writes those x rows into every rank's copy. No NCCL call and no
separate reduction pass; the transfers overlap the GEMM tile by tile.

Because down's input scale is static and F/G is a multiple of 16, the NVFP4 codes and scales of a rank's SwiGLU
output are exactly the corresponding columns of the unsharded ones; the result differs from one GPU only by the
bf16 rounding of the partials and the order of the sum.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from . import linear as L


def shard_gate_up(gu: L.Fp4Linear, rank: int, world: int) -> L.Fp4Linear:
    """[gate; up] (2F rows) -> [gate rows of rank r; up rows of rank r] (2F/G rows)."""
    F = gu.n // 2
    if F % world or (F // world) % 128:
        raise ValueError(f"gate/up width F={F} must split into multiples of 128 over {world} ranks")
    f, lo = F // world, rank * (F // world)
    codes, scales = gu.codes, gu.scales()
    c = torch.cat([codes[lo:lo + f], codes[F + lo:F + lo + f]])
    s = torch.cat([scales[lo:lo + f], scales[F + lo:F + lo + f]])
    return L.Fp4Linear.from_checkpoint(c, s, gu.scale, gu.act)


def shard_down(down: L.Fp4Linear, rank: int, world: int) -> L.Fp4Linear:
    """down [dim, F] -> its input columns [rF/G, (r+1)F/G) (K split)."""
    F = down.k
    if F % world or (F // world) % 128:
        raise ValueError(f"down input width F={F} must split into multiples of 128 over {world} ranks")
    f, lo = F // world, rank * (F // world)
    c = down.codes[:, lo // 2:(lo + f) // 2].contiguous()
    s = down.scales()[:, lo // 16:(lo + f) // 16].contiguous()
    return L.Fp4Linear.from_checkpoint(c, s, down.scale, down.act)


class P2PComm:
    """The NVLink peer-memory communicator of a tensor-parallel group (tfb_tp_comm): one buffer per rank holding its
    copy of the residual stream ``x`` [max_rows, n_cols] bf16, receive slots for the other ranks' partial tiles and
    per-tile counters; exported with CUDA IPC and mapped by every other rank of ``group`` (one node). Serves one
    (M, N) shape per buffer; every rank makes its calls in the same order."""

    def __init__(self, max_rows: int, n_cols: int, group=None, device=None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if not 2 <= self.world <= _lib.TP_MAX_WORLD:
            raise ValueError(f"P2PComm: a tensor-parallel group needs 2 to {_lib.TP_MAX_WORLD} ranks, not {self.world}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        # one GPU per rank: the kernels of two ranks wait on each other, which two launches on one GPU cannot do
        uuids = [None] * self.world
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid), group=group)
        if len(set(uuids)) != self.world:
            raise ValueError("P2PComm needs every rank on its own GPU")
        nbytes, self.offsets = _lib.tp_layout(self.world, max_rows, n_cols)
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)   # counters start at zero
        everyone = [None] * self.world
        dist.all_gather_object(everyone, _lib.ipc_handle(self.buf), group=group)
        self._opened, bases = [], []
        for q, (handle, off) in enumerate(everyone):
            if q == self.rank:
                bases.append(self.buf.data_ptr())
            else:
                ptr = _lib.ipc_open(handle, off)
                self._opened.append((ptr, off))
                bases.append(ptr)
        base = (ctypes.c_void_p * _lib.TP_MAX_WORLD)(*bases)
        self.comm = _lib.TpComm(self.world, self.rank, base, max_rows, n_cols)
        self.max_rows, self.n_cols = max_rows, n_cols
        self.epoch, self.shape = 0, None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)            # every buffer is zeroed and mapped before any rank's first call

    def x(self, rows: int) -> torch.Tensor:
        """This rank's copy of the residual stream, rows [0, rows) as a bf16 [rows, n_cols] view."""
        if rows > self.max_rows:
            raise ValueError(f"P2PComm holds {self.max_rows} rows, {rows} asked")
        o = self.offsets[0]
        return self.buf[o:o + rows * self.n_cols * 2].view(torch.bfloat16).view(rows, self.n_cols)

    def next_epoch(self, M: int, N: int) -> int:
        """Host-side epoch of the next call (for the explicit-epoch form of the entry points)."""
        self.check_shape(M, N)
        self.epoch += 1
        return self.epoch

    def check_shape(self, M: int, N: int) -> None:
        if self.shape is not None and self.shape != (M, N):
            raise ValueError(f"P2PComm was used for {self.shape}; a buffer serves one shape (make another one)")
        self.shape = (M, N)

    def close(self) -> None:
        """Unmaps the other ranks' buffers (after this rank's last call has completed)."""
        torch.cuda.synchronize(self.device)
        for ptr, off in self._opened:
            _lib.ipc_close(ptr, off)
        self._opened = []


class TPMLP:
    """This rank's shard of a static-scale NVFP4 gate/up + down pair; ``__call__`` runs the fused pair on the shard,
    all-reduces the partial output over ``group`` and returns it (or adds it into a residual stream). With ``comm``
    and a residual that is the communicator's ``x``, the reduction and the residual run inside the down GEMM."""

    def __init__(self, gate_up: L.Nvfp4Linear, down: L.Nvfp4Linear, group=None, comm: P2PComm | None = None):
        import torch.distributed as dist

        if gate_up.dynamic or down.dynamic:
            raise ValueError("tensor-parallel MLP needs static input scales (calibrate first)")
        self.group, self.comm = group, comm
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.gate_up = L.Nvfp4Linear.from_fp4(shard_gate_up(gate_up.lin, self.rank, self.world))
        self.down = L.Nvfp4Linear.from_fp4(shard_down(down.lin, self.rank, self.world))

    def _fused(self, x, res: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        d = self.down.lin
        r2, g2, rows = L._residual_views(res, gate, d.n)
        M, N = r2.shape
        if r2.data_ptr() != self.comm.x(1).data_ptr() or r2.stride(0) != N:
            raise ValueError("the fused tensor-parallel MLP updates the communicator's x: pass comm.x(M) as residual")
        q = x if isinstance(x, L.Nvfp4Act) else self.gate_up.quantize(x)
        gu = self.gate_up.lin
        f = gu.n // 2
        h_codes, h_sf = _lib.gemm_nvfp4_swiglu(q.codes, q.sf, gu.codes, gu.bs, q.m, f, gu.k, q.act * gu.scale, d.act)
        # epochs live on the device (advanced by a kernel in stream order), so the three launches can be captured in
        # a CUDA graph and replayed
        self.comm.check_shape(M, N)
        _lib.tp_advance(self.comm.comm, res.device)
        _lib.gemm_nvfp4_tp(h_codes, h_sf, d.codes, d.bs, M, N, f, d.act * d.scale, g2, rows, self.comm.comm, 0)
        _lib.tp_wait(self.comm.comm, M, N, 0, res.device)
        return res

    def __call__(self, x, residual=None) -> torch.Tensor:
        import torch.distributed as dist

        if self.comm is not None and residual is not None:
            return self._fused(x, *residual)
        y = L.swiglu_mlp(self.gate_up, self.down, x)
        dist.all_reduce(y, group=self.group)
        if residual is None:
            return y
        res, gate = residual
        return res.addcmul_(y.view_as(res), gate)
