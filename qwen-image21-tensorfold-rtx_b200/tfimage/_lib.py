"""ctypes binding of libtfb.so (the C ABI in ``include/tfb.h``) plus thin torch-tensor wrappers.

Every wrapper validates nothing beyond what it needs to build pointers: the library checks shapes, alignment and
the device architecture itself and returns a status, which :func:`check` turns into ``TfbError`` (a
``RuntimeError``) carrying ``tfb_last_error()``. Work goes on torch's current CUDA stream; nothing here syncs
except :func:`device_status`. There is no fallback: if the library cannot be loaded, every op raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libtfb.so"
DEFAULT_DIR = Path(__file__).resolve().parent

c_i64, c_int, c_float, c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p

# name -> argtypes, mirroring include/tfb.h
SIGNATURES = {
    "tfb_version": [],
    "tfb_last_error": [],
    "tfb_sf_tiled_bytes": [c_i64, c_i64],
    "tfb_device_status": [ctypes.POINTER(c_int), c_int],
    "tfb_absmax_bf16": [c_vp, c_i64, c_vp, c_vp],
    "tfb_fp8_act_scale": [c_vp, c_i64, c_vp, c_vp],
    "tfb_quant_nvfp4": [c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_vp, c_int, c_vp],
    "tfb_quant_fp8": [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp],
    "tfb_gemm_nvfp4": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_i64, c_vp],
    "tfb_gemm_fp8": [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_int, c_vp, c_i64, c_vp],
    "tfb_gemm_nvfp4_resid": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_i64, c_vp, c_i64, c_i64,
                             c_vp],
    "tfb_gemm_nvfp4_swiglu": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_float, c_vp, c_vp, c_vp, c_vp,
                              c_vp],
    "tfb_mlp_nvfp4": [c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_vp, c_float, c_vp, c_vp, c_float, c_float, c_vp,
                      c_vp, c_vp, c_vp, c_vp, c_vp],
    "tfb_mlp_nvfp4_static": [c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_vp, c_float, c_vp, c_vp, c_float, c_float,
                             c_vp, c_vp],
    "tfb_adaln": [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_float, c_vp, c_float, c_vp, c_vp, c_vp],
    "tfb_rms_rope": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_float, c_vp, c_i64,
                     c_i64, c_vp],
    "tfb_rms_rope_qkv": [c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_float, c_vp, c_i64,
                         c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp],
    "tfb_swiglu": [c_vp, c_i64, c_i64, c_vp, c_vp],
    "tfb_gemm_nvfp4_qkv": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_float, c_vp, c_vp, c_vp, c_vp, c_float,
                           c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp],
    "tfb_tp_layout": [c_int, c_i64, c_i64, ctypes.POINTER(c_i64)],
    "tfb_gemm_nvfp4_tp": [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_vp, c_i64, c_i64, c_vp,
                          ctypes.c_uint32, c_vp],
    "tfb_tp_wait": [c_vp, c_i64, c_i64, ctypes.c_uint32, c_vp],
    "tfb_tp_advance": [c_vp, c_vp],
    "tfb_ipc_handle": [c_vp, c_vp, ctypes.POINTER(c_i64)],
    "tfb_ipc_open": [c_vp, c_i64, ctypes.POINTER(c_vp)],
    "tfb_ipc_close": [c_vp, c_i64],
    "tfb_gguf_block_bytes": [c_int, ctypes.POINTER(c_i64)],
    "tfb_gguf_dequant": [c_int, c_vp, c_i64, c_vp, c_int, c_vp],
}
RESTYPES = {"tfb_version": c_int, "tfb_last_error": ctypes.c_char_p, "tfb_sf_tiled_bytes": c_i64,
            "tfb_gguf_block_bytes": c_i64, "tfb_tp_layout": c_i64}

SF_ROWS, SF_TILED = 0, 1
GGUF_TYPES = {"Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}     # TFB_GGUF_* (ggml type ids)
OUT_DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}  # TFB_DT_*
MLP_STATIC_SCRATCH_BYTES = 32 << 20   # TFB_MLP_STATIC_SCRATCH_BYTES
STATUS = {0: "OK", 1: "BAD_SHAPE", 2: "BAD_ALIGN", 3: "BAD_ARCH", 4: "DEVICE_TIMEOUT", 5: "CUDA_ERR", 6: "BAD_ARG"}

_lib = None
_path: Path | None = None


class TfbError(RuntimeError):
    """A libtfb entry point returned a non-OK status."""


def lib_path(directory: str | os.PathLike | None = None) -> Path:
    root = Path(directory or os.environ.get("TFIMAGE_EXT_DIR") or DEFAULT_DIR)
    return root / LIB_NAME


def load(directory: str | os.PathLike | None = None):
    """Load libtfb.so once (from ``directory``, ``$TFIMAGE_EXT_DIR`` or this package) and bind its symbols."""
    global _lib, _path
    if _lib is not None and (directory is None or lib_path(directory) == _path):
        return _lib
    path = lib_path(directory)
    if not path.is_file():
        raise TfbError(f"{path} not found: build it with qwen-image21-tensorfold-rtx_b200/build.py "
                       f"(there is no fallback path)")
    lib = ctypes.CDLL(str(path))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, c_int)
    _lib, _path = lib, path
    return lib


def check(status: int) -> None:
    if status != 0:
        msg = load().tfb_last_error().decode(errors="replace")
        raise TfbError(f"libtfb {STATUS.get(status, status)}: {msg}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise TfbError("libtfb ops take CUDA tensors (there is no CPU path)")


def sf_tiled_bytes(rows: int, k: int) -> int:
    return int(load().tfb_sf_tiled_bytes(rows, k))


def device_status(reset: bool = True) -> int:
    code = c_int(0)
    st = load().tfb_device_status(ctypes.byref(code), int(reset))
    if st not in (0, 4):
        check(st)
    return code.value


# ----------------------------------------------------------------------------------------------- tensor wrappers
def absmax(x: torch.Tensor) -> torch.Tensor:
    """Device fp32 scalar amax(|x|) of a bf16 tensor (contiguous)."""
    _cuda(x)
    x = x.contiguous()
    out = torch.empty((), dtype=torch.float32, device=x.device)
    check(load().tfb_absmax_bf16(x.data_ptr(), x.numel(), out.data_ptr(), _stream(x)))
    return out


def fp8_act_scale(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _cuda(x)
    x = x.contiguous()
    out = torch.empty((), dtype=torch.float32, device=x.device) if out is None else out
    check(load().tfb_fp8_act_scale(x.data_ptr(), x.numel(), out.data_ptr(), _stream(x)))
    return out


def quant_nvfp4(x: torch.Tensor, g: float, layout: int = SF_TILED, codes=None, sf=None):
    """bf16 [M, K] -> (codes uint8 [M, K/2], scales uint8: [M, K/16] rows or tiled bytes)."""
    _cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TfbError("quant_nvfp4 takes a 2-D bf16 tensor with unit column stride")
    M, K = x.shape
    if codes is None:
        codes = torch.empty((M, K // 2), dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = (torch.empty((max(sf_tiled_bytes(M, K), 0),), dtype=torch.uint8, device=x.device) if layout == SF_TILED
              else torch.empty((M, K // 16), dtype=torch.uint8, device=x.device))
    check(load().tfb_quant_nvfp4(x.data_ptr(), M, K, x.stride(0), float(g), codes.data_ptr(), sf.data_ptr(), layout,
                                 _stream(x)))
    return codes, sf


def quant_fp8(x: torch.Tensor, a: torch.Tensor, out=None) -> torch.Tensor:
    _cuda(x, a)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TfbError("quant_fp8 takes a 2-D bf16 tensor with unit column stride")
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.uint8, device=x.device) if out is None else out
    check(load().tfb_quant_fp8(x.data_ptr(), M, K, x.stride(0), a.data_ptr(), q.data_ptr(), _stream(x)))
    return q


def gemm_nvfp4(a_codes, a_sf, b_codes, b_sf, M: int, N: int, K: int, alpha: float, out=None) -> torch.Tensor:
    _cuda(a_codes, a_sf, b_codes, b_sf)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=a_codes.device) if out is None else out
    check(load().tfb_gemm_nvfp4(a_codes.data_ptr(), a_sf.data_ptr(), b_codes.data_ptr(), b_sf.data_ptr(), M, N, K,
                                float(alpha), y.data_ptr(), y.stride(0), _stream(a_codes)))
    return y


def gemm_nvfp4_resid(a_codes, a_sf, b_codes, b_sf, M: int, N: int, K: int, alpha: float, x: torch.Tensor,
                     gate: torch.Tensor, rows_per_gate: int) -> torch.Tensor:
    """x[m, :] = bf16(fma(bf16(alpha * acc[m, :]), gate[m // rows_per_gate, :], x[m, :])) in place; x bf16 [M, N]
    rows (unit column stride), gate bf16 [G, N] rows (unit column stride)."""
    _cuda(a_codes, a_sf, b_codes, b_sf, x, gate)
    if x.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16 or x.stride(-1) != 1 or gate.stride(-1) != 1:
        raise TfbError("gemm_nvfp4_resid: x and gate must be bf16 rows with unit column stride")
    check(load().tfb_gemm_nvfp4_resid(a_codes.data_ptr(), a_sf.data_ptr(), b_codes.data_ptr(), b_sf.data_ptr(), M, N,
                                      K, float(alpha), x.data_ptr(), x.stride(0), gate.data_ptr(), gate.stride(0),
                                      int(rows_per_gate), _stream(x)))
    return x


def gemm_nvfp4_qkv(a_codes, a_sf, b_codes, b_sf, B: int, ntok: int, H: int, K: int, alpha: float, wq, wk, cos, sin,
                   eps: float, q, k, v) -> None:
    """qkv GEMM with q / k RMSNorm + RoPE and the v copy in the epilogue; q, k, v [B, ntok, H, 128] views (rows of
    H * 128 contiguous)."""
    _cuda(a_codes, a_sf, b_codes, b_sf, wq, wk, cos, sin, q, k, v)
    check(load().tfb_gemm_nvfp4_qkv(a_codes.data_ptr(), a_sf.data_ptr(), b_codes.data_ptr(), b_sf.data_ptr(), B, ntok,
                                    H, K, float(alpha), wq.data_ptr(), wk.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                    float(eps), q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0),
                                    k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), _stream(a_codes)))


def gemm_fp8(a8, b8, M: int, N: int, K: int, a_scale, b_scale, out=None) -> torch.Tensor:
    _cuda(a8, b8, a_scale, b_scale)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=a8.device) if out is None else out
    per_channel = int(b_scale.numel() > 1)
    check(load().tfb_gemm_fp8(a8.data_ptr(), b8.data_ptr(), M, N, K, a_scale.data_ptr(), b_scale.data_ptr(),
                              per_channel, y.data_ptr(), y.stride(0), _stream(a8)))
    return y


def gemm_nvfp4_swiglu(a_codes, a_sf, gu_codes, gu_sf, M: int, F: int, K: int, alpha: float, h_global: float,
                      h_codes=None, h_sf=None, gu_out=None, h_out=None):
    _cuda(a_codes, a_sf, gu_codes, gu_sf)
    dev = a_codes.device
    if h_codes is None:
        h_codes = torch.empty((M, F // 2), dtype=torch.uint8, device=dev)
    if h_sf is None:
        h_sf = torch.empty((sf_tiled_bytes(M, F),), dtype=torch.uint8, device=dev)
    check(load().tfb_gemm_nvfp4_swiglu(a_codes.data_ptr(), a_sf.data_ptr(), gu_codes.data_ptr(), gu_sf.data_ptr(), M, F,
                                       K, float(alpha), float(h_global), h_codes.data_ptr(), h_sf.data_ptr(),
                                       _ptr(gu_out), _ptr(h_out), _stream(a_codes)))
    return h_codes, h_sf


def mlp_nvfp4(x, F: int, act_x: float, gu_codes, gu_sf, g_gu: float, down_codes, down_sf, g_down: float,
              act_h: float, out=None, workspace=None) -> torch.Tensor:
    _cuda(x, gu_codes, gu_sf, down_codes, down_sf)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise TfbError("mlp_nvfp4 takes a contiguous 2-D bf16 tensor")
    M, K = x.shape
    dev = x.device
    y = torch.empty((M, K), dtype=torch.bfloat16, device=dev) if out is None else out
    ws = workspace or mlp_workspace(M, K, F, dev)
    check(load().tfb_mlp_nvfp4(x.data_ptr(), M, K, F, float(act_x), gu_codes.data_ptr(), gu_sf.data_ptr(), float(g_gu),
                               down_codes.data_ptr(), down_sf.data_ptr(), float(g_down), float(act_h), y.data_ptr(),
                               ws[0].data_ptr(), ws[1].data_ptr(), ws[2].data_ptr(), ws[3].data_ptr(), _stream(x)))
    return y


def mlp_workspace(M: int, K: int, F: int, device) -> tuple[torch.Tensor, ...]:
    """Caller-owned scratch of tfb_mlp_nvfp4: x codes/scales and hidden codes/scales."""
    u8 = dict(dtype=torch.uint8, device=device)
    return (torch.empty((M, K // 2), **u8), torch.empty((sf_tiled_bytes(M, K),), **u8),
            torch.empty((M, F // 2), **u8), torch.empty((sf_tiled_bytes(M, F),), **u8))


def mlp_nvfp4_static(x, F: int, act_x: float, gu_codes, gu_sf, g_gu: float, down_codes, down_sf, g_down: float,
                     act_h: float, out=None) -> torch.Tensor:
    """mlp_nvfp4 on the library's per-device static scratch (tfb_mlp_nvfp4_static): no workspace is allocated.
    Calls that may overlap on one device (different streams) must be serialised by the caller."""
    _cuda(x, gu_codes, gu_sf, down_codes, down_sf)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise TfbError("mlp_nvfp4_static takes a contiguous 2-D bf16 tensor")
    M, K = x.shape
    y = torch.empty((M, K), dtype=torch.bfloat16, device=x.device) if out is None else out
    check(load().tfb_mlp_nvfp4_static(x.data_ptr(), M, K, F, float(act_x), gu_codes.data_ptr(), gu_sf.data_ptr(),
                                      float(g_gu), down_codes.data_ptr(), down_sf.data_ptr(), float(g_down),
                                      float(act_h), y.data_ptr(), _stream(x)))
    return y


def adaln(x, scale, shift, eps: float, out=None, q_global: float | None = None, codes=None, sf=None):
    _cuda(x, scale, shift)
    B, N, D = x.shape
    check(load().tfb_adaln(x.data_ptr(), B, N, D, scale.data_ptr(), _ptr(shift), float(eps), _ptr(out),
                           float(q_global or 0.0), _ptr(codes), _ptr(sf), _stream(x)))


def rms_rope(src, part: int, w, cos, sin, eps: float, dst) -> None:
    _cuda(src, w, cos, sin, dst)
    B, N, _, H, D = src.shape
    check(load().tfb_rms_rope(src.data_ptr(), B, N, H, D, src.stride(0), src.stride(1), part * H * D, w.data_ptr(),
                              cos.data_ptr(), sin.data_ptr(), float(eps), dst.data_ptr(), dst.stride(0),
                              dst.stride(1), _stream(src)))


def rms_rope_qkv(src, wq, wk, cos, sin, eps: float, q, k, v) -> None:
    _cuda(src, wq, wk, cos, sin, q, k, v)
    B, N, _, H, D = src.shape
    check(load().tfb_rms_rope_qkv(src.data_ptr(), B, N, H, D, src.stride(0), src.stride(1), wq.data_ptr(),
                                  wk.data_ptr(), cos.data_ptr(), sin.data_ptr(), float(eps), q.data_ptr(), q.stride(0),
                                  q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0),
                                  v.stride(1), _stream(src)))


def swiglu(gu, out) -> None:
    _cuda(gu, out)
    M, F2 = gu.shape
    check(load().tfb_swiglu(gu.data_ptr(), M, F2 // 2, out.data_ptr(), _stream(gu)))


def gguf_block(kind: str) -> tuple[int, int]:
    """(values, bytes) per block of a GGUF type decoded here."""
    v = c_i64(0)
    b = load().tfb_gguf_block_bytes(GGUF_TYPES[kind], ctypes.byref(v))
    return int(v.value), int(b)


def gguf_dequant(kind: str, raw, out) -> None:
    """raw uint8 blocks of ``kind`` -> ``out`` (f32 / f16 / bf16, out.numel() values), on raw's stream."""
    _cuda(raw, out)
    if kind not in GGUF_TYPES:
        raise TfbError(f"GGUF type {kind} is not decoded here (decoded: {', '.join(GGUF_TYPES)})")
    if out.dtype not in OUT_DTYPES or not out.is_contiguous():
        raise TfbError("gguf_dequant: out must be a contiguous f32 / f16 / bf16 tensor")
    vals, nbytes = gguf_block(kind)
    if raw.numel() * vals != out.numel() * nbytes:
        raise TfbError(f"gguf_dequant: {raw.numel()} bytes of {kind} do not hold {out.numel()} values")
    check(load().tfb_gguf_dequant(GGUF_TYPES[kind], raw.data_ptr(), out.numel(), out.data_ptr(),
                                  OUT_DTYPES[out.dtype], _stream(raw)))


# ------------------------------------------------------------------ tensor-parallel down projection over NVLink
TP_MAX_WORLD = 8


class TpComm(ctypes.Structure):
    """tfb_tp_comm: every rank's communication buffer as mapped in this process, and the shape it was laid out for."""
    _fields_ = [("world", c_int), ("rank", c_int), ("base", c_vp * TP_MAX_WORLD), ("max_rows", c_i64),
                ("n_cols", c_i64)]


def tp_layout(world: int, max_rows: int, n_cols: int) -> tuple[int, list[int]]:
    """(bytes, [x, receive slots, partial counters, x counters, device epoch] offsets) of one rank's buffer."""
    off = (c_i64 * 5)()
    n = load().tfb_tp_layout(world, max_rows, n_cols, off)
    if n < 0:
        raise TfbError(f"tp_layout: bad arguments (world={world}, max_rows={max_rows}, n_cols={n_cols})")
    return int(n), [int(v) for v in off]


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """CUDA IPC handle (64 bytes) of the allocation holding ``t`` and t's byte offset inside it."""
    _cuda(t)
    h = (ctypes.c_uint8 * 64)()
    off = c_i64(0)
    check(load().tfb_ipc_handle(t.data_ptr(), h, ctypes.byref(off)))
    return bytes(h), int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Maps another process's allocation into this one; returns the device address at ``offset``."""
    h = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    ptr = c_vp(0)
    check(load().tfb_ipc_open(h, offset, ctypes.byref(ptr)))
    return int(ptr.value)


def ipc_close(ptr: int, offset: int) -> None:
    check(load().tfb_ipc_close(ptr, offset))


def gemm_nvfp4_tp(a_codes, a_sf, b_codes, b_sf, M: int, N: int, K: int, alpha: float, gate: torch.Tensor,
                  rows_per_gate: int, comm: TpComm, epoch: int) -> None:
    _cuda(a_codes, a_sf, b_codes, b_sf, gate)
    check(load().tfb_gemm_nvfp4_tp(a_codes.data_ptr(), a_sf.data_ptr(), b_codes.data_ptr(), b_sf.data_ptr(), M, N, K,
                                   float(alpha), gate.data_ptr(), gate.stride(0), rows_per_gate, ctypes.byref(comm),
                                   epoch, _stream(a_codes)))


def tp_wait(comm: TpComm, M: int, N: int, epoch: int, device) -> None:
    check(load().tfb_tp_wait(ctypes.byref(comm), M, N, epoch, torch.cuda.current_stream(device).cuda_stream))


def tp_advance(comm: TpComm, device) -> None:
    check(load().tfb_tp_advance(ctypes.byref(comm), torch.cuda.current_stream(device).cuda_stream))
