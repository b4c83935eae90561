"""ctypes binding of libema_ssd_b200.so (the C ABI in include/ema_ssd_b200.h).

The shared library is the only compute path: there is no Triton, no PyTorch
fallback and no CPU path.  Importing this module raises ImportError when the
library has not been built (``python ema-kernels_b200/build.py``).

Scratch memory: the EMA scan kernels need a zero-initialised workspace for
their inter-CTA look-back.  :func:`workspace` keeps one per (device, stream),
allocated through PyTorch's caching allocator and grown by powers of two.  A
buffer a CUDA graph capture used is never freed while the process lives, so
captured graphs stay valid; launches on different streams never share one.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libema_ssd_b200.so")

if not os.path.exists(_LIB_PATH):
    raise ImportError(
        f"{_LIB_PATH} is missing: build the CUDA library with `python ema-kernels_b200/build.py` "
        "(there is no fallback implementation)")

lib = ctypes.CDLL(_LIB_PATH)

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
IDX_CODES = {torch.int8: 1, torch.int32: 2, torch.int64: 3}

EMA_OK = 0
ERR_NAMES = {1: "invalid argument", 2: "unsupported", 3: "workspace", 4: "CUDA error"}
DEVSTATUS_LOOKBACK_TIMEOUT = 1
DEVSTATUS_TMA_TIMEOUT = 2

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_ptr = ctypes.c_void_p


class EmaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64), ("chunk_size", _i64),
        ("dtype", _i32), ("seq_idx_type", _i32),
        ("x", _ptr), ("x_stride", _i64 * 3),
        ("out", _ptr), ("out_stride", _i64 * 3),
        ("dA", _ptr), ("dt", _ptr), ("A", _ptr), ("seq_idx", _ptr), ("initial_state", _ptr),
        ("states", _ptr), ("states_stride", _i64 * 4),
        ("da_cs", _ptr), ("da_cs_sum", _ptr), ("final_state", _ptr),
        ("workspace", _ptr), ("workspace_bytes", ctypes.c_size_t),
        ("mid_states", _ptr), ("mid_states_stride", _i64 * 4),
        ("dt_rows", _ptr),
    ]


class EmaBwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64), ("chunk_size", _i64),
        ("dtype", _i32), ("reserved", _i32),
        ("x", _ptr), ("x_stride", _i64 * 3),
        ("dout", _ptr), ("dout_stride", _i64 * 3),
        ("dx", _ptr), ("dx_stride", _i64 * 3),
        ("da_cs", _ptr), ("da_cs_sum", _ptr), ("dt", _ptr), ("A", _ptr),
        ("states", _ptr), ("states_stride", _i64 * 4),
        ("d_final_state", _ptr), ("d_last_token", _ptr),
        ("dl", _ptr), ("ddt", _ptr), ("dA_out", _ptr), ("d_initial_state", _ptr),
        ("workspace", _ptr), ("workspace_bytes", ctypes.c_size_t),
        ("dt_rows", _ptr),
    ]


class SsdFwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64), ("dstate", _i64), ("ngroups", _i64),
        ("dtype", _i32), ("reserved", _i32),
        ("x", _ptr), ("x_stride", _i64 * 3),
        ("dt", _ptr), ("A", _ptr),
        ("B", _ptr), ("B_stride", _i64 * 3),
        ("C", _ptr), ("C_stride", _i64 * 3),
        ("D", _ptr), ("initial_state", _ptr),
        ("out", _ptr), ("out_stride", _i64 * 3),
        ("chunk_states", _ptr), ("final_state", _ptr),
        ("dt_bias", _ptr), ("dt_softplus", _i32), ("dt_clamp", _i32), ("dt_min", ctypes.c_float),
        ("dt_max", ctypes.c_float),
    ]


class SsdBwdArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64), ("dstate", _i64), ("ngroups", _i64),
        ("dtype", _i32), ("reserved", _i32),
        ("x", _ptr), ("x_stride", _i64 * 3),
        ("dt", _ptr), ("A", _ptr),
        ("B", _ptr), ("B_stride", _i64 * 3),
        ("C", _ptr), ("C_stride", _i64 * 3),
        ("D", _ptr), ("chunk_states", _ptr),
        ("dout", _ptr), ("dout_stride", _i64 * 3),
        ("d_final_state", _ptr),
        ("dx", _ptr), ("dx_stride", _i64 * 3),
        ("ddt", _ptr), ("dA", _ptr), ("dB", _ptr), ("dC", _ptr), ("dD", _ptr), ("d_initial_state", _ptr),
        ("dt_bias", _ptr), ("dt_softplus", _i32), ("dt_clamp", _i32), ("dt_min", ctypes.c_float),
        ("dt_max", ctypes.c_float), ("ddt_bias", _ptr),
    ]


class SsdGateArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64),
        ("dtype", _i32), ("reserved", _i32),
        ("y", _ptr), ("y_stride", _i64 * 3),
        ("z", _ptr), ("z_stride", _i64 * 3),
        ("out", _ptr), ("out_stride", _i64 * 3),
        ("dout", _ptr), ("dout_stride", _i64 * 3),
        ("dz", _ptr), ("dz_stride", _i64 * 3),
    ]


class EmaSpanFoldArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("subspans", _i64), ("nheads", _i64), ("headdim", _i64),
        ("direction", _i32), ("reserved", _i32),
        ("log_decay", _ptr), ("values", _ptr), ("boundary", _ptr), ("out", _ptr), ("span_decay", _ptr),
    ]


SPAN_EXCHANGE_MAX_RANKS = 8
P2P_HANDLE_BYTES = 64


class EmaSpanExchangeArgs(ctypes.Structure):
    _fields_ = [
        ("batch", _i64), ("subspans", _i64), ("nheads", _i64), ("headdim", _i64),
        ("direction", _i32), ("rank", _i32), ("world", _i32), ("reserved", _i32),
        ("log_decay", _ptr), ("values", _ptr), ("boundary", _ptr), ("span_in", _ptr), ("out", _ptr),
        ("buffer_bytes", ctypes.c_uint64), ("buffers", _ptr * SPAN_EXCHANGE_MAX_RANKS),
    ]


class EmaSpanStateArgs(ctypes.Structure):
    _fields_ = [
        ("rows", _i64), ("seqlen", _i64), ("nheads", _i64), ("headdim", _i64),
        ("dtype", _i32), ("direction", _i32),
        ("x", _ptr), ("x_stride", _i64 * 3),
        ("dt", _ptr), ("A", _ptr), ("out", _ptr), ("log_decay", _ptr),
    ]


lib.ema_scan_workspace_size.restype = ctypes.c_size_t
lib.ema_scan_workspace_size.argtypes = [_i64] * 5
lib.ema_fwd_launch.restype = ctypes.c_int
lib.ema_fwd_launch.argtypes = [ctypes.POINTER(EmaFwdArgs), _ptr]
lib.ema_bwd_launch.restype = ctypes.c_int
lib.ema_bwd_launch.argtypes = [ctypes.POINTER(EmaBwdArgs), _ptr]
lib.chunk_cumsum_launch.restype = ctypes.c_int
lib.chunk_cumsum_launch.argtypes = [_ptr, ctypes.POINTER(_i64), _ptr, ctypes.POINTER(_i64), _ptr,
                                    ctypes.POINTER(_i64), _i64, _i64, _i64, _i64, _i32, _ptr]
lib.ema_dt_rows_launch.restype = ctypes.c_int
lib.ema_dt_rows_launch.argtypes = [_ptr, _ptr, _i64, _i64, _i64, _ptr]
lib.ema_workspace_status.restype = ctypes.c_int
lib.ema_workspace_status.argtypes = [_ptr, ctypes.POINTER(ctypes.c_uint32), _ptr]
lib.ema_workspace_clear_status.restype = ctypes.c_int
lib.ema_workspace_clear_status.argtypes = [_ptr, _ptr]
lib.ema_set_tensor_core_path.restype = ctypes.c_int
lib.ema_set_tensor_core_path.argtypes = [ctypes.c_int32]
lib.ssd_internal_chunks.restype = _i64
lib.ssd_internal_chunks.argtypes = [_i64]
lib.ssd_fwd_launch.restype = ctypes.c_int
lib.ssd_fwd_launch.argtypes = [ctypes.POINTER(SsdFwdArgs), _ptr]
lib.ssd_bwd_launch.restype = ctypes.c_int
lib.ssd_bwd_launch.argtypes = [ctypes.POINTER(SsdBwdArgs), _ptr]
lib.ssd_gate_fwd_launch.restype = ctypes.c_int
lib.ssd_gate_fwd_launch.argtypes = [ctypes.POINTER(SsdGateArgs), _ptr]
lib.ssd_gate_bwd_launch.restype = ctypes.c_int
lib.ssd_gate_bwd_launch.argtypes = [ctypes.POINTER(SsdGateArgs), _ptr]
lib.ema_span_summary.restype = ctypes.c_int
lib.ema_span_summary.argtypes = [ctypes.POINTER(EmaSpanFoldArgs), _ptr]
lib.ema_span_expand.restype = ctypes.c_int
lib.ema_span_expand.argtypes = [ctypes.POINTER(EmaSpanFoldArgs), _ptr]
lib.ema_span_state_launch.restype = ctypes.c_int
lib.ema_span_state_launch.argtypes = [ctypes.POINTER(EmaSpanStateArgs), _ptr]
lib.ema_span_exchange_bytes.restype = ctypes.c_size_t
lib.ema_span_exchange_bytes.argtypes = [_i64, _i64, _i64]
lib.ema_span_exchange.restype = ctypes.c_int
lib.ema_span_exchange.argtypes = [ctypes.POINTER(EmaSpanExchangeArgs), _ptr]
lib.ema_span_exchange_status.restype = ctypes.c_int
lib.ema_span_exchange_status.argtypes = [_ptr, ctypes.POINTER(ctypes.c_uint32), _i32]
lib.ema_p2p_alloc.restype = ctypes.c_int
lib.ema_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
lib.ema_p2p_free.restype = ctypes.c_int
lib.ema_p2p_free.argtypes = [_ptr]
lib.ema_p2p_handle.restype = ctypes.c_int
lib.ema_p2p_handle.argtypes = [_ptr, ctypes.POINTER(ctypes.c_ubyte)]
lib.ema_p2p_open.restype = ctypes.c_int
lib.ema_p2p_open.argtypes = [ctypes.POINTER(ctypes.c_ubyte), ctypes.POINTER(ctypes.c_void_p)]
lib.ema_p2p_close.restype = ctypes.c_int
lib.ema_p2p_close.argtypes = [_ptr]
lib.ssd_device_status.restype = ctypes.c_int
lib.ssd_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, _ptr]
lib.ema_last_error.restype = ctypes.c_char_p
lib.ema_version.restype = ctypes.c_char_p


class EmaLaunchError(RuntimeError):
    pass


def check(code: int, what: str):
    if code != EMA_OK:
        msg = lib.ema_last_error().decode(errors="replace")
        raise EmaLaunchError(f"{what}: {ERR_NAMES.get(code, code)}: {msg}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


# --------------------------------------------------------------------------
# workspaces
# --------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws: dict = {}
_ws_captured: set = set()  # keys whose current buffer was handed to a CUDA graph capture
_ws_retired: list = []     # replaced buffers a captured graph may still launch with


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch of at least ``nbytes`` for the current stream of ``device``.

    Sizes grow by powers of two (at least 1 MiB), so a process replaces a
    stream's buffer only a few times.  A replaced buffer is kept alive only if
    a CUDA graph capture used it (the graph holds its address); otherwise it
    returns to PyTorch's caching allocator, which reuses memory in stream order,
    so kernels still queued on this stream finish with it first."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr(device))
    capturing = torch.cuda.is_current_stream_capturing()
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None and key in _ws_captured:
                _ws_retired.append(buf)
            _ws_captured.discard(key)
            size = 1 << max(20, (max(nbytes, 1) - 1).bit_length())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            _ws[key] = buf
        if capturing:
            _ws_captured.add(key)
        return buf


def device_status(clear: bool = False) -> int:
    """OR of the status words of every workspace (synchronises).  Non-zero means a
    device-side wait timed out (EMA_DEVSTATUS_* bits) and results are invalid."""
    st = 0
    with _ws_lock:
        bufs = list(_ws.items())
    for (dev, sp), buf in bufs:
        with torch.cuda.device(dev):
            torch.cuda.synchronize(dev)
            v = int(buf[12:16].view(torch.int32).item())
            st |= v
            if clear and v:
                buf[12:16].zero_()
    return st


def tma_ok(t: torch.Tensor) -> bool:
    """True when ``t`` (B, L, H, P) can be addressed by a TMA tile map as is."""
    if t.stride(-1) != 1 or t.data_ptr() % 16:
        return False
    es = t.element_size()
    return all(s > 0 and (s * es) % 16 == 0 for s in t.stride()[:3])


def tma_ready(t: torch.Tensor) -> torch.Tensor:
    return t if tma_ok(t) else t.contiguous()


def strides3(t: torch.Tensor):
    s = t.stride()
    return (_i64 * 3)(s[0], s[1], s[2])
