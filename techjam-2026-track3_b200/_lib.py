"""ctypes binding of libtechjam_b200.so (the C ABI declared in include/techjam_b200.h).

Only plain pointers, ints and floats cross the boundary; torch tensors are
unwrapped here with ``data_ptr()`` and the current CUDA stream handle.  A
missing library or a non-B200 device raises: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtechjam_b200.so"

TJ_OK = 0
TJ_ERR_INVALID_ARGUMENT = 1
TJ_ERR_UNSUPPORTED = 2
TJ_ERR_CUDA = 3
TJ_ERR_DEVICE = 4
TJ_ERR_WORKSPACE = 5

TJ_WITHHOLD_NONE = 0
TJ_WITHHOLD_ATTN_P_READY = 1

_ERR_NAMES = {
    TJ_ERR_INVALID_ARGUMENT: "invalid argument",
    TJ_ERR_UNSUPPORTED: "unsupported",
    TJ_ERR_CUDA: "CUDA error",
    TJ_ERR_DEVICE: "device error",
    TJ_ERR_WORKSPACE: "workspace error",
}

c_int = ctypes.c_int
c_i64 = ctypes.c_int64
c_float = ctypes.c_float
c_vp = ctypes.c_void_p


class EncoderDesc(ctypes.Structure):
    _fields_ = [
        ("batch", c_int),
        ("seq_len", c_int),
        ("d_model", c_int),
        ("num_heads", c_int),
        ("ffn_dim", c_int),
        ("num_layers", c_int),
        ("causal", c_int),
        ("ln_eps", c_float),
    ]


class CopySegment(ctypes.Structure):
    _fields_ = [("dst", c_vp), ("src", c_vp), ("bytes", c_i64)]


TJ_IPC_HANDLE_BYTES = 64
TJ_PUSH_MAX_DST = 8
TJ_PUSH_MAX_SEGS = 64


class PushSegment(ctypes.Structure):
    _fields_ = [("dst_offset", c_i64), ("src", c_vp), ("bytes", c_i64)]


class LayerWeights(ctypes.Structure):
    _fields_ = [
        ("ln1_gamma", c_vp),
        ("ln1_beta", c_vp),
        ("w_qkv16", c_vp),
        ("b_qkv", c_vp),
        ("w_out16", c_vp),
        ("b_out", c_vp),
        ("ln2_gamma", c_vp),
        ("ln2_beta", c_vp),
        ("w_ffn_in16", c_vp),
        ("b_ffn_in", c_vp),
        ("w_ffn_out16", c_vp),
        ("b_ffn_out", c_vp),
    ]


# name -> (restype, argtypes); every symbol include/techjam_b200.h declares.
SIGNATURES = {
    "tj_abi_version": (c_int, []),
    "tj_last_error": (ctypes.c_char_p, []),
    "tj_get_last_error": (c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "tj_set_sync_check": (c_int, [c_int]),
    "tj_device_status": (c_int, [ctypes.POINTER(c_int), c_vp]),
    "tj_set_small_encoder": (c_int, [c_int]),
    "tj_debug_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "tj_debug_withhold_arrive": (c_int, [c_int]),
    "tj_token_plan_ints": (c_i64, [c_int, c_int]),
    "tj_token_plan": (c_int, [c_vp, c_int, c_int, c_vp, c_vp]),
    "tj_ln_cast_f16": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp]),
    "tj_ln_final_mask": (c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp]),
    "tj_add_ln_cast_f16": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp, c_vp],
    ),
    "tj_add2_ln_final_mask": (
        c_int,
        [c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp],
    ),
    "tj_add_ln_final_mask": (
        c_int,
        [c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp],
    ),
    "tj_gemm_qkv_headmajor": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "tj_gemm_bias_residual_f32": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp],
    ),
    "tj_gemm_bias_f16": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "tj_gemm_bias_gelu_f16": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_vp, c_vp]),
    "tj_flash_attn_fwd": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_i64, c_int, c_int, c_int,
            c_vp, c_vp, c_vp, c_float, c_int, c_vp, c_vp, c_vp,
        ],
    ),
    "tj_flash_attn_fwd_strided": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_i64, c_int, c_int, c_int,
            c_vp, c_vp, c_vp, c_float, c_int, c_vp, c_vp, c_i64, c_vp,
        ],
    ),
    "tj_flash_attn_fwd_partial": (
        c_int,
        [
            c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_i64, c_i64, c_int, c_int, c_int,
            c_vp, c_vp, c_vp, c_float, c_int, c_vp, c_vp, c_i64, c_vp, c_vp, c_int, c_vp,
        ],
    ),
    "tj_encoder_workspace_bytes": (c_i64, [ctypes.POINTER(EncoderDesc)]),
    "tj_encoder_forward": (
        c_int,
        [
            ctypes.POINTER(EncoderDesc), ctypes.POINTER(LayerWeights), c_vp, c_vp, c_vp, c_vp,
            c_vp, c_vp, c_i64, c_vp,
        ],
    ),
    "tj_ipc_export": (c_int, [c_vp, c_vp, ctypes.POINTER(c_i64)]),
    "tj_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "tj_ipc_close": (c_int, [c_vp]),
    "tj_copy_segments": (c_int, [ctypes.POINTER(CopySegment), c_int, c_vp]),
    "tj_push_segments": (c_int, [ctypes.POINTER(c_vp), c_int, ctypes.POINTER(PushSegment), c_int, c_int, c_vp]),
    "tj_encoder_forward_noalloc": (
        c_int,
        [ctypes.POINTER(EncoderDesc), ctypes.POINTER(LayerWeights), c_vp, c_vp, c_vp, c_vp, c_vp, c_vp],
    ),
}

_lib = None
_lock = threading.Lock()


class TJError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, op: str, code: int, message: str) -> None:
        super().__init__(f"{op}: {_ERR_NAMES.get(code, 'error')} ({code}): {message}")
        self.op = op
        self.code = code


def load(path: Path | None = None) -> ctypes.CDLL:
    """Loads the shared library once and declares every entry point."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        lib_path = Path(path) if path is not None else LIB_PATH
        if not lib_path.exists():
            raise RuntimeError(
                f"{lib_path.name} is not built; run `python {PKG_DIR.name}/build.py` "
                "(or __graft_entry__.build()) first"
            )
        lib = ctypes.CDLL(str(lib_path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().tj_last_error()
    return msg.decode() if msg else ""


def check(rc: int, op: str) -> None:
    if rc != TJ_OK:
        raise TJError(op, rc, last_error())


_sync_check = False


def set_sync_check(enabled: bool) -> bool:
    """Turns the library's per-call synchronise + device-status check on or
    off (tests, debugging); returns the previous setting."""
    global _sync_check
    _sync_check = bool(enabled)
    return bool(load().tj_set_sync_check(1 if enabled else 0))


def sync_check_enabled() -> bool:
    return _sync_check


def device_status(stream: int = 0) -> list[int]:
    out = (c_int * 4)()
    rc = load().tj_device_status(out, c_vp(stream))
    status = list(out)
    if rc == TJ_ERR_DEVICE:
        raise TJError("device_status", rc, last_error())
    check(rc, "device_status")
    return status


# ---- peer exchange ------------------------------------------------------------
def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(handle bytes, byte offset of ptr in its allocation) for the peers."""
    h = ctypes.create_string_buffer(TJ_IPC_HANDLE_BYTES)
    off = c_i64(0)
    check(load().tj_ipc_export(c_vp(ptr), h, ctypes.byref(off)), "ipc_export")
    return h.raw, int(off.value)


def ipc_open(handle: bytes) -> int:
    """Maps a peer allocation; returns its base address in this process."""
    if len(handle) != TJ_IPC_HANDLE_BYTES:
        raise ValueError("IPC handle must be %d bytes" % TJ_IPC_HANDLE_BYTES)
    base = c_vp()
    check(load().tj_ipc_open(ctypes.create_string_buffer(handle, TJ_IPC_HANDLE_BYTES), ctypes.byref(base)),
          "ipc_open")
    return int(base.value)


def ipc_close(base: int) -> None:
    check(load().tj_ipc_close(c_vp(base)), "ipc_close")


def copy_segments(segments, stream: int) -> None:
    """Enqueues (dst, src or 0 for a zero fill, bytes) copies on `stream`."""
    n = len(segments)
    if n == 0:
        return
    arr = (CopySegment * n)()
    for i, (dst, src, nbytes) in enumerate(segments):
        arr[i].dst = dst
        arr[i].src = src or None
        arr[i].bytes = nbytes
    check(load().tj_copy_segments(arr, n, c_vp(stream)), "copy_segments")


def push_segments(dst_bases, segments, stream: int, blocks: int = 0) -> None:
    """One kernel copying each (dst_offset, src, bytes) segment to every
    destination base address (at most TJ_PUSH_MAX_SEGS per call)."""
    if not segments:
        return
    dst = (c_vp * len(dst_bases))(*dst_bases)
    for i in range(0, len(segments), TJ_PUSH_MAX_SEGS):
        part = segments[i : i + TJ_PUSH_MAX_SEGS]
        arr = (PushSegment * len(part))()
        for k, (off, src, nbytes) in enumerate(part):
            arr[k].dst_offset = off
            arr[k].src = src
            arr[k].bytes = nbytes
        check(load().tj_push_segments(dst, len(dst_bases), arr, len(part), blocks, c_vp(stream)), "push_segments")
