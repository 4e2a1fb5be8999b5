"""Loading of the in-tree native libraries.

There is deliberately no fallback: if ``libmlora_b200.so`` or the
``torch.ops.mlora`` binding cannot be loaded, every op raises. Build them with
``python -m multi_lora_b200.build``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
CUDA_LIB_PATH = PKG / "libmlora_b200.so"
TORCH_LIB_PATH = PKG / "_mlora_torch.so"

# dtype codes of include/mlora_b200.h
DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_lock = threading.Lock()
_capi = None
_ops_loaded = False


class NativeLibraryError(RuntimeError):
    """The CUDA extension is missing or failed to load."""


class PeerExchangeT(ctypes.Structure):
    """ctypes mirror of ``mlora_peer_exchange_t``."""

    _fields_ = [
        ("tp", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("max_rows", ctypes.c_int32),
        ("max_rank", ctypes.c_int32),
        ("buffers", ctypes.c_void_p * 8),
    ]


class MetadataT(ctypes.Structure):
    """ctypes mirror of ``mlora_kernel_input_metadata_t``."""

    _fields_ = [
        ("bs", ctypes.c_int32),
        ("max_len", ctypes.c_int32),
        ("num_slots", ctypes.c_int32),
        ("scalings_dtype", ctypes.c_int32),
        ("seg_lens", ctypes.c_void_p),
        ("seg_indptr", ctypes.c_void_p),
        ("weight_indices", ctypes.c_void_p),
        ("lora_ranks", ctypes.c_void_p),
        ("scalings", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32

# name -> (restype, argtypes); the exported symbols of include/mlora_b200.h
CAPI_SIGNATURES = {
    "mlora_sgemm_lora_a_fwd": (_I32, [_P, _I64, _I64, _I64, _P, _I64, ctypes.POINTER(MetadataT), _P, _I64, _I32,
                                      _I32, _I32, _P, _P]),
    "mlora_sgemm_lora_b_fwd": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _I64, ctypes.POINTER(MetadataT), _P, _I64,
                                      _I32, _P, _P]),
    "mlora_apply_lora": (_I32, [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, ctypes.POINTER(MetadataT), _P, _I64, _P,
                                _I64, _I32, _P, _P]),
    "mlora_apply_lora_group": (_I32, [_P, _I64, _I64, _I64, _I32, ctypes.POINTER(_P), ctypes.POINTER(_P),
                                      ctypes.POINTER(_I64), ctypes.POINTER(_P), ctypes.POINTER(_I64), _I64,
                                      ctypes.POINTER(MetadataT), _P, _I64, _I32, _P, _P]),
    "mlora_apply_lora_group_noalloc": (_I32, [_P, _I64, _I64, _I64, _I32, ctypes.POINTER(_P), ctypes.POINTER(_P),
                                              ctypes.POINTER(_I64), ctypes.POINTER(_P), ctypes.POINTER(_I64), _I64,
                                              ctypes.POINTER(MetadataT), _I32, _P, _P]),
    "mlora_rmsnorm_fwd": (_I32, [_P, _I64, _I64, _I64, _I64, _I64, _P, _I32, _P, _I64, ctypes.c_float, _I32, _P]),
    "mlora_fused_add_rmsnorm_fwd": (_I32, [_P, _I64, _P, _I64, _I64, _I64, _P, _I32, _P, _I64, ctypes.c_float,
                                           _I32, _P]),
    "mlora_scatter_stage": (_I32, [_P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P]),
    "mlora_peer_exchange_bytes": (ctypes.c_size_t, [_I32, _I32, _I32]),
    "mlora_peer_buffer_create": (_I32, [ctypes.c_size_t, ctypes.POINTER(_P), _P]),
    "mlora_peer_buffer_open": (_I32, [_P, ctypes.POINTER(_P)]),
    "mlora_peer_buffer_close": (_I32, [_P]),
    "mlora_peer_buffer_destroy": (_I32, [_P]),
    "mlora_row_parallel_apply_p2p": (_I32, [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, ctypes.POINTER(MetadataT), _P,
                                            _I64, _P, _I32, _I32, _P, _P]),
    "mlora_set_pdl": (None, [ctypes.c_int]),
    "mlora_get_pdl": (ctypes.c_int, []),
    "mlora_last_error": (ctypes.c_char_p, []),
    "mlora_version": (ctypes.c_int, []),
    "mlora_last_apply_path": (ctypes.c_int, []),
    "mlora_set_apply_path": (None, [ctypes.c_int]),
    "mlora_get_apply_path": (ctypes.c_int, []),
}

# mlora_set_apply_path codes
APPLY_PATHS = {"auto": 0, "fused": 1, "split": 2, "stream": 3, "tc": 4}


def capi() -> ctypes.CDLL:
    """The C ABI library with argument types declared."""
    global _capi
    with _lock:
        if _capi is None:
            if not CUDA_LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{CUDA_LIB_PATH.name} not built; run `python -m multi_lora_b200.build`")
            try:
                lib = ctypes.CDLL(str(CUDA_LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the box
                raise NativeLibraryError(f"cannot load {CUDA_LIB_PATH}: {e}") from e
            for name, (res, args) in CAPI_SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _capi = lib
    return _capi


def ops():
    """``torch.ops.mlora`` (loads the binding on first use)."""
    global _ops_loaded
    with _lock:
        if not _ops_loaded:
            if not TORCH_LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{TORCH_LIB_PATH.name} not built; run `python -m multi_lora_b200.build`")
            # load the C ABI first so the binding resolves it from this directory
            ctypes.CDLL(str(CUDA_LIB_PATH), mode=ctypes.RTLD_GLOBAL)
            torch.ops.load_library(str(TORCH_LIB_PATH))
            _ops_loaded = True
    return torch.ops.mlora


def check(rc: int) -> None:
    """Raise RuntimeError with the library's message for a non-zero return code."""
    if rc != 0:
        msg = capi().mlora_last_error()
        raise RuntimeError(f"mlora: {msg.decode() if msg else 'error'} (code {rc})")


def set_pdl(enable: bool) -> None:
    """Turn programmatic dependent launch on or off for later launches."""
    capi().mlora_set_pdl(1 if enable else 0)


def get_pdl() -> bool:
    return bool(capi().mlora_get_pdl())


def set_apply_path(name: str) -> None:
    """Force the apply_lora path tried first: "auto", "fused", "split", "stream" or "tc"."""
    capi().mlora_set_apply_path(APPLY_PATHS[name])


def get_apply_path() -> str:
    code = capi().mlora_get_apply_path()
    return next(k for k, v in APPLY_PATHS.items() if v == code)


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"mlora: unsupported dtype {dtype}") from None


def meta_struct(meta) -> MetadataT:
    """``mlora_kernel_input_metadata_t`` for a :class:`KernelInputMetaData` (device int32 tables)."""
    m = MetadataT()
    m.bs, m.max_len = int(meta.bs), int(meta.max_len)
    m.num_slots = int(meta.lora_ranks.numel())
    m.scalings_dtype = DTYPE_CODE[meta.scalings.dtype]
    m.seg_lens = meta.seg_lens.data_ptr()
    m.seg_indptr = meta.seg_indptr.data_ptr()
    m.weight_indices = meta.weight_indices.data_ptr()
    m.lora_ranks = meta.lora_ranks.data_ptr()
    m.scalings = meta.scalings.data_ptr()
    return m
