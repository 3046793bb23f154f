"""ctypes binding of the sm_100a C-ABI library (``lib/liblpc_b200.so``).

This is the only door to the GPU kernels.  There is no fallback: if the
library is missing or a call fails, the caller gets an exception.  Error
translation mirrors the reference bindings (src/csrc/ops/bindings.cpp:51-105):
invalid arguments raise ``ValueError`` (the reference throws
``std::invalid_argument``), unsupported dtypes/sizes raise ``TypeError``, CUDA
failures raise ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "liblpc_b200.so"

LPC_OK = 0
LPC_ERR_INVALID = 1
LPC_ERR_UNSUPPORTED = 2
LPC_ERR_CUDA = 3

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> (restype, argtypes); kept in the order of include/lpc_b200.h
SIGNATURES = {
    "lpc_version": (_I, []),
    "lpc_last_error": (ctypes.c_char_p, []),
    "lpc_device_status": (_I, []),
    "lpc_update_kv_cache": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I64, _I64, _I, _P]),
    "lpc_rope_forward": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _I, _I64, _I, _I, _P]),
    "lpc_rope_kv_append": (_I, [_P, _P, _P, _P, _I64, _P, _P, _P, _I64, _I64, _I, _I, _I, _I64,
                                _I64, _I, _I, _P]),
    "lpc_rmsnorm_forward": (_I, [_P, _P, _P, _I64, _I, _F, _I, _I, _P]),
    "lpc_rmsswiglu_workspace_bytes": (_I64, [_I64, _I, _I]),
    "lpc_rmsswiglu_forward": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _F, _I, _I, _P]),
    "lpc_flash_attention": (_I, [_P, _P, _P, _P, _I64, _I, _I, _I64, _I64, _I, _I64, _I64, _I, _F,
                                 _I, _P]),
    "lpc_rmsswiglu_folded_forward": (_I, [_P, _P, _P, _P, _I64, _I, _I, _F, _I, _P]),
    "lpc_decode_attention_workspace_bytes": (_I64, [_I64, _I, _I64, _I]),
    "lpc_decode_attention_split_keys": (_I, [_I64, _I, _I64, _I64]),
    "lpc_decode_attention": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I, _I64, _I64, _F,
                                  _I, _P]),
    "lpc_decode_attention_noalloc": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _I64, _I64, _F, _I,
                                          _P]),
    "lpc_rope_kv_append_ragged": (_I, [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I,
                                       _I, _I, _I64, _I, _I, _P]),
    "lpc_decode_attention_ragged": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I,
                                         _I64, _I64, _F, _I, _P]),
    "lpc_packed_weight_bytes": (_I64, [_I64, _I, _I]),
    "lpc_pack_weights": (_I, [_P, _P, _P, _P, _I64, _I, _I, _I, _P]),
    "lpc_wsgemm": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _I, _I, _F, _P]),
    "lpc_qkv_rope_append": (_I, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I, _I,
                                 _I, _I, _I64, _I64, _I64, _I, _I, _F, _P]),
    "lpc_hbm_read_probe": (_I, [_P, _I64, _P]),
}

_lib = None
_lock = threading.Lock()

# Number of kernels each entry point enqueues (for launch accounting).
KERNELS_PER_CALL = {
    "lpc_update_kv_cache": 1, "lpc_rope_forward": 1, "lpc_rope_kv_append": 1,
    "lpc_rmsnorm_forward": 1, "lpc_rmsswiglu_forward": 2, "lpc_flash_attention": 1,
    "lpc_decode_attention": 2, "lpc_decode_attention_noalloc": 2,
    "lpc_pack_weights": 1, "lpc_wsgemm": 1, "lpc_qkv_rope_append": 1, "lpc_rope_kv_append_ragged": 1,
    "lpc_decode_attention_ragged": 2, "lpc_rmsswiglu_folded_forward": 1, "lpc_hbm_read_probe": 1,
}
launch_count = 0


def decode_kernels(batch: int, kv_heads: int, max_seq_len: int, total_rows: int = 0) -> int:
    """Kernels one decode-attention call enqueues: none for an empty batch,
    the split kernel alone when one split covers the cache length, else the
    split and combine kernels (total_rows: the ragged cache's rows per KV
    head, 0 for the dense cache)."""
    if batch <= 0:
        return 0
    keys = load().lpc_decode_attention_split_keys(batch, kv_heads, max_seq_len, total_rows)
    return 1 if keys >= max_seq_len else 2


def count_launch(name: str, n: int | None = None) -> None:
    """Adds the kernels that a successful call of `name` enqueued to launch_count."""
    global launch_count
    launch_count += KERNELS_PER_CALL.get(name, 1) if n is None else n


class BackendUnavailable(RuntimeError):
    """The sm_100a library is not built or cannot be loaded."""


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Loads (once) and returns the library; raises BackendUnavailable if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise BackendUnavailable(
                f"{p} is missing: build it with `python -m llama_pure_compute_b200.csrc.build`")
        try:
            lib = ctypes.CDLL(str(p), mode=ctypes.RTLD_LOCAL)
        except OSError as e:  # pragma: no cover - depends on the host
            raise BackendUnavailable(f"cannot load {p}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def available() -> bool:
    try:
        load()
        return True
    except BackendUnavailable:
        return False


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc == LPC_OK:
        return
    msg = (load().lpc_last_error() or b"").decode(errors="replace")
    text = f"LlamaPureComputeError: {what}: {msg}"
    if rc == LPC_ERR_INVALID:
        raise ValueError(text)
    if rc == LPC_ERR_UNSUPPORTED:
        raise TypeError(text)
    raise RuntimeError(text)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(dt: torch.dtype, what: str) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"LlamaPureComputeError: {what}: unsupported dtype {dt}") from None


def device_status() -> int:
    """OR of device-side error flags since the last call (synchronises)."""
    v = load().lpc_device_status()
    if v < 0:
        check(LPC_ERR_CUDA, "device_status")
    return v
