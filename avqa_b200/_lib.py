"""ctypes binding of the in-tree CUDA library (C ABI in include/avqa_b200.h).

The library is ``avqa_b200/libavqa_b200.so``; there is no fallback: if it is
missing, every CUDA call raises :class:`BackendError`.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

from avqa_b200.exceptions import BackendError

LIB_PATH = Path(__file__).resolve().parent / "libavqa_b200.so"
DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_Z = ctypes.c_size_t
_L = ctypes.c_longlong

_SIGS = {
    "avq_version": ([], ctypes.c_char_p),
    "avq_last_error": ([ctypes.c_char_p, _I], _I),
    "avq_prepare_codebook": ([_I, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P], _I),
    "avq_quantize_workspace_size": ([_I, _I, _I, _I], _Z),
    "avq_quantize": ([_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                      _P, _P, _P, _Z, _P], _I),
    "avq_selection_stride": ([_I, _I, _F], _I),
    "avq_forward_workspace_size": ([_I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I], _Z),
    "avq_dense_attention": ([_I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P], _I),
    "avq_bcar_workspace_size": ([_I, _I, _I, _I, _I], _Z),
    "avq_bcar_update": ([_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _Z, _P], _I),
    "avq_stream_workspace_size": ([_I, _I, _I, _I], _Z),
    "avq_stream_extend": ([_I, _P, _L, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _L, _L, _P, _P, _P, _P, _P, _Z,
                           _P], _I),
    "avq_presence_words": ([_I], _I),
    "avq_codeword_presence": ([_P, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P, _P, _Z, _P], _I),
    "avq_presence_workspace_size": ([_I, _I, _I], _Z),
    "avq_forward": ([_I, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _I, _I, _F, _I, _F,
                     _F, _P, _P, _P, _P, _P, _P, _Z, _P], _I),
    "avq_append_workspace_size": ([_I, _I, _I], _Z),
    "avq_append": ([_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                    _P, _I, _P, _Z, _P], _I),
    "avq_reduce_min": ([_P, _I, _P, _P], _I),
    "avq_device_fault": ([_P, _P], _I),
    "avq_quantize_noalloc": ([_I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                              _P, _P, _P, _P, _P], _I),
    "avq_profile_begin": ([], _I),
    "avq_profile_end": ([ctypes.c_char_p, _I, _P, _P, _I], _I),
}


def profile_begin() -> None:
    load().avq_profile_begin()


def profile_end() -> dict[str, tuple[float, int]]:
    """Per-kernel (total ms, launches) recorded since :func:`profile_begin`."""
    names = ctypes.create_string_buffer(4096)
    ms = (ctypes.c_float * 64)()
    cnt = (ctypes.c_int * 64)()
    n = load().avq_profile_end(names, len(names), ctypes.addressof(ms), ctypes.addressof(cnt), 64)
    if n < 0:
        raise BackendError(f"avq_profile_end failed: {last_error()}")
    keys = names.value.decode().split("\n")[:n]
    return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(keys)}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once; raise BackendError when it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("AVQA_B200_LIB", LIB_PATH))
    if not path.exists():
        raise BackendError("CUDA library not built: run `python -m avqa_b200.build_ext`", {"path": str(path)})
    try:
        lib = ctypes.CDLL(str(path))
    except OSError as exc:
        raise BackendError(f"cannot load the CUDA library: {exc}", {"path": str(path)}) from exc
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().avq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise BackendError(f"{what} failed: {last_error()}", {"status": rc})


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def strides3(t: torch.Tensor) -> ctypes.Array:
    """Element strides (b, h, s) of a 4-D ``[B, H, S, D]`` view with unit d-stride."""
    if t.dim() != 4 or (t.shape[-1] > 1 and t.stride(3) != 1):
        raise BackendError("operand must be a 4-D view with a contiguous last dimension",
                           {"shape": tuple(t.shape), "stride": tuple(t.stride())})
    return (ctypes.c_longlong * 3)(t.stride(0), t.stride(1), t.stride(2))


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise BackendError(f"unsupported dtype {dt}", {"dtype": str(dt)}) from None
