"""ctypes binding of the C ABI declared in ``include/memt_gdn2.h``.

The shared library is built in-tree by ``memt_b200.build``. There is no fallback:
importing an operator without the library raises immediately.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libmemt_gdn2.so")

MEMT_OK = 0
MEMT_ERR_INVALID_ARGUMENT = -1
MEMT_ERR_UNSUPPORTED = -2
MEMT_ERR_MISALIGNED = -3
MEMT_ERR_WORKSPACE = -4
MEMT_ERR_CUDA = -5

MEMT_F32 = 0
MEMT_BF16 = 1

GATE_NONE = 0
GATE_PER_HEAD = 1
GATE_PER_CHANNEL = 2


class _SizedArgs(ctypes.Structure):
    """An argument struct whose leading ``struct_size`` is set to its own size (the library
    rejects any other value with MEMT_ERR_INVALID_ARGUMENT)."""

    def __init__(self, **fields):
        fields.setdefault("struct_size", ctypes.sizeof(type(self)))
        super().__init__(**fields)


class UpdateArgs(_SizedArgs):
    _fields_ = [
        ("struct_size", c_uint32),
        ("num_samples", c_int32), ("num_heads", c_int32), ("key_dim", c_int32), ("value_dim", c_int32),
        ("total_tokens", c_int64), ("chunk_tokens", c_int32), ("dtype", c_int32),
        ("cu_seqlens", c_void_p), ("k", c_void_p), ("v", c_void_p), ("g", c_void_p), ("g_layout", c_int32),
        ("beta", c_void_p), ("beta_layout", c_int32), ("erase", c_void_p), ("erase_layout", c_int32),
        ("write", c_void_p), ("write_layout", c_int32), ("initial_state", c_void_p), ("final_state", c_void_p),
        ("initial_slots", c_void_p), ("num_initial_slots", c_int32), ("final_slots", c_void_p),
        ("num_final_slots", c_int32), ("k_stride", c_int64), ("v_stride", c_int64), ("write_stride", c_int64),
    ]


class ReadArgs(_SizedArgs):
    _fields_ = [
        ("struct_size", c_uint32),
        ("num_blocks", c_int32), ("num_heads", c_int32), ("key_dim", c_int32), ("value_dim", c_int32),
        ("total_tokens", c_int64), ("max_block_tokens", c_int32), ("cu_seqlens", c_void_p),
        ("q", c_void_p), ("q_dtype", c_int32), ("states", c_void_p), ("scale", c_float),
        ("out", c_void_p), ("out_dtype", c_int32), ("state_slots", c_void_p), ("num_slots", c_int32),
    ]


class ReadoutArgs(_SizedArgs):
    _fields_ = [
        ("struct_size", c_uint32),
        ("num_blocks", c_int32), ("num_heads", c_int32), ("head_dim", c_int32), ("total_tokens", c_int64),
        ("max_block_tokens", c_int32), ("cu_seqlens", c_void_p), ("q", c_void_p), ("normalize_q", c_int32),
        ("q_eps", c_float), ("states", c_void_p), ("scale", c_float), ("gate", c_void_p),
        ("norm_weight", c_void_p), ("norm_eps", c_float), ("softcap", c_float), ("residual", c_void_p),
        ("out", c_void_p), ("row_stride", c_int64), ("head_offset", c_int32), ("state_slots", c_void_p),
        ("num_slots", c_int32),
    ]


class PrologueArgs(_SizedArgs):
    _fields_ = [
        ("struct_size", c_uint32),
        ("num_heads", c_int32), ("head_dim", c_int32), ("total_tokens", c_int64),
        ("q", c_void_p), ("q_stride", c_int64), ("k", c_void_p), ("k_stride", c_int64),
        ("erase_latent", c_void_p), ("erase_stride", c_int64), ("write_latent", c_void_p),
        ("write_stride", c_int64), ("decay_latent", c_void_p), ("decay_stride", c_int64),
        ("decay_bias", c_void_p), ("decay_scale_log", c_void_p), ("eps", c_float), ("norm_kind", c_int32),
        ("q_out", c_void_p),
        ("k_out", c_void_p), ("write_out", c_void_p), ("log_decay_out", c_void_p),
    ]


class LatentNormArgs(_SizedArgs):
    _fields_ = [
        ("struct_size", c_uint32),
        ("groups", c_int32), ("rank", c_int32), ("total_tokens", c_int64), ("x", c_void_p), ("x_stride", c_int64),
        ("weight", c_void_p), ("eps", c_void_p), ("eps_scalar", c_float), ("out", c_void_p),
    ]


# name -> (restype, argtypes): every symbol include/memt_gdn2.h declares
SIGNATURES = {
    "memt_version": (c_int, []),
    "memt_status_string": (c_char_p, [c_int]),
    "memt_last_cuda_error": (c_int, []),
    "memt_gdn2_count_chunks": (c_int64, [POINTER(c_int32), c_int32, c_int32]),
    "memt_gdn2_update_workspace_size": (c_size_t, [c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32]),
    "memt_gdn2_update": (c_int, [POINTER(UpdateArgs), c_void_p, c_size_t, c_void_p]),
    "memt_gdn2_workspace_status": (c_int, [c_void_p, c_void_p, POINTER(c_int32)]),
    "memt_gdn2_read": (c_int, [POINTER(ReadArgs), c_void_p]),
    "memt_read_status": (c_int, [c_void_p, POINTER(c_int32)]),
    "memt_gdn2_update_read": (c_int, [POINTER(UpdateArgs), c_void_p, c_size_t, POINTER(ReadArgs), c_void_p]),
    "memt_memory_readout": (c_int, [POINTER(ReadoutArgs), c_void_p]),
    "memt_qwen_prologue": (c_int, [POINTER(PrologueArgs), c_void_p]),
    "memt_latent_rms_norm": (c_int, [POINTER(LatentNormArgs), c_void_p]),
    "memt_gdn2_update_noalloc": (c_int, [POINTER(UpdateArgs), c_void_p]),
    "memt_gdn2_noalloc_status": (c_int, [c_void_p, POINTER(c_int32)]),
    "memt_profiler_enable": (c_int, [c_int]),
    "memt_profiler_reset": (c_int, []),
    "memt_profiler_read": (c_int, [POINTER(ctypes.c_double), POINTER(c_int64), c_int]),
}

PROF_FAMILIES = ["plan", "intra", "scan", "read_gemv", "read_tile", "recurrent", "prologue"]


def profiler_enable(on: bool) -> None:
    load().memt_profiler_enable(1 if on else 0)


def profiler_reset() -> None:
    load().memt_profiler_reset()


def profiler_read() -> dict:
    """{family: (total device ms, launches)}; synchronises the recorded events."""
    n = len(PROF_FAMILIES)
    ms = (ctypes.c_double * n)()
    cnt = (c_int64 * n)()
    check(load().memt_profiler_read(ms, cnt, n), "memt_profiler_read")
    return {name: (ms[i], cnt[i]) for i, name in enumerate(PROF_FAMILIES)}

_lib = None


def load(path: str | Path | None = None):
    """Load the shared library (once) and attach the ctypes signatures."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"memt_b200: CUDA library {p} is missing; build it with `python -m memt_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class MemtError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    """Map a C-ABI status to the reference's exception types (ValueError before launch)."""
    if status == MEMT_OK:
        return
    lib = load()
    msg = f"{what}: {lib.memt_status_string(status).decode()}"
    if status == MEMT_ERR_CUDA:
        raise MemtError(f"{msg} (cudaError {lib.memt_last_cuda_error()})")
    raise ValueError(msg)
