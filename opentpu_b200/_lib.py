"""ctypes binding of libotq.so (the C ABI of include/otq.h).

The library is built in-tree (`python -m opentpu_b200.csrc.build` or `__graft_entry__.build()`).
There is no fallback: if the library is missing or the GPU is not a compute-capability 10.x
device, every GPU entry point raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_int, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libotq.so"

OK, ERR_ARG, ERR_ALIGN, ERR_FORMAT, ERR_CUDA, ERR_DEVICE = 0, -1, -2, -3, -4, -5
FMT = {"int8": 0, "int4": 1, "fp4": 2, "nvfp4": 3}     # MM's WF codes (opentpu/isa.py:26-27)
MM_UNIT, MM_ACC, MM_ASCALE, MM_RSC = 0x1, 0x2, 0x8, 0x80

class Proj(ctypes.Structure):
    """struct otq_proj of include/otq.h: one projection of otq_qmm_chain."""
    _fields_ = [("fmt", c_int), ("flags", c_int), ("rows", c_void_p), ("rs", c_int64),
                ("srows", c_void_p), ("srs", c_int64), ("k0", c_int), ("N", c_int64),
                ("K", c_int64), ("x", c_void_p), ("row_mode", c_int), ("y", c_void_p)]


class Peer(ctypes.Structure):
    """struct otq_peer of include/otq.h: the NVLink fan-out of otq_qmm_peer."""
    _fields_ = [("rank", c_int), ("world", c_int), ("wait", c_int), ("tags", c_int),
                ("delta", c_int64 * 8), ("seq", c_void_p), ("done", c_void_p),
                ("step_pos", c_int), ("step_last", c_int)]

TAGS_COUNTED, TAGS_STEPPED = 0, 1


class StepProj(ctypes.Structure):
    """struct otq_step_proj of include/otq.h: one projection of otq_decode_step."""
    _fields_ = [("rows", c_void_p), ("rs", c_int64), ("srows", c_void_p), ("srs", c_int64),
                ("N", c_int64), ("K", c_int64), ("src", c_int), ("fmt", c_int),
                ("input", c_int), ("res", c_int), ("gamma", c_void_p), ("q_gain", c_void_p),
                ("k_gain", c_void_p), ("kcache", c_void_p), ("vcache", c_void_p),
                ("n_q", c_int), ("n_kv", c_int), ("head_dim", c_int), ("epilogue", c_int),
                ("replicated", c_int)]


STEP_RSC, STEP_G32, STEP_ATTN = 0, 1, 2
IN_DEFAULT, IN_NORM, IN_SWIGLU, IN_ATTN = 0, 1, 2, 3
EPI_NONE, EPI_SWIGLU = 0, 1


class Step(ctypes.Structure):
    """struct otq_step of include/otq.h: one decode step as one launch."""
    _fields_ = [("projs", c_void_p), ("count", c_int), ("rank", c_int), ("world", c_int),
                ("delta", c_int64 * 8), ("x0", c_void_p), ("out", c_void_p),
                ("counters", c_void_p), ("token", c_void_p), ("eps", ctypes.c_float),
                ("rope_cos", c_void_p), ("rope_sin", c_void_p), ("max_pos", c_int),
                ("pos", c_void_p), ("embed", c_void_p), ("token_in", c_void_p),
                ("vocab", c_int64)]


class GemmProj(ctypes.Structure):
    """struct otq_gemm_proj of include/otq.h: one projection of otq_gemm_w8a16_group."""
    _fields_ = [("flags", c_int), ("rows", c_void_p), ("rs", c_int64), ("srows", c_void_p),
                ("srs", c_int64), ("N", c_int64), ("K", c_int64), ("x", c_void_p),
                ("ldx", c_int64), ("M", c_int64), ("y", c_void_p), ("ldy", c_int64)]


class Gemm8Proj(ctypes.Structure):
    """struct otq_gemm8_proj of include/otq.h: one projection of otq_gemm_w8a8_group."""
    _fields_ = [("flags", c_int), ("rows", c_void_p), ("rs", c_int64), ("srows", c_void_p),
                ("srs", c_int64), ("N", c_int64), ("K", c_int64), ("planes", c_void_p),
                ("M", c_int64), ("y", c_void_p), ("ldy", c_int64)]


# name -> (restype, argtypes); every pointer is passed as an integer address
_P, _I, _L = c_void_p, c_int, c_int64
SIGNATURES = {
    "otq_version": (c_char_p, []),
    "otq_status_string": (c_char_p, [_I]),
    "otq_last_cuda_error": (c_char_p, []),
    "otq_device_check": (_I, []),
    "otq_quantize_rows": (_I, [_P, _L, _L, _L, _I, _I, _P, _L, _P, _P, _L, _P]),
    "otq_pack_int8": (_I, [_P, _L, _L, _L, _I, _P, _L, _P, _L, _P]),
    "otq_quantize_mxu": (_I, [_I, _P, _L, _L, _L, _P, _L, _P, _L, _P]),
    "otq_mm": (_I, [_I, _I, _P, _L, _P, _L, _I, _L, _L, _P, _L, _P, _P, _L, _L, _P, _P, _L, _P]),
    "otq_qmm": (_I, [_I, _I, _P, _L, _P, _L, _I, _L, _L, _P, _L, _I, _L, _P, _P, _L, _P]),
    "otq_qmm_ex": (_I, [_I, _I, _P, _L, _P, _L, _I, _L, _L, _P, _L, _I, _L, _P, _P, _L, _I, _I,
                        _P]),
    "otq_qmm_chain": (_I, [_P, _I, _P]),
    "otq_qmm_peer": (_I, [_I, _I, _P, _L, _P, _L, _I, _L, _L, _P, _L, _I, _P, _P, _I, _P]),
    "otq_gemm_w8a16": (_I, [_I, _P, _L, _P, _L, _L, _L, _P, _L, _L, _P, _L, _P]),
    "otq_gemm_w8a16_group": (_I, [_P, _I, _P]),
    "otq_qact_planes_bytes": (_L, [_L, _L]),
    "otq_qact_planes": (_I, [_P, _L, _L, _L, _I, _P, _L, _P]),
    "otq_gemm_w8a8_group": (_I, [_P, _I, _P]),
    "otq_qmm_tc": (_I, [_I, _P, _L, _P, _L, _L, _L, _P, _L, _I, _L, _P, _L, _P, _L, _P]),
    "otq_status_word": (_I, [_P, _I]),
    "otq_set_wait_limit": (_I, [ctypes.c_uint32]),
    "otq_step_layout": (_I, [_P, _I, _I, _P, _P]),
    "otq_step_table_bytes": (_I, [_P]),
    "otq_step_prepare": (_I, [_P, _P]),
    "otq_decode_step": (_I, [_P, _P, _P]),
    "otq_argmax": (_I, [_P, _L, _L, _P, _P]),
    "otq_argmax_noalloc": (_I, [_P, _L, _L, _P, _P]),
    "otq_pack_g32": (_I, [_P, _L, _L, _L, _P, _P, _P]),
    "otq_linear_g32": (_I, [_P, _P, _L, _L, _P, _L, _L, _I, _P, _L, _P]),
}

_lib = None


def load():
    """The loaded library (ctypes.CDLL), loading it on first use; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m opentpu_b200.csrc.build` "
            "(nvcc, sm_100a). There is no CPU implementation of this library.")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    """Raise for a non-zero status: ValueError for argument errors (the reference raises
    ValueError for bad shapes and formats), RuntimeError for CUDA and device errors."""
    if status == OK:
        return
    lib = load()
    msg = f"{what}: {lib.otq_status_string(status).decode()}"
    if status == ERR_CUDA:
        msg += f" ({lib.otq_last_cuda_error().decode()})"
    if status in (ERR_ARG, ERR_ALIGN, ERR_FORMAT):
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def status_word(reset: bool = True) -> int:
    """The device status word (synchronous): bit 0 = a kernel's bounded wait ran out."""
    v = ctypes.c_int(0)
    call("otq_status_word", ctypes.byref(v), int(reset))
    return v.value
