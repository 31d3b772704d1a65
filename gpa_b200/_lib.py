"""ctypes binding of the C ABI declared in ``include/gpa_b200.h``.

The shared library ``gpa_b200/libgpa_b200.so`` is built in-tree for sm_100a
(``python -m gpa_b200.build``).  There is no fallback: if the library is
missing or was built for another ABI version, every call raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_void_p

MAX_LEVELS = 8
MAX_EDGES = 56
ABI_VERSION = 2
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgpa_b200.so")

STATUS = {0: "ok", 1: "bad argument", 2: "unsupported configuration", 3: "CUDA launch failure",
          4: "device timeout"}


class GpaDims(ctypes.Structure):
    _fields_ = [("batch", c_int32), ("length", c_int32), ("heads", c_int32),
                ("key_dim", c_int32), ("value_dim", c_int32), ("levels", c_int32),
                ("slots", c_int32 * MAX_LEVELS), ("chunk_size", c_int32),
                ("chunk_offset", c_int32), ("input_dtype", c_int32),
                ("positional_none", c_int32), ("read_scale", c_float),
                ("query_scale", c_float), ("beta_max", c_float), ("reader_mode", c_int32),
                ("positional_moments", c_int32), ("position", c_int32)]


_LEVEL_PARAMS = ("center", "route_weight", "query_weight", "route_up", "route_down",
                 "gate_weight", "gate_bias")
_SCALAR_PARAMS = ("residual_raw", "count_gain_raw", "route_mlp_gain", "output_logits",
                  "edge_logits", "relation_gain", "relation_decay_raw", "relation_beta_raw",
                  "moment_gain")


class GpaParams(ctypes.Structure):
    _fields_ = ([(n, c_void_p * MAX_LEVELS) for n in _LEVEL_PARAMS] +
                [(n, c_void_p) for n in _SCALAR_PARAMS])


class GpaParamGrads(ctypes.Structure):
    _fields_ = GpaParams._fields_


class GpaStateRef(ctypes.Structure):
    _fields_ = [("inner", c_void_p * MAX_LEVELS), ("outer", c_void_p * MAX_LEVELS),
                ("count", c_void_p * MAX_LEVELS), ("relation", c_void_p * MAX_EDGES),
                ("frozen_inner", c_void_p * MAX_LEVELS), ("frozen_outer", c_void_p * MAX_LEVELS),
                ("moment", c_void_p * MAX_LEVELS)]


EXPORTS = ("gpa_b200_saved_bytes", "gpa_b200_scratch_bytes", "gpa_b200_forward",
           "gpa_b200_backward", "gpa_b200_routes", "gpa_b200_last_error",
           "gpa_b200_abi_version", "gpa_b200_launch_count", "gpa_b200_profile_start",
           "gpa_b200_profile_stop", "gpa_b200_forward_noalloc", "gpa_b200_noalloc_capacity",
           "gpa_b200_step", "gpa_b200_umma_selftest", "gpa_b200_device_status")

_lib = None


def load():
    """Load the library once (raises if it is missing or incompatible)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run `python -m gpa_b200.build` "
                           "(the b200 backend has no CPU or library fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.gpa_b200_saved_bytes.argtypes = [POINTER(GpaDims)]
    lib.gpa_b200_saved_bytes.restype = c_size_t
    lib.gpa_b200_scratch_bytes.argtypes = [POINTER(GpaDims)]
    lib.gpa_b200_scratch_bytes.restype = c_size_t
    lib.gpa_b200_forward.argtypes = [POINTER(GpaDims), POINTER(GpaParams), c_void_p, c_void_p,
                                     c_void_p, POINTER(GpaStateRef), POINTER(GpaStateRef),
                                     c_void_p, c_void_p, c_size_t, c_void_p]
    lib.gpa_b200_forward.restype = c_int
    lib.gpa_b200_backward.argtypes = [POINTER(GpaDims), POINTER(GpaParams), POINTER(GpaStateRef),
                                      c_void_p, c_void_p, POINTER(GpaStateRef), c_void_p,
                                      c_void_p, c_void_p, POINTER(GpaStateRef),
                                      POINTER(GpaParamGrads), c_void_p, c_size_t, c_void_p]
    lib.gpa_b200_backward.restype = c_int
    lib.gpa_b200_forward_noalloc.argtypes = [POINTER(GpaDims), POINTER(GpaParams), c_void_p,
                                             c_void_p, c_void_p, POINTER(GpaStateRef),
                                             POINTER(GpaStateRef), c_void_p, c_void_p]
    lib.gpa_b200_forward_noalloc.restype = c_int
    lib.gpa_b200_step.argtypes = [POINTER(GpaDims), POINTER(GpaParams), c_void_p, c_void_p,
                                  c_void_p, POINTER(GpaStateRef), c_void_p, c_void_p, c_void_p]
    lib.gpa_b200_step.restype = c_int
    lib.gpa_b200_device_status.argtypes = [c_int]
    lib.gpa_b200_device_status.restype = c_int
    lib.gpa_b200_umma_selftest.argtypes = [c_int] * 7 + [c_void_p] * 6
    lib.gpa_b200_umma_selftest.restype = c_int
    lib.gpa_b200_noalloc_capacity.argtypes = []
    lib.gpa_b200_noalloc_capacity.restype = c_size_t
    lib.gpa_b200_routes.argtypes = [POINTER(GpaDims), c_void_p, POINTER(c_void_p), c_void_p]
    lib.gpa_b200_routes.restype = c_int
    lib.gpa_b200_last_error.argtypes = [c_char_p, c_size_t]
    lib.gpa_b200_last_error.restype = c_int
    lib.gpa_b200_abi_version.argtypes = []
    lib.gpa_b200_abi_version.restype = c_int
    lib.gpa_b200_launch_count.argtypes = []
    lib.gpa_b200_launch_count.restype = ctypes.c_longlong
    lib.gpa_b200_profile_start.argtypes = []
    lib.gpa_b200_profile_start.restype = c_int
    lib.gpa_b200_profile_stop.argtypes = [c_char_p, c_size_t]
    lib.gpa_b200_profile_stop.restype = c_int
    if lib.gpa_b200_abi_version() != ABI_VERSION:
        raise RuntimeError("libgpa_b200.so ABI version mismatch; rebuild it")
    _lib = lib
    return lib


def check(rc: int, what: str):
    """Raise ValueError (argument / configuration) or RuntimeError (launch) on failure."""
    if rc == 0:
        return
    buf = ctypes.create_string_buffer(1024)
    load().gpa_b200_last_error(buf, len(buf))
    msg = f"{what}: {STATUS.get(rc, rc)}: {buf.value.decode(errors='replace')}"
    if rc in (1, 2):
        raise ValueError(msg)
    raise RuntimeError(msg)


def launch_count() -> int:
    """Kernels launched by the library in this process."""
    return int(load().gpa_b200_launch_count())


def profile_start():
    check(load().gpa_b200_profile_start(), "gpa_b200_profile_start")


def profile_stop() -> dict:
    """{kernel: (launches, total_ms)} of the launches since profile_start()."""
    import json
    buf = ctypes.create_string_buffer(1 << 16)
    check(load().gpa_b200_profile_stop(buf, len(buf)), "gpa_b200_profile_stop")
    return {k: (int(v[0]), float(v[1])) for k, v in json.loads(buf.value.decode()).items()}


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def device_status(clear: bool = False) -> int:
    """0, or 4 (device timeout) when a bounded wait inside a tensor-core kernel gave up."""
    return int(load().gpa_b200_device_status(int(clear)))
