"""ctypes binding of libasap.so (include/asap.h).  The product path has no fallback: if the library is
missing or a call fails, this module raises."""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_uint8, c_uint32, c_uint64, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libasap.so")

ASAP_OK, ASAP_EINVAL, ASAP_ECUDA, ASAP_ETIMEOUT, ASAP_EPOISONED = 0, -1, -2, -3, -4
ST_NAMES = {
    0: "ok",
    1: "backpressure timeout",
    2: "doorbell timeout",
    3: "bad doorbell",
    4: "reply timeout",
    5: "pipeline timeout",
    6: "bad job",
}
MAX_F = 16
MAX_LOCAL_EXPERTS = 256
MAX_JOB_ROWS = 8


class AsapError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


class Geometry_t(ctypes.Structure):
    _fields_ = [(n, c_int32) for n in ("num_a", "group", "slots", "n_max", "hidden", "topk", "num_f")]


class Offsets_t(ctypes.Structure):
    _fields_ = [(n, c_uint64) for n in ("ids_off", "w_off", "region_bytes", "recv_bytes", "host_bytes",
                                         "flags_bytes", "seg_bytes", "result_bytes")]


class Mxfp4Experts_t(ctypes.Structure):
    _fields_ = [("num_local", c_int32), ("expert_base", c_int32), ("hidden", c_int32), ("inter", c_int32),
                ("w13", c_uint64), ("w13_sf", c_uint64), ("w2", c_uint64), ("w2_sf", c_uint64)]


class FfnRow_t(ctypes.Structure):
    _fields_ = [(n, c_uint64) for n in ("x", "ids", "w", "reply_seg", "reply_done")]


class Fp8Experts_t(ctypes.Structure):
    _fields_ = [("num_local", c_int32), ("expert_base", c_int32), ("hidden", c_int32), ("inter", c_int32),
                ("w13", c_uint64), ("w13_scale", c_uint64), ("w2", c_uint64), ("w2_scale", c_uint64)]


# name -> (restype, argtypes); every int-returning call is checked
_SIGS = {
    "asap_last_error_string": (c_char_p, []),
    "asap_version": (c_char_p, []),
    "asap_geometry_offsets": (c_int32, [POINTER(Geometry_t), POINTER(Offsets_t)]),
    "asap_pack_doorbell": (c_int32, [c_uint32, c_uint32, c_uint32, c_uint32, POINTER(c_uint64)]),
    "asap_unpack_doorbell": (None, [c_uint64, POINTER(c_uint32), POINTER(c_uint32), POINTER(c_uint32),
                                    POINTER(c_uint32)]),
    "asap_init": (c_int32, [c_int32]),
    "asap_arena_alloc": (c_int32, [c_uint64, POINTER(c_uint64), POINTER(c_uint8)]),
    "asap_arena_free": (c_int32, [c_uint64]),
    "asap_arena_open": (c_int32, [POINTER(c_uint8), POINTER(c_uint64)]),
    "asap_arena_close": (c_int32, [c_uint64]),
    "asap_host_register": (c_int32, [c_uint64, c_uint64, POINTER(c_uint64)]),
    "asap_host_page_create": (c_int32, [c_char_p, c_uint64, POINTER(c_uint64), POINTER(c_uint64)]),
    "asap_host_page_open": (c_int32, [c_char_p, c_uint64, POINTER(c_uint64), POINTER(c_uint64)]),
    "asap_release": (c_int32, [c_uint64]),
    "asap_host_unregister": (c_int32, [c_uint64]),
    "asap_memset32": (c_int32, [c_uint64, c_uint32, c_uint64, c_void_p]),
    "asap_write32": (c_int32, [c_uint64, c_uint32, c_void_p]),
    "asap_route_ws_bytes": (c_uint64, [POINTER(Geometry_t)]),
    "asap_dispatch": (c_int32, [POINTER(Geometry_t), c_int32, c_int32, c_uint32, c_int32, POINTER(c_int32),
                                c_uint64, c_uint64, c_int32, c_uint64, c_int32, c_int32, POINTER(c_int32),
                                POINTER(c_uint64), POINTER(c_uint64), c_uint64, c_uint64, c_int32, c_uint64,
                                c_uint64, c_void_p]),
    "asap_dispatch_noalloc": (c_int32, [POINTER(Geometry_t), c_int32, c_int32, c_uint32, c_int32, POINTER(c_int32),
                                        c_uint64, c_uint64, c_int32, c_uint64, c_int32, c_int32, POINTER(c_int32),
                                        POINTER(c_uint64), POINTER(c_uint64), c_uint64, c_int32, c_uint64, c_uint64,
                                        c_void_p, POINTER(c_uint64)]),
    "asap_combine": (c_int32, [POINTER(Geometry_t), c_int32, c_uint32, c_int32, c_uint64, c_uint64, c_uint64,
                               c_uint64, c_uint64, c_uint64, c_void_p]),
    "asap_wait_replies": (c_int32, [POINTER(Geometry_t), c_int32, c_uint32, c_uint64, c_uint64, c_uint64,
                                    c_void_p]),
    "asap_experts_register": (c_int32, [POINTER(Mxfp4Experts_t), POINTER(c_uint64)]),
    "asap_experts_register_fp8": (c_int32, [POINTER(Fp8Experts_t), POINTER(c_uint64)]),
    "asap_experts_release": (c_int32, [c_uint64]),
    "asap_ffn_ws_bytes": (c_uint64, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "asap_ffn_ws_register": (c_int32, [c_uint64, c_int32, c_int32, c_int32, c_int32, c_int32, POINTER(c_uint64)]),
    "asap_ffn_ws_release": (c_int32, [c_uint64]),
    "asap_ffn_wait": (c_int32, [c_uint64, c_uint64, c_uint32, c_int32, c_int32, c_uint64, c_uint64, c_void_p]),
    "asap_ffn_post": (c_int32, [c_uint64, c_uint32, c_int32, c_int32, c_int32, c_void_p]),
    "asap_ffn_wait_rows": (c_int32, [c_uint64, c_int32, POINTER(c_uint64), POINTER(c_uint32), POINTER(c_int32), c_int32,
                                     c_uint64, c_uint64, c_void_p]),
    "asap_ffn_wait_state": (c_int32, [c_uint64, c_int32, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_int32), c_int32,
                                      c_uint64, c_uint64, c_void_p]),
    "asap_ffn_wait_any": (c_int32, [c_uint64, c_int32, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_int32), c_int32,
                                    c_uint64, c_uint64, c_uint64, c_void_p]),
    "asap_ffn_wait_rest": (c_int32, [c_uint64, c_int32, POINTER(c_uint64), POINTER(c_uint64), POINTER(c_uint32),
                                     POINTER(c_int32), c_int32, c_uint64, c_uint64, c_void_p]),
    "asap_graph_begin": (c_int32, [c_void_p]),
    "asap_graph_end": (c_int32, [c_void_p, POINTER(c_uint64)]),
    "asap_graph_launch": (c_int32, [c_uint64, c_void_p]),
    "asap_graph_release": (c_int32, [c_uint64]),
    "asap_ffn_post_rows": (c_int32, [c_uint64, c_int32, POINTER(c_uint32), POINTER(c_int32), c_int32,
                                     POINTER(c_int32), c_void_p]),
    "asap_ffn_job_rows": (c_int32, [c_uint64, c_uint64, c_int32, POINTER(FfnRow_t), c_float, c_uint64, c_uint64,
                                    c_void_p]),
    "asap_ffn_job_rows_overlap": (c_int32, [c_uint64, c_uint64, c_int32, POINTER(FfnRow_t), c_float, c_uint64,
                                            c_uint64, c_void_p, c_void_p, c_int32, c_int32]),
    "asap_ffn_job": (c_int32, [c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_uint64, c_float,
                               c_uint64, c_uint64, c_void_p]),
    "asap_ffn_enable_timing": (c_int32, [c_uint64, c_int32]),
    "asap_ffn_last_timing": (c_int32, [c_uint64, POINTER(c_float), c_int32]),
    "asap_ffn_job_info": (c_int32, [c_uint64, POINTER(c_int32), POINTER(c_int32), POINTER(c_uint32),
                                    POINTER(c_int32), POINTER(c_int32), POINTER(c_uint64), POINTER(c_uint64),
                                    c_void_p]),
    "asap_dispatch_info": (c_int32, [c_uint64, c_int32, POINTER(c_int32), POINTER(c_uint64), POINTER(c_uint64),
                                     c_void_p]),
    "asap_ffn_debug_ptrs": (c_int32, [c_uint64] + [POINTER(c_uint64)] * 7),
}

_lib = None


def lib():
    """The loaded library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python sgl-afd-plugin_b200/build.py` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(name: str, rc: int) -> None:
    if rc != ASAP_OK:
        msg = lib().asap_last_error_string()
        raise AsapError(name, rc, msg.decode() if msg else "")


def call(name: str, *args) -> int:
    rc = getattr(lib(), name)(*args)
    check(name, rc)
    return rc


def geometry_struct(g) -> Geometry_t:
    return Geometry_t(g.num_a, g.group, g.slots, g.n_max, g.hidden, g.topk, g.num_f)


def decode_status(word: int) -> dict:
    code = word & 0xFF
    return {"code": code, "what": ST_NAMES.get(code, f"code {code}"), "f": (word >> 8) & 0xFF,
            "slot": (word >> 16) & 0xFF, "seq": word >> 32}
