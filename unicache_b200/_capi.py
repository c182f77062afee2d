"""ctypes binding of ``libunicache_b200.so`` (declared in include/unicache_b200.h).

The library is the only compute path of this package: there is no CPU or
PyTorch fallback.  If the shared object is missing or fails to load, every call
raises ``RuntimeError`` (build it with ``python -m unicache_b200.build``).

Error convention (mirrors the reference: ``ValueError`` for argument errors,
``RuntimeError`` for an unavailable backend or a device failure, e.g.
unicache/storage/kivi_cuda.py:104-110 and :136-138):
UCB_ERR_INVALID / UCB_ERR_UNSUPPORTED -> ValueError, UCB_ERR_CUDA /
UCB_ERR_DEVICE -> RuntimeError.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libunicache_b200.so")

UCB_OK = 0
UCB_ERR_INVALID = -1
UCB_ERR_UNSUPPORTED = -2
UCB_ERR_CUDA = -3
UCB_ERR_DEVICE = -4

UCB_BF16 = 0
UCB_F16 = 1
UCB_F32 = 2

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int64 = ctypes.c_int64
c_float = ctypes.c_float


class UcbSpan(ctypes.Structure):
    _fields_ = [
        ("key_code", c_void_p),
        ("key_scale", c_void_p),
        ("key_minimum", c_void_p),
        ("value_code", c_void_p),
        ("value_scale", c_void_p),
        ("value_minimum", c_void_p),
        ("key_stride", c_int64),
        ("value_stride", c_int64),
        ("kind", ctypes.c_int32),
        ("tokens", ctypes.c_int32),
        ("pair", ctypes.c_int32),
        ("unit_begin", ctypes.c_int32),
    ]


class UcbPackSide(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("stride_t", c_int64), ("stride_h", c_int64), ("codes", c_void_p),
                ("scale", c_void_p), ("minimum", c_void_p)]


class UcbPackJob(ctypes.Structure):
    _fields_ = [("k", UcbPackSide), ("v", UcbPackSide), ("tokens", ctypes.c_int32), ("key_blocks", ctypes.c_int32),
                ("blocks", ctypes.c_int32), ("pad", ctypes.c_int32)]


class UcbDecodeCta(ctypes.Structure):
    _fields_ = [
        ("unit_begin", ctypes.c_int32),
        ("unit_end", ctypes.c_int32),
        ("span_begin", ctypes.c_int32),
        ("pair_begin", ctypes.c_int32),
        ("num_pairs", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 3),
    ]


class UcbDecodePair(ctypes.Structure):
    _fields_ = [
        ("seq", ctypes.c_int32),
        ("kv_head", ctypes.c_int32),
        ("partial_begin", ctypes.c_int32),
        ("partial_count", ctypes.c_int32),
        ("cta_first", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 3),
    ]


# name -> (restype, argtypes); the exact set declared in include/unicache_b200.h.
SIGNATURES = {
    "ucb_last_error": (ctypes.c_char_p, []),
    "ucb_version": (c_int, []),
    "ucb_device_status": (c_int, [ctypes.POINTER(ctypes.c_uint), c_void_p]),
    "ucb_kivi_pack_key": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "ucb_kivi_pack_value": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                    c_void_p, c_void_p, c_void_p, c_void_p]),
    "ucb_kivi_pack_kv": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                 c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p]),
    "ucb_kivi_pack_job_bytes": (c_int64, []),
    "ucb_kivi_pack_kv_batched": (c_int, [c_void_p, c_int, c_int, c_int64, c_int, c_int, c_int, c_void_p]),
    "ucb_kivi_dequant_key": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_int,
                                     c_int64, c_int64, c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "ucb_kivi_dequant_value": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int,
                                       c_int, c_int64, c_int64, c_void_p, c_int, c_int64, c_int64, c_void_p]),
    "ucb_fake_quant": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_int, c_void_p]),
    "ucb_decode_partial_bytes": (c_int64, [c_int]),
    "ucb_decode_attention": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                     c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                     c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "ucb_decode_attention_noalloc": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_int, c_void_p,
                                             c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int,
                                             c_int, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "ucb_decode_config": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "ucb_decode_set_trace": (c_int, [c_void_p]),
    "ucb_prefill_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p,
                                      c_void_p, c_void_p]),
    "ucb_prefill_attention_batched": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int,
                                              c_float, c_void_p, c_void_p, c_void_p]),
    "ucb_prefill_attention_items": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int,
                                            c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ucb_prefill_partial_bytes": (ctypes.c_int64, []),
    "ucb_long_query_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                                         c_int, c_int, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ucb_prefill_set_trace": (c_int, [c_void_p]),
    "ucb_long_query_stage": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                     c_void_p, c_int64, c_void_p]),
    "ucb_long_query_attention_staged": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                                c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                                c_float, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                                c_void_p, c_void_p]),
    "ucb_rms_norm": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p]),
    "ucb_qkv_rope_append": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_int, c_void_p]),
    "ucb_silu_mul": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ucb_peer_buffer_bytes": (ctypes.c_int64, [c_int64]),
    "ucb_peer_buffer_alloc": (c_int, [c_int64, ctypes.POINTER(c_void_p), c_void_p]),
    "ucb_peer_buffer_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "ucb_peer_buffer_close": (c_int, [c_void_p]),
    "ucb_peer_buffer_free": (c_int, [c_void_p]),
    "ucb_split_merge_peer": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p,
                                     c_void_p]),
    "ucb_lse_merge": (c_int, [c_int, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_int, c_int64, c_int64,
                              c_int64, c_void_p, c_void_p, c_void_p]),
    "ucb_h2o_select": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "ucb_gather_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p, c_int, c_int64, c_void_p,
                                c_void_p]),
    "ucb_h2o_accumulate_probs": (c_int, [c_void_p, c_int, c_int, c_int64, c_int64, c_int, c_void_p, c_int,
                                         c_void_p]),
    "ucb_h2o_scores_workspace_floats": (c_int64, [c_int64, c_int, c_int64]),
    "ucb_h2o_scores_from_lse": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_int64, c_int64, c_int,
                                        c_int, c_void_p, c_float, c_void_p, c_int, c_void_p]),
    "ucb_kivi_attention_logits": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                          c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                          c_float, c_void_p, c_void_p]),
    "ucb_kivi_attention_apply": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                         c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int, c_int,
                                         c_void_p, c_void_p]),
    "ucb_h2o_scores": (c_int, [c_void_p, c_int, c_int64, c_int, c_void_p, c_int64, c_int64, c_int64, c_int, c_int,
                               c_void_p, c_void_p, c_float, c_void_p, c_int, c_void_p]),
    "ucb_compact_rows": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                 ctypes.POINTER(c_int64), c_void_p]),
    "ucb_selftest_mma_subnormal": (c_int, [ctypes.POINTER(c_float), c_void_p]),
    "ucb_host_device_pointer": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "ucb_copy_ranges": (c_int, [c_int, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), ctypes.POINTER(c_int64),
                                c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_load_error: str | None = None


def load() -> ctypes.CDLL:
    """Load the library once; raise RuntimeError if it is missing."""

    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            _load_error = f"{LIB_PATH} is missing; build it with `python -m unicache_b200.build`"
            raise RuntimeError(_load_error)
        lib = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc == UCB_OK:
        return
    message = load().ucb_last_error().decode(errors="replace") or what
    if rc in (UCB_ERR_INVALID, UCB_ERR_UNSUPPORTED):
        raise ValueError(message)
    raise RuntimeError(message)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def struct_array_bytes(structs) -> bytes:
    if not structs:
        return b""
    kind = type(structs[0])
    arr = (kind * len(structs))(*structs)
    return ctypes.string_at(ctypes.addressof(arr), ctypes.sizeof(arr))
