"""ctypes declarations of the C ABI in include/kyro_spec.h.

The shared library is kyro_b200/libkyro_spec.so, built in-tree by
``python -m kyro_b200.build``.  There is no fallback: if the library is
missing, importing the package's operators raises.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkyro_spec.so")

KYRO_OK = 0
KYRO_ERR_INVALID_ARG = 1
KYRO_ERR_CUDA = 2
KYRO_ERR_NCCL = 3
KYRO_ERR_TIMEOUT = 4
KYRO_ERR_OOB = 5
KYRO_ERR_OOM = 6
KYRO_ERR_UNSUPPORTED = 7
KYRO_ERR_WORKSPACE = 8

# size of the library's static scratch used by kyro_spec_accept_static
ACCEPT_STATIC_SCRATCH_BYTES = 8 << 20

DEV_BAD_TOKEN = 0x1
DEV_BAD_BLOCK = 0x2
DEV_BAD_LENGTH = 0x4
DEV_WAIT_TIMEOUT = 0x8
DEV_STACK_OVERFLOW = 0x10

ACCEPT_STOCHASTIC = 0
ACCEPT_GREEDY = 1
ACCEPT_GREEDY_REF = 2

# Every symbol include/kyro_spec.h declares.
EXPORTS = (
    "kyro_ctx_create", "kyro_ctx_destroy", "kyro_ctx_set_stream", "kyro_ctx_device_status",
    "kyro_last_error", "kyro_status_string", "kyro_version", "kyro_kernel_names",
    "kyro_spec_accept_workspace_size", "kyro_spec_accept", "kyro_spec_accept_static",
    "kyro_spec_accept_commit",
    "kyro_sample_workspace_size",
    "kyro_sample_tokens", "kyro_verify_attention_workspace_size", "kyro_verify_attention",
    "kyro_verify_attention_rope",
    "kyro_kv_reserve", "kyro_kv_reserve_cow", "kyro_kv_commit", "kyro_kv_commit_tree", "kyro_kv_write",
    "kyro_rope_kv_write", "kyro_philox_uniforms", "kyro_selftest_exp",
    "kyro_tp_unique_id", "kyro_ctx_tp_init", "kyro_ctx_tp_transport",
    "kyro_ctx_set_wait_timeout", "kyro_ctx_tp_inject_skip", "kyro_selftest_exchange_timeout",
    "kyro_selftest_watchdog",
    "kyro_spec_accept_tp_workspace_size",
    "kyro_spec_accept_tp", "kyro_spec_accept_tree_workspace_size", "kyro_spec_accept_tree",
)

TP_UNIQUE_ID_BYTES = 128

# callback types of kyro_selftest_watchdog
POLL_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)
ABORT_FN = C.CFUNCTYPE(None, C.c_void_p)


class AcceptParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_draft", C.c_int32), ("vocab", C.c_int32),
                ("mode", C.c_int32), ("temperature", C.c_float), ("step", C.c_uint32),
                ("seed", C.c_uint64), ("seq_offset", C.c_int64)]


class TreeParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_nodes", C.c_int32), ("vocab", C.c_int32),
                ("mode", C.c_int32), ("temperature", C.c_float), ("step", C.c_uint32),
                ("seed", C.c_uint64), ("seq_offset", C.c_int64)]


class SampleParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_pos", C.c_int32), ("vocab", C.c_int32),
                ("temperature", C.c_float), ("step", C.c_uint32), ("seq_stride", C.c_uint32),
                ("seed", C.c_uint64), ("seq_offset", C.c_int64)]


class AttnParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_query", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("block_size", C.c_int32),
                ("max_blocks_per_seq", C.c_int32), ("num_blocks", C.c_int32),
                ("scale", C.c_float), ("kv_split_blocks", C.c_int32)]


class KVParams(C.Structure):
    _fields_ = [("batch", C.c_int32), ("block_size", C.c_int32),
                ("max_blocks_per_seq", C.c_int32), ("num_blocks", C.c_int32)]


class KyroError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"kyro status {status}: {message}")
        self.status = status


_lib = None


def load():
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m kyro_b200.build` "
            "(the verify-step kernels have no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    vp, i32, u32, u64, sz = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64, C.c_size_t
    P = C.POINTER
    sig = {
        "kyro_ctx_create": (C.c_int, [C.c_int, vp, P(vp)]),
        "kyro_ctx_destroy": (C.c_int, [vp]),
        "kyro_ctx_set_stream": (C.c_int, [vp, vp]),
        "kyro_ctx_device_status": (C.c_int, [vp, P(u32), C.c_int]),
        "kyro_last_error": (sz, [C.c_char_p, sz]),
        "kyro_status_string": (C.c_char_p, [C.c_int]),
        "kyro_version": (C.c_int, []),
        "kyro_kernel_names": (C.c_char_p, []),
        "kyro_spec_accept_workspace_size": (sz, [P(AcceptParams)]),
        "kyro_spec_accept": (C.c_int, [vp, P(AcceptParams), vp, vp, vp, vp, vp, vp, vp, vp, sz]),
        "kyro_spec_accept_static": (C.c_int, [vp, P(AcceptParams), vp, vp, vp, vp, vp, vp, vp]),
        "kyro_spec_accept_commit": (C.c_int, [vp, P(AcceptParams), vp, vp, vp, vp, vp, vp, vp, vp,
                                              sz, P(KVParams), i32, i32, vp, vp, vp, vp, vp, vp]),
        "kyro_sample_workspace_size": (sz, [P(SampleParams)]),
        "kyro_sample_tokens": (C.c_int, [vp, P(SampleParams), vp, vp, vp, vp, sz]),
        "kyro_verify_attention_workspace_size": (sz, [P(AttnParams)]),
        "kyro_verify_attention": (C.c_int, [vp, P(AttnParams), vp, vp, vp, vp, vp, vp, vp, vp,
                                            sz]),
        "kyro_verify_attention_rope": (C.c_int, [vp, P(AttnParams), C.c_float, vp, vp, vp, vp, vp,
                                                 vp, vp, vp, vp, vp, vp, sz]),
        "kyro_kv_reserve": (C.c_int, [vp, P(KVParams), i32, vp, vp, vp, vp, vp, vp]),
        "kyro_kv_commit": (C.c_int, [vp, P(KVParams), i32, vp, vp, vp, vp, vp, vp]),
        "kyro_kv_reserve_cow": (C.c_int, [vp, P(KVParams), i32, i32, vp, vp, i32, i32, vp, vp, vp,
                                          vp, vp, vp, vp]),
        "kyro_kv_commit_tree": (C.c_int, [vp, P(KVParams), i32, vp, vp, i32, vp, vp, i32, i32, vp,
                                          vp, vp, vp, vp]),
        "kyro_kv_write": (C.c_int, [vp, P(KVParams), i32, i32, i32, vp, vp, vp, vp, vp, vp]),
        "kyro_rope_kv_write": (C.c_int, [vp, P(KVParams), i32, i32, i32, i32, C.c_float, vp, vp,
                                         vp, vp, vp, vp, vp, vp, vp]),
        "kyro_philox_uniforms": (C.c_int, [vp, u64, u32, u32, u32, u32, i32, vp]),
        "kyro_selftest_exp": (C.c_int, [vp, vp]),
        "kyro_tp_unique_id": (C.c_int, [vp]),
        "kyro_spec_accept_tree_workspace_size": (C.c_size_t, [vp]),
        "kyro_spec_accept_tree": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                            C.c_size_t]),
        "kyro_ctx_tp_init": (C.c_int, [vp, vp, C.c_int, C.c_int]),
        "kyro_ctx_tp_transport": (C.c_int, [vp]),
        "kyro_ctx_set_wait_timeout": (C.c_int, [vp, u32]),
        "kyro_ctx_tp_inject_skip": (C.c_int, [vp, i32]),
        "kyro_selftest_exchange_timeout": (C.c_int, [vp, vp, sz]),
        "kyro_selftest_watchdog": (C.c_int, [u32, POLL_FN, ABORT_FN, vp]),
        "kyro_spec_accept_tp_workspace_size": (C.c_size_t, [vp, C.c_int]),
        "kyro_spec_accept_tp": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, C.c_size_t]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    L = load()
    buf = C.create_string_buffer(1024)
    L.kyro_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != KYRO_OK:
        raise KyroError(status, last_error())
