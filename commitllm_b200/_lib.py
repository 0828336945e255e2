"""ctypes binding of libvcommit.so (include/vcommit.h).

The library is built in-tree (``commitllm_b200/libvcommit.so``) by
``commitllm_b200.build_lib``.  There is no fallback: if it cannot be loaded,
every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_int32, c_int64, c_size_t, c_uint8, c_uint32, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvcommit.so")

VC_OK, VC_EINVAL, VC_ENOMEM, VC_ECUDA, VC_ETIMEDOUT, VC_ERANGE, VC_ENOTSUP = range(7)
VC_DTYPE_BF16, VC_DTYPE_F32, VC_DTYPE_F64 = 0, 1, 2
VC_ROPE_NONE, VC_ROPE_LLAMA3, VC_ROPE_LINEAR = 0, 1, 2

SYMBOLS = (
    "vc_abi_version", "vc_last_error", "vc_ctx_create", "vc_ctx_destroy", "vc_ctx_sync",
    "vc_kv_commit", "vc_trace_leaves", "vc_io_chain", "vc_prompt_hash", "vc_seed_commitment",
    "vc_build_trees", "vc_prove", "vc_tree_set_count", "vc_tree_nodes", "vc_tree_set_free",
    "vc_int_peak", "vc_wait_probe", "vc_kv_commit_noalloc", "vc_kv_open", "vc_io_extend", "vc_io_genesis",
    "vc_kv_transcript", "vc_kv_transcript_commit",
)


class VcError(RuntimeError):
    """A libvcommit call returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[vc status {status}] {msg}")
        self.status = status


class VcValueError(VcError, ValueError):
    """VC_EINVAL / VC_ERANGE: the argument errors the reference raises as ValueError."""


class KvDesc(ctypes.Structure):
    _fields_ = [
        ("n_layers", c_int32), ("layer_base", c_int32), ("n_kv_heads", c_int32), ("head_dim", c_int32),
        ("dtype", c_int32), ("n_seqs", c_int32),
        ("seq_lens", POINTER(c_int32)), ("seq_row_offset", POINTER(c_int64)),
        ("block_tables", c_void_p), ("block_size", c_int32), ("max_blocks_per_seq", c_int32),
        ("stride_page", c_int64), ("stride_row", c_int64), ("stride_head", c_int64),
        ("cache_elems", c_int64),
        ("k_layers", POINTER(c_void_p)), ("v_layers", POINTER(c_void_p)),
        ("pos_base", POINTER(c_int64)), ("tree_log2", c_int32),
    ]


class TraceDesc(ctypes.Structure):
    _fields_ = [
        ("n_tokens", c_int32), ("n_layers", c_int32), ("hidden", c_int32), ("n_fwd", c_int32),
        ("fwd_rows", POINTER(c_int32)), ("tok_fwd", POINTER(c_int32)), ("tok_row", POINTER(c_int32)),
        ("a_rows", POINTER(c_void_p)), ("scale_a", POINTER(c_void_p)), ("scale_stride", c_int64),
        ("x_attn_rows", POINTER(c_void_p)), ("scale_x_attn", POINTER(c_void_p)), ("scale_x_stride", c_int64),
        ("final_residual", c_void_p), ("fr_dim", c_int32), ("fr_rows", c_int32), ("fr_stride", c_int64),
        ("tok_fr_row", POINTER(c_int32)),
        ("lp_hidden", c_void_p), ("lp_dim", c_int32), ("lp_rows", c_int32), ("lp_stride", c_int64),
        ("tok_lp_row", POINTER(c_int32)),
        ("logits", c_void_p), ("vocab", c_int32), ("logits_rows", c_int32), ("logits_stride", c_int64),
        ("tok_logits_row", POINTER(c_int32)),
    ]


class KvtDesc(ctypes.Structure):
    _fields_ = [
        ("n_tokens", c_int32), ("n_layers", c_int32), ("hidden", c_int32), ("n_kv_heads", c_int32),
        ("head_dim", c_int32), ("use_rope", c_int32),
        ("x_layers", POINTER(c_void_p)), ("x_row_stride", c_int64),
        ("wk_layers", POINTER(c_void_p)), ("wv_layers", POINTER(c_void_p)),
        ("scale_x", c_void_p), ("sx_tstride", c_int64), ("sx_lstride", c_int64),
        ("sw_k", POINTER(ctypes.c_float)), ("sw_v", POINTER(ctypes.c_float)),
        ("ch_k", POINTER(c_void_p)), ("ch_v", POINTER(c_void_p)),
        ("bias_k", POINTER(c_void_p)), ("bias_v", POINTER(c_void_p)),
        ("rope_theta", c_double), ("rope_scaling", c_int32), ("rope_original_max_position_embeddings", c_int32),
        ("rope_factor", c_double), ("rope_low_freq_factor", c_double), ("rope_high_freq_factor", c_double),
    ]


_lib = None
_load_error = None


def _declare(lib):
    P = c_void_p
    lib.vc_abi_version.restype = c_int32
    lib.vc_abi_version.argtypes = []
    lib.vc_last_error.restype = c_size_t
    lib.vc_last_error.argtypes = [ctypes.c_char_p, c_size_t]
    for name, args in {
        "vc_ctx_create": [c_int32, P, POINTER(P)],
        "vc_ctx_destroy": [P],
        "vc_ctx_sync": [P, c_int32],
        "vc_kv_commit": [P, POINTER(KvDesc), P, POINTER(P)],
        "vc_trace_leaves": [P, POINTER(TraceDesc), P],
        "vc_io_chain": [P, c_int32, POINTER(c_int64), P, P, P, P],
        "vc_io_extend": [P, c_int32, POINTER(c_int64), P, P, P, P],
        "vc_io_genesis": [P, c_int32, P, P],
        "vc_prompt_hash": [P, c_int32, P, POINTER(c_int64), P],
        "vc_seed_commitment": [P, c_int32, P, P],
        "vc_build_trees": [P, c_int32, POINTER(c_int64), P, P, POINTER(P)],
        "vc_prove": [P, P, c_int32, POINTER(c_int32), POINTER(c_uint32), P, c_int32, POINTER(c_int32)],
        "vc_tree_nodes": [P, c_int32, POINTER(P), POINTER(c_int64), POINTER(c_int64)],
        "vc_tree_set_free": [P],
        "vc_int_peak": [P, c_int32, c_int64, POINTER(c_double)],
        "vc_wait_probe": [P, c_int64],
        "vc_kv_commit_noalloc": [POINTER(KvDesc), P, P, P],
        "vc_kv_open": [P, POINTER(KvDesc), P, c_int32, c_int32, POINTER(c_int32), c_int32, P, P, c_int32,
                       POINTER(c_int32)],
        "vc_kv_transcript": [P, POINTER(KvtDesc), P, P],
        "vc_kv_transcript_commit": [P, POINTER(KvtDesc), c_int32, P, POINTER(P)],
    }.items():
        fn = getattr(lib, name)
        fn.restype = c_int32
        fn.argtypes = args
    lib.vc_tree_set_count.restype = c_int32
    lib.vc_tree_set_count.argtypes = [P]


def lib():
    """The loaded library; raises if it is missing (no CPU fallback exists)."""
    global _lib, _load_error
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m commitllm_b200.build_lib`")
        try:
            l = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - depends on the machine
            _load_error = e
            raise RuntimeError(f"cannot load {LIB_PATH}: {e}") from e
        _declare(l)
        _lib = l
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().vc_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != VC_OK:
        msg = last_error()
        if status in (VC_EINVAL, VC_ERANGE):
            raise VcValueError(status, msg)
        raise VcError(status, msg)
