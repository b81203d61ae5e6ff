"""ctypes binding of the C-ABI library ``libsparkb200.so`` (include/spark_b200.h).

The library is built in-tree by ``__graft_entry__.build()`` (or ``make -C
spark-mlx-llm_b200/csrc``). There is no fallback: if the library is missing
or fails to load, every operator raises ``RuntimeError``.
"""

import ctypes
import os
import threading

__all__ = ["lib", "check", "SBError", "LIB_PATH", "DTYPE_CODES"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libsparkb200.so")

SB_OK, SB_EINVAL, SB_EUNSUPPORTED, SB_ECUDA, SB_ETIMEOUT = 0, 1, 2, 3, 4
DTYPE_CODES = {"bfloat16": 0, "float16": 1, "float32": 2}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_size = ctypes.c_size_t
_float = ctypes.c_float


class SBError(RuntimeError):
    """A CUDA-side failure reported by the library (status SB_ECUDA/SB_ETIMEOUT)."""


class sb_linear_ex_desc(ctypes.Structure):
    """Mirror of ``sb_linear_ex_desc`` in include/spark_b200_decoder.h."""

    _fields_ = [
        ("x", _c_void_p),
        ("x_dtype", _int),
        ("ldx", _i64),
        ("M", _i64),
        ("N", _i64),
        ("K", _i64),
        ("weight_format", _int),
        ("weight", _c_void_p),
        ("scales", _c_void_p),
        ("biases", _c_void_p),
        ("weight2", _c_void_p),
        ("scales2", _c_void_p),
        ("biases2", _c_void_p),
        ("group_size", _int),
        ("norm_weight", _c_void_p),
        ("norm_eps", _float),
        ("epilogue", _int),
        ("y", _c_void_p),
        ("ldy", _i64),
        ("residual", _c_void_p),
        ("ldr", _i64),
        ("positions", _c_void_p),
        ("num_heads", _int),
        ("num_kv_heads", _int),
        ("head_dim", _int),
        ("seq_len", _int),
        ("rope_base", _float),
        ("q_out", _c_void_p),
        ("k_out", _c_void_p),
        ("v_out", _c_void_p),
        ("argmax_keys", _c_void_p),
        ("argmax_offset", _int),
        ("workspace", _c_void_p),
        ("workspace_bytes", _size),
        ("weights_constant", _int),
        ("kv_k_cache", _c_void_p),
        ("kv_k_scale", _c_void_p),
        ("kv_v_cache", _c_void_p),
        ("kv_v_scale", _c_void_p),
        ("kv_capacity", _i64),
        ("ar_world", _int),
        ("ar_rank", _int),
        ("ar_channel", _int),
        ("ar_buffers", _c_void_p * 8),
        ("activation", _int),
        ("k_chunks", _int),
        ("plan_rows", _i64),
        ("plan_k_chunks", _int),
        ("y_fp32", _int),
        ("scales_ld", _i64),
    ]


class sb_step_layer(ctypes.Structure):
    """Mirror of ``sb_step_layer`` (include/spark_b200_step.h)."""

    _fields_ = [(name, ctypes.c_void_p) for name in
                ("qkv", "qkv_scale", "o", "o_scale", "gateup", "down", "in_norm", "post_norm", "k_cache", "k_scale",
                 "v_cache", "v_scale")]


class sb_step_desc(ctypes.Structure):
    """Mirror of ``sb_step_desc`` (include/spark_b200_step.h)."""

    _fields_ = [
        ("layers", ctypes.c_void_p), ("num_layers", ctypes.c_int), ("hidden", ctypes.c_int),
        ("num_heads", ctypes.c_int), ("num_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("inter", ctypes.c_int), ("inter_total", ctypes.c_int), ("vocab", ctypes.c_int),
        ("vocab_offset", ctypes.c_int), ("capacity", ctypes.c_int), ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("embed", ctypes.c_void_p), ("vocab_total", ctypes.c_int),
        ("head", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("tokens", ctypes.c_void_p),
        ("positions", ctypes.c_void_p), ("x", ctypes.c_void_p), ("q", ctypes.c_void_p), ("kv_new", ctypes.c_void_p),
        ("attn", ctypes.c_void_p), ("act", ctypes.c_void_p), ("argmax_key", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t), ("world", ctypes.c_int),
        ("rank", ctypes.c_int), ("trace", ctypes.c_void_p),
    ]



# name -> (restype, argtypes); every symbol declared in include/*.h.
SIGNATURES = {
    "sb_version": (_int, []),
    "sb_last_error_message": (ctypes.c_char_p, []),
    "sb_device_supported": (_int, [_int]),
    "sb_affine_linear": (
        _int,
        [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _int, _int,
         _c_void_p, _size, _c_void_p],
    ),
    "sb_affine_linear_workspace_size": (_size, [_i64, _i64, _i64, _int, _int]),
    "sb_w8a16_per_channel": (
        _int,
        [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _size, _c_void_p],
    ),
    "sb_w8a16_per_channel_workspace_size": (_size, [_i64, _i64, _i64]),
    "sb_quantize_per_token": (_int, [_c_void_p, _int, _c_void_p, _c_void_p, _i64, _i64, _c_void_p]),
    "sb_int8_matmul_int32": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p]),
    "sb_w8a8_linear": (
        _int,
        [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _int, _c_void_p, _i64, _i64, _i64, _c_void_p,
         _size, _c_void_p],
    ),
    "sb_w8a8_linear_workspace_size": (_size, [_i64, _i64, _i64]),
    "sb_qkv_rope": (
        _int,
        [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64,
         _i64, _i64, _int, _int, _int, _int, _float, _int, _int, _c_void_p, _size, _c_void_p],
    ),
    "sb_qkv_rope_workspace_size": (_size, [_i64, _i64, _i64, _int, _int, _int, _int, _int]),
    "sb_int8_sdpa_decode": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _i64, _i64,
         _int, _float, _c_void_p, _size, _c_void_p],
    ),
    "sb_int8_sdpa_workspace_size": (_size, [_i64, _int, _int, _i64, _int]),
    "sb_int8_sdpa_prefill": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _i64, _i64, _i64,
         _int, _float, _int, _int, _c_void_p],
    ),
    "sb_int8_sdpa_prefill_window": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _i64, _i64, _i64,
         _int, _float, _int, _int, _c_void_p],
    ),
    "sb_bf16_sdpa_multiquery": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _i64, _i64, _i64, _int, _float, _int, _int,
         _c_void_p, _i64, _int, _c_void_p],
    ),
    "sb_rope_kv_append": (
        _int,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int,
         _int, _int, _i64, _int, _float, _c_void_p],
    ),
    "sb_rope_kv_append_ring": (
        _int,
        [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int,
         _int, _int, _i64, _int, _float, _i64, _c_void_p],
    ),
    "sb_swiglu": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "sb_gated_activation": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _int, _c_void_p]),
    "sb_head_gate": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int, _int, _c_void_p]),
    "sb_int8_sdpa_decode_static": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _i64, _i64, _int,
         _float, _c_void_p],
    ),
    "sb_affine_sdpa": (
        _int,
        [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int,
         _int, _i64, _i64, _int, _int, _int, _int, _float, _int, _c_void_p, _size, _c_void_p],
    ),
    "sb_affine_sdpa_workspace_size": (_size, [_i64, _int, _i64, _i64, _int]),
    "sb_rms_norm": (_int, [_c_void_p, _c_void_p, _c_void_p, _int, _i64, _i64, _float, _c_void_p]),
    # decoder header
    "sb_linear_ex": (_int, [ctypes.POINTER(sb_linear_ex_desc), _c_void_p]),
    "sb_linear_ex_workspace_size": (_size, [ctypes.POINTER(sb_linear_ex_desc)]),
    "sb_embed_rows_affine": (_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _int,
                                    _int, _c_void_p]),
    "sb_linear_ex_plan": (_int, [ctypes.POINTER(sb_linear_ex_desc), ctypes.POINTER(ctypes.c_int)]),
    "sb_kv_append_int8": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _i64, _int, _i64,
         _c_void_p, _c_void_p],
    ),
    "sb_int8_sdpa_decode_dev": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _int, _int, _c_void_p, _int,
         _i64, _i64, _int, _float, _int, _int, _c_void_p, _size, _c_void_p],
    ),
    "sb_embed_rows": (_int, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p]),
    "sb_decode_advance": (_int, [_c_void_p, _c_void_p, _c_void_p, _int, _int, _c_void_p]),
    "sb_residual_add": (_int, [_c_void_p, _c_void_p, _i64, _c_void_p]),
    "sb_tp_exchange_bytes": (_size, [_int, _i64]),
    "sb_peer_buffer_alloc": (_int, [_size, ctypes.POINTER(_c_void_p), _c_void_p]),
    "sb_peer_buffer_open": (_int, [_c_void_p, ctypes.POINTER(_c_void_p)]),
    "sb_peer_buffer_close": (_int, [_c_void_p]),
    "sb_peer_buffer_free": (_int, [_c_void_p]),
    # persistent decode step header
    "sb_step_workspace_size": (_size, [ctypes.POINTER(sb_step_desc)]),
    "sb_step_tile_bytes": (_int, [ctypes.POINTER(sb_step_desc), ctypes.POINTER(_i64)]),
    "sb_step_run": (_int, [ctypes.POINTER(sb_step_desc), _c_void_p]),
    "sb_step_trace_slots": (_int, [_int]),
    "sb_step_status_offset": (_size, []),
}

_lock = threading.Lock()
_lib = None


def lib():
    """Load (once) and return the library; raise RuntimeError if unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"spark_b200 CUDA library not found at {LIB_PATH}; build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` or "
                    "`make -C spark-mlx-llm_b200/csrc` (there is no CPU fallback)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def check(status, what):
    """Map a status code to the reference's error classes."""
    if status == SB_OK:
        return
    message = lib().sb_last_error_message().decode(errors="replace")
    text = f"{what}: {message}" if message else what
    if status in (SB_EINVAL, SB_EUNSUPPORTED):
        raise ValueError(text)
    raise SBError(text)
