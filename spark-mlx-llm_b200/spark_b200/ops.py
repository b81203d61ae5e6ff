"""PyTorch custom operators (``torch.ops.spark_b200.*``) over the C-ABI library.

Each operator validates its inputs, allocates its outputs with ``torch.empty``
on the input's device, and enqueues the CUDA kernels on the current torch
stream through ``libsparkb200.so``. Inputs are never modified. There is no
CPU implementation: CPU tensors raise ``ValueError`` like the reference's
GPU-only primitives (``src/spark_w8a8.cpp:156-158``).
"""

import threading
from typing import Optional

import torch

from ._lib import DTYPE_CODES, check, lib

__all__ = [
    "affine_linear",
    "w8a16_per_channel",
    "quantize_per_token",
    "int8_matmul_int32",
    "w8a8_linear",
    "qkv_rope",
    "int8_sdpa_decode",
    "int8_sdpa_prefill",
    "bf16_sdpa_multiquery",
    "gated_activation",
    "head_gate",
    "rms_norm",
    "workspace",
]

_FLOAT_DTYPES = (torch.bfloat16, torch.float16, torch.float32)


def _code(dtype):
    return DTYPE_CODES[str(dtype).replace("torch.", "")]


def _stream(t):
    return ctypes_stream(torch.cuda.current_stream(t.device))


def ctypes_stream(stream):
    return stream.cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError("spark_b200 operators are GPU-only (no CPU fallback); got a CPU tensor")


class _Workspace:
    """Zero-initialised scratch per (device, stream); kernels leave it zeroed."""

    def __init__(self):
        self._buffers = {}
        self._lock = threading.Lock()

    def get(self, device, nbytes):
        if nbytes == 0:
            return None, 0
        stream = torch.cuda.current_stream(device)
        key = (device.index, stream.cuda_stream)
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                buf = torch.zeros(size, dtype=torch.uint8, device=device)
                self._buffers[key] = buf
        return buf.data_ptr(), buf.numel()


workspace = _Workspace()


# ----------------------------------------------------------------- affine linear
@torch.library.custom_op("spark_b200::affine_linear", mutates_args=())
def affine_linear(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                  group_size: int, bits: int) -> torch.Tensor:
    """``mx.quantized_matmul(x, w, scales, biases, transpose=True, group_size, bits,
    mode="affine")`` (spark_mlx_llm/ops/linear.py:180-191) on the GPU."""
    _require_cuda(x, weight, scales, biases)
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("affine linear requires bfloat16 or float16 activations")
    if weight.dtype not in (torch.int32, torch.uint32) or weight.ndim != 2:
        raise ValueError("weight must be uint32-packed [N, K*bits/32]")
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        raise ValueError("scales and biases must have the activation dtype")
    k = x.shape[-1]
    n = weight.shape[0]
    if weight.shape[1] * 32 != k * bits or scales.shape != (n, k // group_size) or biases.shape != scales.shape:
        raise ValueError("packed weight and quantization metadata shapes do not match x, group_size and bits")
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    weight, scales, biases = weight.contiguous(), scales.contiguous(), biases.contiguous()
    ws, ws_bytes = workspace.get(x.device, lib().sb_affine_linear_workspace_size(m, n, k, group_size, bits))
    check(
        lib().sb_affine_linear(x2.data_ptr(), _code(x.dtype), weight.data_ptr(), scales.data_ptr(),
                               biases.data_ptr(), y.data_ptr(), m, n, k, group_size, bits, ws, ws_bytes,
                               _stream(x)),
        "affine_linear",
    )
    return y.reshape(*x.shape[:-1], n)


@affine_linear.register_fake
def _(x, weight, scales, biases, group_size, bits):
    return x.new_empty((*x.shape[:-1], weight.shape[0]))


# ------------------------------------------------------------- W8A16 per channel
@torch.library.custom_op("spark_b200::w8a16_per_channel", mutates_args=())
def w8a16_per_channel(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """``w8a16_per_channel`` (extensions/spark-mlx-ext/src/spark_w8a16.cpp:80-110)."""
    _require_cuda(x, weight, scales)
    if x.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("w8a16_per_channel x must have dtype bfloat16 or float16.")
    if weight.dtype != torch.int8 or weight.ndim != 2:
        raise ValueError("w8a16_per_channel weight must have dtype int8.")
    n, k = weight.shape
    if scales.dtype != torch.float32 or tuple(scales.shape) not in ((n,), (n, 1)):
        raise ValueError("w8a16_per_channel scales must have dtype float32 and shape [N] or [N, 1].")
    if x.shape[-1] != k:
        raise ValueError("x[..., K] and weight[N, K] must have matching K")
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    weight, scales = weight.contiguous(), scales.reshape(-1).contiguous()
    ws, ws_bytes = workspace.get(x.device, lib().sb_w8a16_per_channel_workspace_size(m, n, k))
    check(
        lib().sb_w8a16_per_channel(x2.data_ptr(), _code(x.dtype), weight.data_ptr(), scales.data_ptr(),
                                   y.data_ptr(), m, n, k, ws, ws_bytes, _stream(x)),
        "w8a16_per_channel",
    )
    return y.reshape(*x.shape[:-1], n)


@w8a16_per_channel.register_fake
def _(x, weight, scales):
    return x.new_empty((*x.shape[:-1], weight.shape[0]))


# ------------------------------------------------------------------------- W8A8
@torch.library.custom_op("spark_b200::quantize_per_token", mutates_args=())
def quantize_per_token(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token INT8 quantization (src/kernels/w8a8_quantize.metal:6-43)."""
    _require_cuda(x)
    if x.dtype not in _FLOAT_DTYPES:
        raise ValueError("x must have dtype float16, bfloat16, or float32.")
    k = x.shape[-1]
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m,), dtype=torch.float32, device=x.device)
    check(lib().sb_quantize_per_token(x2.data_ptr(), _code(x.dtype), q.data_ptr(), s.data_ptr(), m, k, _stream(x)),
          "quantize_per_token")
    return q.reshape(x.shape), s.reshape(x.shape[:-1])


@quantize_per_token.register_fake
def _(x):
    return torch.empty_like(x, dtype=torch.int8), x.new_empty(x.shape[:-1], dtype=torch.float32)


@torch.library.custom_op("spark_b200::int8_matmul_int32", mutates_args=())
def int8_matmul_int32(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Exact ``x[M,K] @ weight[N,K]^T`` in int32 (src/spark_w8a8.cpp:218-228)."""
    _require_cuda(x, weight)
    if x.ndim != 2 or x.dtype != torch.int8:
        raise ValueError("int8_matmul_int32 requires x[M, K] with dtype int8.")
    if weight.ndim != 2 or weight.dtype != torch.int8 or weight.shape[1] != x.shape[1]:
        raise ValueError("Expected nonempty x[..., K] and weight[N, K] with matching K.")
    m, k = x.shape
    n = weight.shape[0]
    out = torch.empty((m, n), dtype=torch.int32, device=x.device)
    check(lib().sb_int8_matmul_int32(x.contiguous().data_ptr(), weight.contiguous().data_ptr(), out.data_ptr(),
                                     m, n, k, _stream(x)), "int8_matmul_int32")
    return out


@int8_matmul_int32.register_fake
def _(x, weight):
    return x.new_empty((x.shape[0], weight.shape[0]), dtype=torch.int32)


@torch.library.custom_op("spark_b200::w8a8_linear", mutates_args=())
def w8a8_linear(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor,
                bias: torch.Tensor | None = None) -> torch.Tensor:
    """``w8a8_linear`` (src/spark_w8a8.cpp:230-257): per-token INT8 activations,
    INT32 accumulation, ``float(acc) * sa * sw + bias`` cast to x's dtype."""
    _require_cuda(x, weight, scales, bias)
    if x.dtype not in _FLOAT_DTYPES:
        raise ValueError("x must have dtype float16, bfloat16, or float32.")
    if weight.ndim != 2 or weight.dtype != torch.int8:
        raise ValueError("weight must contain signed INT8 values.")
    n, k = weight.shape
    if x.ndim < 1 or x.shape[-1] != k or x.numel() == 0:
        raise ValueError("Expected nonempty x[..., K] and weight[N, K] with matching K.")
    if k % 32 or k > 131040:
        raise ValueError("K must be a multiple of 32 in [32, 131040].")
    if scales.dtype != torch.float32 or tuple(scales.shape) not in ((n,), (n, 1)):
        raise ValueError("scales must have shape [N] or [N, 1] and dtype float32.")
    if bias is not None and (tuple(bias.shape) != (n,) or bias.dtype not in _FLOAT_DTYPES):
        raise ValueError("bias must have shape [N] and a real floating dtype.")
    x2 = x.reshape(-1, k).contiguous()
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    ws, ws_bytes = workspace.get(x.device, lib().sb_w8a8_linear_workspace_size(m, n, k))
    b = None if bias is None else bias.contiguous()
    check(
        lib().sb_w8a8_linear(x2.data_ptr(), _code(x.dtype), weight.contiguous().data_ptr(),
                             scales.reshape(-1).contiguous().data_ptr(), _ptr(b),
                             _code(b.dtype) if b is not None else 0, y.data_ptr(), m, n, k, ws, ws_bytes,
                             _stream(x)),
        "w8a8_linear",
    )
    return y.reshape(*x.shape[:-1], n)


@w8a8_linear.register_fake
def _(x, weight, scales, bias=None):
    return x.new_empty((*x.shape[:-1], weight.shape[0]))


# --------------------------------------------------------------------- QKV+RoPE
@torch.library.custom_op("spark_b200::qkv_rope", mutates_args=())
def qkv_rope(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
             positions: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int, rope_dims: int,
             rope_base: float, group_size: int, bits: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused QKV projection + head split + RoPE (src/spark_qkv_rope.cpp:14-104).
    ``x[B, L, hidden]``, ``positions[B, L]`` int32 absolute positions."""
    _require_cuda(x, weight, scales, biases, positions)
    if x.ndim != 3:
        raise ValueError("x must have shape [B, L, hidden]")
    bsz, length, hidden = x.shape
    if positions.dtype != torch.int32 or positions.numel() != bsz * length:
        raise ValueError("positions must be int32 with B*L entries")
    q = torch.empty((bsz, num_heads, length, head_dim), dtype=x.dtype, device=x.device)
    k = torch.empty((bsz, num_kv_heads, length, head_dim), dtype=x.dtype, device=x.device)
    v = torch.empty_like(k)
    x2 = x.contiguous()
    pos = positions.reshape(-1).contiguous()
    weight, scales, biases = weight.contiguous(), scales.contiguous(), biases.contiguous()
    ws, ws_bytes = workspace.get(
        x.device, lib().sb_qkv_rope_workspace_size(bsz, length, hidden, num_heads, num_kv_heads, head_dim,
                                                   group_size, bits))
    check(
        lib().sb_qkv_rope(x2.data_ptr(), _code(x.dtype), weight.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                          pos.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), bsz, length, hidden,
                          num_heads, num_kv_heads, head_dim, rope_dims, float(rope_base), group_size, bits, ws,
                          ws_bytes, _stream(x)),
        "spark_qkv_rope",
    )
    return q, k, v


@qkv_rope.register_fake
def _(x, weight, scales, biases, positions, num_heads, num_kv_heads, head_dim, rope_dims, rope_base, group_size,
      bits):
    bsz, length, _ = x.shape
    return (x.new_empty((bsz, num_heads, length, head_dim)), x.new_empty((bsz, num_kv_heads, length, head_dim)),
            x.new_empty((bsz, num_kv_heads, length, head_dim)))


# ----------------------------------------------------------------- INT8-KV SDPA
@torch.library.custom_op("spark_b200::int8_sdpa_decode", mutates_args=())
def int8_sdpa_decode(q: torch.Tensor, k: torch.Tensor, k_scale: torch.Tensor, v: torch.Tensor,
                     v_scale: torch.Tensor, length: int, scale: float) -> torch.Tensor:
    """Single-query decode attention over INT8 K/V with fp16 per-token/per-head
    scales (int8_quantized_sdpa.py:156-287 decode path). ``q[B,H,1,D]`` bf16,
    ``k/v[B,KH,capacity,D]`` int8, scales ``[B,KH,capacity]`` fp16; attends to
    the first ``length`` tokens."""
    _require_cuda(q, k, k_scale, v, v_scale)
    if q.ndim != 4 or q.shape[2] != 1 or q.dtype != torch.bfloat16:
        raise ValueError("q must be bfloat16 [B, H, 1, D]")
    if k.dtype != torch.int8 or v.dtype != torch.int8 or k.shape != v.shape or k.ndim != 4:
        raise ValueError("k and v must be int8 [B, KH, capacity, D] of equal shape")
    if k_scale.dtype != torch.float16 or v_scale.dtype != torch.float16 or k_scale.shape != k.shape[:3]:
        raise ValueError("k_scale and v_scale must be float16 [B, KH, capacity]")
    bsz, heads, _, dim = q.shape
    kv_heads, capacity = k.shape[1], k.shape[2]
    out = torch.empty_like(q)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    ksc, vsc = k_scale.contiguous(), v_scale.contiguous()
    ws, ws_bytes = workspace.get(q.device, lib().sb_int8_sdpa_workspace_size(bsz, heads, kv_heads, length, dim))
    check(
        lib().sb_int8_sdpa_decode(qc.data_ptr(), kc.data_ptr(), ksc.data_ptr(), vc.data_ptr(), vsc.data_ptr(),
                                  out.data_ptr(), bsz, heads, kv_heads, length, capacity, dim, float(scale), ws,
                                  ws_bytes, _stream(q)),
        "int8_quantized_sdpa",
    )
    return out


@int8_sdpa_decode.register_fake
def _(q, k, k_scale, v, v_scale, length, scale):
    return torch.empty_like(q)


@torch.library.custom_op("spark_b200::int8_sdpa_prefill", mutates_args=())
def int8_sdpa_prefill(q: torch.Tensor, k: torch.Tensor, k_scale: torch.Tensor, v: torch.Tensor,
                      v_scale: torch.Tensor, length: int, scale: float, causal: bool) -> torch.Tensor:
    """Multi-query attention over INT8 K/V with fp16 per-token/per-head scales
    (the prefill route of int8_quantized_sdpa, int8_quantized_sdpa_prefill.py:44-57,
    for the BASELINE KV format). ``q[B,H,L,D]`` bf16 holds the last L of
    ``length`` positions; ``k/v[B,KH,capacity,D]`` int8, scales ``[B,KH,capacity]``
    fp16. ``causal``: query l sees keys ``[0, length - L + l]`` (bottom-right),
    else all ``length`` keys."""
    _require_cuda(q, k, k_scale, v, v_scale)
    if q.ndim != 4 or q.dtype != torch.bfloat16:
        raise ValueError("q must be bfloat16 [B, H, L, D]")
    if k.dtype != torch.int8 or v.dtype != torch.int8 or k.shape != v.shape or k.ndim != 4:
        raise ValueError("k and v must be int8 [B, KH, capacity, D] of equal shape")
    if k_scale.dtype != torch.float16 or v_scale.dtype != torch.float16 or k_scale.shape != k.shape[:3]:
        raise ValueError("k_scale and v_scale must be float16 [B, KH, capacity]")
    bsz, heads, q_len, dim = q.shape
    kv_heads, capacity = k.shape[1], k.shape[2]
    out = torch.empty_like(q)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    ksc, vsc = k_scale.contiguous(), v_scale.contiguous()
    check(
        lib().sb_int8_sdpa_prefill(qc.data_ptr(), kc.data_ptr(), ksc.data_ptr(), vc.data_ptr(), vsc.data_ptr(),
                                   out.data_ptr(), bsz, heads, kv_heads, q_len, length, capacity, dim, float(scale),
                                   int(bool(causal)), 0, _stream(q)),
        "int8_quantized_sdpa",
    )
    return out


@int8_sdpa_prefill.register_fake
def _(q, k, k_scale, v, v_scale, length, scale, causal):
    return torch.empty_like(q)


@torch.library.custom_op("spark_b200::bf16_sdpa_multiquery", mutates_args=())
def bf16_sdpa_multiquery(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool,
                         window: int, mask: Optional[torch.Tensor]) -> torch.Tensor:
    """BF16 multi-query attention (bf16_sdpa_multiquery.py:155-189). ``q[B,H,L,D]``
    holds the last L of N positions, ``k/v[B,KH,N,D]``; ``causal`` is the
    bottom-right mask, ``window > 0`` also limits each query to its last
    ``window`` keys, ``mask`` an optional bool/uint8 ``[L, N]`` (True = visible)
    shared by every batch row and head."""
    _require_cuda(q, k, v)
    if q.ndim != 4 or k.ndim != 4 or v.shape != k.shape:
        raise ValueError("q must be [B, H, L, D], k and v [B, KH, N, D] of equal shape")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise ValueError("q, k and v must be bfloat16")
    bsz, heads, q_len, dim = q.shape
    kv_heads, n = k.shape[1], k.shape[2]
    m = None
    if mask is not None:
        if tuple(mask.shape) != (q_len, n) or mask.dtype not in (torch.bool, torch.uint8):
            raise ValueError("mask must be bool or uint8 [L, N]")
        m = mask.to(device=q.device, dtype=torch.uint8).contiguous()
    out = torch.empty_like(q)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    check(
        lib().sb_bf16_sdpa_multiquery(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), bsz, heads,
                                      kv_heads, q_len, n, n, dim, float(scale), int(bool(causal)), int(window),
                                      m.data_ptr() if m is not None else None, n, 0, _stream(q)),
        "bf16_sdpa_multiquery",
    )
    return out


@bf16_sdpa_multiquery.register_fake
def _(q, k, v, scale, causal, window, mask):
    return torch.empty_like(q)


@torch.library.custom_op("spark_b200::gated_activation", mutates_args=())
def gated_activation(gate: torch.Tensor, up: torch.Tensor, activation: int) -> torch.Tensor:
    """``bf16(act(gate) * up)``: activation 0 SiLU (SwiGLU), 1 exact GELU (the
    Spark2_5 FFN, ``spark_mlx_llm/ops/ffn.py:98-103``). bf16 tensors of one shape."""
    _require_cuda(gate, up)
    if gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16 or gate.shape != up.shape:
        raise ValueError("gate and up must be bfloat16 tensors of one shape")
    if activation not in (0, 1):
        raise ValueError("activation must be 0 (SiLU) or 1 (GELU)")
    g, u = gate.contiguous(), up.contiguous()
    out = torch.empty_like(g)
    check(lib().sb_gated_activation(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), int(activation),
                                    _stream(g)), "gated activation")
    return out


@gated_activation.register_fake
def _(gate, up, activation):
    return torch.empty_like(gate)


@torch.library.custom_op("spark_b200::head_gate", mutates_args=())
def head_gate(x: torch.Tensor, gate_weight: torch.Tensor, attn: torch.Tensor) -> torch.Tensor:
    """Attention-output head gate (``ops/attention_output.py:91-95``): ``x[M, hidden]``,
    ``gate_weight[H, hidden]``, ``attn[M, H, D]`` bf16; returns ``attn * gate`` with
    ``gate = bf16(sigmoid(bf16(x . gate_weight[h])))``."""
    _require_cuda(x, gate_weight, attn)
    if any(t.dtype != torch.bfloat16 for t in (x, gate_weight, attn)):
        raise ValueError("x, gate_weight and attn must be bfloat16")
    if x.ndim != 2 or gate_weight.ndim != 2 or attn.ndim != 3 or gate_weight.shape[1] != x.shape[1] \
            or attn.shape[:2] != (x.shape[0], gate_weight.shape[0]):
        raise ValueError("expected x [M, hidden], gate_weight [H, hidden], attn [M, H, D]")
    xc, wc, ac = x.contiguous(), gate_weight.contiguous(), attn.contiguous()
    out = torch.empty_like(ac)
    check(lib().sb_head_gate(xc.data_ptr(), wc.data_ptr(), ac.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
                             gate_weight.shape[0], attn.shape[2], _stream(x)), "head gate")
    return out


@head_gate.register_fake
def _(x, gate_weight, attn):
    return torch.empty_like(attn)


# ---------------------------------------------------------------------- RMSNorm
@torch.library.custom_op("spark_b200::rms_norm", mutates_args=())
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``mx.fast.rms_norm`` (spark_mlx_llm/ops/ffn.py:99)."""
    _require_cuda(x, weight)
    if x.dtype not in _FLOAT_DTYPES or weight.dtype != x.dtype:
        raise ValueError("x and weight must share a floating dtype")
    d = x.shape[-1]
    x2 = x.reshape(-1, d).contiguous()
    y = torch.empty_like(x2)
    check(lib().sb_rms_norm(x2.data_ptr(), weight.contiguous().data_ptr(), y.data_ptr(), _code(x.dtype),
                            x2.shape[0], d, float(eps), _stream(x)), "rms_norm")
    return y.reshape(x.shape)


@rms_norm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)
