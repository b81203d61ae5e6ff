"""The ``spark_mlx_ext`` function surface over the B200 kernels.

Same names, argument order, keyword defaults and error classes as the
reference extension (extensions/spark-mlx-ext/spark_mlx_ext/_ext.pyi:1-44,
w4a16_qmv.py:37-98, w4a16_multirow.py:238-260, w8a16_multirow.py:43-54,
int8_quantized_sdpa.py:156-166, linear.py:9-55), taking torch CUDA tensors
instead of MLX arrays:

* ``TypeError``  - an argument is not a tensor;
* ``ValueError`` - unsupported dtype / shape / configuration, or a CPU tensor
  or stream (the reference raises for CPU execution, ``_validation.py:8-19``);
* ``RuntimeError`` - the CUDA library is missing or a kernel failed.

``stream`` is ``None`` (the current torch stream) or a ``torch.cuda.Stream``.
Inputs are never modified; outputs are new tensors. Every function runs on
``libsparkb200.so`` kernels - there is no CPU or library fallback.
"""

import contextlib
import math

import torch

from . import ops
from ._lib import DTYPE_CODES, check, lib

__all__ = [
    "W8A8Linear",
    "bf16_sdpa_multiquery",
    "int8_matmul_int32",
    "int8_quantized_sdpa",
    "is_w8a8_available",
    "spark_qkv_rope",
    "w4a16_multirow",
    "w4a16_qmv",
    "w8a16_multirow",
    "w8a16_per_channel",
    "w8a8_linear",
]


def _tensors(names, *values):
    for name, v in zip(names, values):
        if v is not None and not isinstance(v, torch.Tensor):
            raise TypeError(f"{name} must be torch tensors")


@contextlib.contextmanager
def _on(stream, operator, *tensors):
    """Run on `stream` (None = current); reject CPU placement like gpu_stream()."""
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"{operator} requires CUDA GPU execution")
    if stream is None:
        yield
        return
    if not isinstance(stream, torch.cuda.Stream):
        raise TypeError("stream must be a torch.cuda.Stream or None")
    with torch.cuda.stream(stream):
        yield


def is_w8a8_available() -> bool:
    """True when the CUDA library is loaded and device 0 is a B200 (sm_100)."""
    try:
        if not torch.cuda.is_available():
            return False
        return bool(lib().sb_device_supported(torch.cuda.current_device()))
    except (RuntimeError, OSError):
        return False


def w8a16_per_channel(x, weight, scales, *, stream=None):
    """``x @ weight.T * scales`` for signed INT8 weights (src/spark_w8a16.cpp:80-110)."""
    _tensors(("x, weight and scales",) * 3, x, weight, scales)
    with _on(stream, "w8a16_per_channel", x, weight, scales):
        return ops.w8a16_per_channel(x, weight, scales)


def int8_matmul_int32(x, weight, *, stream=None):
    """Exact int32 ``x[M,K] @ weight[N,K].T`` (src/spark_w8a8.cpp:218-228)."""
    _tensors(("x and weight",) * 2, x, weight)
    with _on(stream, "int8_matmul_int32", x, weight):
        return ops.int8_matmul_int32(x, weight)


def w8a8_linear(x, weight, scales, bias=None, *, stream=None):
    """Per-token INT8 activations x per-channel INT8 weights (src/spark_w8a8.cpp:230-257)."""
    _tensors(("x, weight, scales and bias",) * 4, x, weight, scales, bias)
    with _on(stream, "w8a8_linear", x, weight, scales, bias):
        return ops.w8a8_linear(x, weight, scales, bias)


def spark_qkv_rope(x, weight, scales, biases, q_size, kv_size, num_heads, num_key_value_heads, head_dim,
                   rope_dims, rope_base, offset, group_size=128, bits=4, *, stream=None):
    """Fused QKV projection + head split + RoPE (src/spark_qkv_rope.cpp:14-104).

    ``x[B, L, hidden]``; token l of every batch row is at position
    ``offset + l`` (the reference's scalar offset). Returns ``[q, k, v]`` with
    shapes ``[B, H, L, D]`` / ``[B, KH, L, D]``.
    """
    _tensors(("x, weight, scales and biases",) * 4, x, weight, scales, biases)
    if x.ndim != 3:
        raise ValueError("x must have shape [B, L, hidden]")
    if q_size != num_heads * head_dim or kv_size != num_key_value_heads * head_dim:
        raise ValueError("q_size and kv_size must equal heads * head_dim")
    if not isinstance(offset, int):
        raise ValueError("offset must be a Python int")
    bsz, length, _ = x.shape
    with _on(stream, "spark_qkv_rope", x, weight, scales, biases):
        positions = (offset + torch.arange(length, device=x.device, dtype=torch.int32)).repeat(bsz)
        q, k, v = ops.qkv_rope(x, weight, scales, biases, positions, num_heads, num_key_value_heads, head_dim,
                               rope_dims, float(rope_base), group_size, bits)
    return [q, k, v]


def w4a16_qmv(x, weight, scales, biases, *, stream=None):
    """One-row affine W4/G32 QMV (w4a16_qmv.py:37-98): BF16 x with K % 512 == 0,
    UINT32 weight [N, K/8] with N % 4 == 0, BF16 scales/biases [N, K/32]."""
    _tensors(("x, weight, scales and biases",) * 4, x, weight, scales, biases)
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise ValueError("W4A16 QMV requires BF16 x, scales and biases")
    if weight.dtype not in (torch.uint32, torch.int32):
        raise ValueError("W4A16 QMV requires UINT32-packed W4 weights")
    if x.ndim < 1 or math.prod(x.shape[:-1]) != 1:
        raise ValueError("W4A16 QMV requires exactly one activation row")
    k = x.shape[-1]
    if k <= 0 or k % 512:
        raise ValueError("W4A16 QMV requires positive K divisible by 512")
    if weight.ndim != 2:
        raise ValueError("W4A16 packed weight must have shape [N,K/8]")
    n = weight.shape[0]
    if n <= 0 or n % 4 or weight.shape[1] != k // 8:
        raise ValueError("W4A16 QMV requires positive N divisible by 4 and weight [N,K/8]")
    if tuple(scales.shape) != (n, k // 32) or biases.shape != scales.shape:
        raise ValueError("W4A16 QMV requires scales and biases with shape [N,K/32]")
    with _on(stream, "W4A16 QMV", x, weight, scales, biases):
        return ops.affine_linear(x, weight, scales, biases, 32, 4)


def w4a16_multirow(x, weight, scales, biases, *, algorithm="wide", k_lanes=8, splits=4, simdgroups=2,
                   layout="native", static_layout=False, multiply_mode=False, static_slice=False,
                   contiguous_k=False, stream=None):
    """Affine W4/G32 matmul for 2..8 BF16 activation rows (w4a16_multirow.py:238-260).

    The Metal schedule knobs (algorithm, k_lanes, splits, simdgroups, static
    options) are accepted for signature compatibility; the B200 kernel picks its
    own schedule. Only the native layout exists (no prepared layouts)."""
    _tensors(("x, weight, scales and biases",) * 4, x, weight, scales, biases)
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise ValueError("W4 multirow requires BF16 x, scales and biases")
    if weight.dtype not in (torch.uint32, torch.int32):
        raise ValueError("W4 multirow requires UINT32-packed weights")
    m = math.prod(x.shape[:-1]) if x.ndim >= 1 else 0
    if m < 2 or m > 8:
        raise ValueError("W4 multirow requires 2..8 activation rows")
    k = x.shape[-1]
    if k <= 0 or k % 32:
        raise ValueError("W4 multirow requires positive K divisible by 32")
    if weight.ndim != 2 or weight.shape[0] <= 0 or weight.shape[1] != k // 8:
        raise ValueError("W4 multirow requires positive weight [N,K/8]")
    if tuple(scales.shape) != (weight.shape[0], k // 32) or biases.shape != scales.shape:
        raise ValueError("W4 multirow requires metadata [N,K/32]")
    if layout != "native":
        raise ValueError("layout must be native (prepared layouts are not used on B200)")
    for name, flag in (("static_layout", static_layout), ("multiply_mode", multiply_mode),
                       ("static_slice", static_slice), ("contiguous_k", contiguous_k)):
        if not isinstance(flag, bool):
            raise ValueError(f"{name} must be bool")
    with _on(stream, "W4 multirow", x, weight, scales, biases):
        return ops.affine_linear(x, weight, scales, biases, 32, 4)


def w8a16_multirow(x, weight, scales, *, output_dtype=None, variant="matrix", tile_rows=8, k_lanes=8,
                   simdgroups=4, stream=None):
    """``x @ weight.T * scales`` for 2..8 BF16 rows (w8a16_multirow.py:43-75);
    ``output_dtype`` BF16 (default) or FP32. Schedule knobs are accepted for
    signature compatibility."""
    _tensors(("x, weight and scales",) * 3, x, weight, scales)
    if x.dtype != torch.bfloat16:
        raise ValueError("W8 multirow requires BF16 x")
    m = math.prod(x.shape[:-1]) if x.ndim >= 1 else 0
    if m < 2 or m > 8:
        raise ValueError("W8 multirow requires 2..8 activation rows")
    if x.shape[-1] <= 0 or x.shape[-1] % 32:
        raise ValueError("W8 multirow requires positive K divisible by 32")
    if output_dtype not in (None, torch.bfloat16, torch.float32):
        raise ValueError("output_dtype must be bfloat16 or float32")
    with _on(stream, "W8 multirow", x, weight, scales):
        y = ops.w8a16_per_channel(x, weight, scales)
    return y if output_dtype in (None, torch.bfloat16) else y.float()


def int8_quantized_sdpa(queries, keys, values, *, scale, group_size=32, bits=8, mask=None,
                        single_pass_max_length=1023):
    """Attention over MLX affine packed KV tuples ``(packed, scales, biases)``
    (int8_quantized_sdpa.py:156-287): ``queries[B,H,L,D]``; packed uint32
    ``[B,KH,N,D*bits/32]``; scales/biases ``[B,KH,N,D/G]`` in the query dtype.
    ``mask`` is None or ``"causal"`` (bottom-right). fp32 scores, softmax and
    P.V; output in the query dtype. ``single_pass_max_length`` is the Metal
    decode-pass policy, validated and otherwise unused.
    """
    if type(single_pass_max_length) is not int or single_pass_max_length < 0:
        raise ValueError("single_pass_max_length must be a nonnegative Python int")
    if not isinstance(queries, torch.Tensor) or queries.ndim != 4 or len(keys) != 3 or len(values) != 3:
        raise ValueError("Expected Q[B,H,L,D] and affine (packed, scales, biases) KV tuples")
    _tensors(("keys and values",) * 6, *keys, *values)
    batch, heads, length, dim = queries.shape
    if any(x.ndim != 4 for x in (*keys, *values)):
        raise ValueError("Every packed KV and metadata array must have four dimensions")
    kv_heads, n = keys[0].shape[1:3]
    if min(batch, heads, length, dim, kv_heads, n) <= 0 or heads % kv_heads:
        raise ValueError("Nonempty inputs and query heads divisible by KV heads required")
    if not isinstance(scale, (float, int)) or not math.isfinite(scale):
        raise ValueError("scale must be a finite Python number")
    if bits not in (2, 4, 8) or group_size not in (32, 64, 128):
        raise ValueError("Supported affine formats: bits 2/4/8, group size 32/64/128")
    pack = 32 // bits
    widths = {}
    for name, tensors in (("key", keys), ("value", values)):
        packed, s, b = tensors
        width = dim if name == "key" else packed.shape[-1] * pack
        if (width <= 0 or width % group_size or tuple(packed.shape) != (batch, kv_heads, n, width // pack)
                or tuple(s.shape) != (batch, kv_heads, n, width // group_size) or b.shape != s.shape
                or packed.dtype not in (torch.uint32, torch.int32) or s.dtype != queries.dtype
                or b.dtype != queries.dtype):
            raise ValueError(f"Incompatible {name} packed shape, affine metadata or dtype")
        widths[name] = width
    if queries.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("Q and metadata must be float16, bfloat16 or float32")
    if mask is not None and not (isinstance(mask, str) and mask == "causal"):
        if isinstance(mask, str):
            raise ValueError("mask string must be 'causal'")
        raise ValueError("array masks are not supported; use None or 'causal'")
    causal = mask == "causal"
    if causal and length > n:
        raise ValueError("causal queries need at least as many keys as queries")
    if widths["key"] > 256 or widths["value"] > 256:
        raise ValueError("head dimensions above 256 are not supported")
    with _on(None, "int8_quantized_sdpa", queries, *keys, *values):
        out = torch.empty((batch, heads, length, widths["value"]), dtype=queries.dtype, device=queries.device)
        q = queries.contiguous()
        kt = [t.contiguous() for t in keys]
        vt = [t.contiguous() for t in values]
        ws, ws_bytes = ops.workspace.get(
            queries.device, lib().sb_affine_sdpa_workspace_size(batch, heads, length, n, widths["value"]))
        code = DTYPE_CODES[str(queries.dtype).replace("torch.", "")]
        check(
            lib().sb_affine_sdpa(q.data_ptr(), code, kt[0].data_ptr(), kt[1].data_ptr(), kt[2].data_ptr(),
                                 vt[0].data_ptr(), vt[1].data_ptr(), vt[2].data_ptr(), out.data_ptr(), batch, heads,
                                 kv_heads, length, n, widths["key"], widths["value"], group_size, bits, float(scale),
                                 1 if causal else 0, ws, ws_bytes,
                                 torch.cuda.current_stream(queries.device).cuda_stream),
            "int8_quantized_sdpa",
        )
    return out


def bf16_sdpa_multiquery(queries, keys, values, *, scale, mask=None, stream=None):
    """BF16 SDPA for a few queries (speculative verification) and the sliding
    layers (bf16_sdpa_multiquery.py:155-189): Q ``[B,H,M,D]``, K/V ``[B,KH,N,D]``
    BF16; ``mask`` None, ``"causal"`` (bottom-right) or a boolean array
    broadcast to ``[B,Hq,M,N]`` that is the same for every batch row and head
    (shape ``[M,N]``, ``[1,M,N]`` or ``[1,1,M,N]``). fp32 scores and softmax,
    BF16 output of Q's first three dimensions."""
    if not all(isinstance(t, torch.Tensor) for t in (queries, keys, values)):
        raise TypeError("queries, keys and values must be torch tensors")
    if queries.ndim != 4 or keys.ndim != 4 or values.shape != keys.shape:
        raise ValueError("Expected Q[B,H,M,D] and K/V[B,KH,N,D] of equal shape")
    if any(t.dtype != torch.bfloat16 for t in (queries, keys, values)):
        raise ValueError("Q, K and V must be bfloat16")
    batch, heads, m, dim = queries.shape
    kv_heads, n = keys.shape[1], keys.shape[2]
    if keys.shape[0] != batch or keys.shape[3] != dim or heads % kv_heads or min(batch, heads, m, n) <= 0:
        raise ValueError("Incompatible Q/K/V geometry")
    if not isinstance(scale, (float, int)) or not math.isfinite(scale):
        raise ValueError("scale must be a finite Python number")
    causal, bool_mask = False, None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError("mask string must be 'causal'")
        causal = True
    elif mask is not None:
        if not isinstance(mask, torch.Tensor) or mask.dtype != torch.bool:
            raise ValueError("array masks must be boolean")
        lead = tuple(mask.shape[:-2])
        if mask.ndim < 2 or tuple(mask.shape[-2:]) != (m, n) or any(d != 1 for d in lead) or len(lead) > 2:
            raise ValueError("boolean masks must be [M,N] (shared by every batch row and head)")
        bool_mask = mask.reshape(m, n)
    if m > n:
        raise ValueError("more queries than keys")
    with _on(stream, "bf16_sdpa_multiquery", queries, keys, values):
        return ops.bf16_sdpa_multiquery(queries, keys, values, float(scale), causal, 0, bool_mask)


class W8A8Linear(torch.nn.Module):
    """Linear layer on existing symmetric per-channel INT8 weights (linear.py:9-55).

    ``weight`` INT8 ``[out_features, in_features]``; ``scales`` FP32 ``[N]`` or
    ``[N, 1]``; optional floating ``bias [N]``. Activations are quantized per
    token on every call. Inference only (parameters are buffers).
    """

    def __init__(self, weight, scales, bias=None):
        super().__init__()
        if weight.ndim != 2 or weight.dtype != torch.int8:
            raise ValueError("weight must be an INT8 matrix [N, K]")
        n, k = weight.shape
        if n <= 0 or k <= 0 or k % 32 or k > 131040:
            raise ValueError("N must be positive; K must be a multiple of 32 in [32, 131040]")
        if scales.dtype != torch.float32 or tuple(scales.shape) not in ((n,), (n, 1)):
            raise ValueError("scales must be FP32 with shape [N] or [N, 1]")
        if bias is not None and (tuple(bias.shape) != (n,) or
                                 bias.dtype not in (torch.float16, torch.bfloat16, torch.float32)):
            raise ValueError("bias must be a floating array of shape [N]")
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("bias", bias)

    @property
    def input_dims(self):
        return self.weight.shape[1]

    @property
    def output_dims(self):
        return self.weight.shape[0]

    def forward(self, x):
        return w8a8_linear(x, self.weight, self.scales, self.bias)

    def extra_repr(self):
        return f"input_dims={self.input_dims}, output_dims={self.output_dims}, bias={self.bias is not None}"
