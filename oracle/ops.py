"""Reference arithmetic of the hot-path operators (oracle, test only).

Floating-point results are computed in float64 from the exact quantized inputs
(the "fp32 dequantized reference" of the tolerance contract) and rounded to
bf16 only where the reference stores a bf16 tensor. Integer results are exact.
"""

import math

import numpy as np

from .formats import round_bf16, unpack_codes
from .quant import dequantize_affine, quantize_per_token

__all__ = [
    "affine_linear",
    "w8a16_per_channel",
    "int8_matmul_int32",
    "w8a8_linear",
    "rope_inv_freq",
    "rope",
    "qkv_rope",
    "sdpa_int8",
    "sdpa_affine",
    "rms_norm",
    "swiglu",
]


def affine_linear(x, packed, scales, biases, group_size, bits, weight_round=None):
    """``y = x @ W^T`` with MLX-affine ``W = scale * q + bias``, float64.

    The arithmetic of ``mx.quantized_matmul(x, w, scales, biases,
    transpose=True, group_size, bits, mode="affine")`` as called at
    ``spark_mlx_llm/ops/linear.py:180-191``; the reference kernels evaluate
    it as ``scale * sum(q*x) + bias * sum(x)`` per group in fp32
    (``spark_mlx_ext/_w4a16_sources.py:24-39``), which equals this up to fp32
    rounding. ``scales``/``biases`` are float values. Returns float64
    ``[..., N]`` (unrounded).

    ``weight_round`` ("bf16" or "f16") rounds the dequantized weights to the
    activation dtype first: the multi-row (GEMM) path of mx.quantized_matmul
    (mlx 0.32.4, a dependency pinned at ``uv.lock:421-422``) dequantizes each
    weight tile into the activation type before its matrix multiply, and the
    tensor-core kernel for more than 8 rows does the same.
    """
    x = np.asarray(x, dtype=np.float64)
    w = dequantize_affine(packed, scales, biases, group_size, bits)
    if weight_round == "bf16":
        w = round_bf16(w.astype(np.float32)).astype(np.float64)
    elif weight_round == "f16":
        w = w.astype(np.float16).astype(np.float64)
    return x @ w.T


def w8a16_per_channel(x, weight, scales):
    """``bf16((x . w_int8) * scale[n])``; ``src/kernels/w8a16_matvec.metal:40-94``.

    The dot product is exact in float64, scaled in float64 and rounded once.
    """
    x = np.asarray(x, dtype=np.float64)
    acc = x @ np.asarray(weight, dtype=np.float64).T
    return acc * np.asarray(scales, dtype=np.float64).reshape(-1)


def int8_matmul_int32(x_int8, w_int8):
    """Exact ``x[M,K] @ w[N,K]^T`` as int32 (``src/spark_w8a8.cpp:218-228``).

    K <= 131040 keeps full-range int8 sums inside int32 (``:57-61``).
    """
    acc = np.asarray(x_int8, dtype=np.int64) @ np.asarray(w_int8, dtype=np.int64).T
    if np.abs(acc).max(initial=0) >= 2**31:
        raise OverflowError("int32 accumulator overflow")
    return acc.astype(np.int32)


def w8a8_linear(x, w_int8, w_scales, bias=None):
    """W8A8 linear: per-token INT8 activations, exact INT32 GEMM, fp32 epilogue.

    Quantizer ``w8a8_quantize.metal:11-27``; epilogue
    ``float(acc) * scale_a[m] * scale_w[n] + bias[n]`` evaluated left to right
    in float32 without contraction (``w8a8_matmul.metal:73-74``). Returns the
    float32 epilogue value (before the cast to the activation dtype), the int32
    accumulators and the activation scales.
    """
    xq, sa = quantize_per_token(x)
    acc = int8_matmul_int32(xq, w_int8)
    y = acc.astype(np.float32) * sa[:, None]
    y = (y * np.asarray(w_scales, dtype=np.float32).reshape(1, -1)).astype(np.float32)
    b = np.zeros(y.shape[1], np.float32) if bias is None else np.asarray(bias, np.float32)
    return (y + b[None, :]).astype(np.float32), acc, sa


def rope_inv_freq(dims, base):
    """``inv_freq[i] = base ** (-2i/dims)``, i < dims/2, rounded once to float32.

    Non-traditional RoPE (RoFormer rotary embedding applied to the two halves
    of the rotated dimensions), as ``nn.RoPE(dims, traditional=False,
    base)`` is configured at ``spark_mlx_llm/model.py:166-170``.
    """
    i = np.arange(dims // 2, dtype=np.float64)
    return (np.float64(base) ** (-2.0 * i / dims)).astype(np.float32)


def rope(x, positions, dims, base):
    """Rotate ``x[..., L, D]`` at integer ``positions`` (broadcast over leading).

    The angle is the float32 product ``float32(pos) * inv_freq``; cos/sin and
    the rotation are evaluated in float64. Pairs are ``(i, i + dims/2)`` for
    ``i < dims/2``; columns ``>= dims`` pass through. Returns float64.
    """
    x = np.asarray(x, dtype=np.float64)
    half = dims // 2
    inv = rope_inv_freq(dims, base)
    pos = np.asarray(positions, dtype=np.float32)
    angle = (pos[..., None] * inv).astype(np.float32).astype(np.float64)
    c, s = np.cos(angle), np.sin(angle)
    out = x.copy()
    a, b = x[..., :half], x[..., half:dims]
    out[..., :half] = a * c - b * s
    out[..., half:dims] = b * c + a * s
    return out


def qkv_rope(x, packed, scales, biases, group_size, bits, n_heads, n_kv_heads,
             head_dim, rope_dims, rope_base, positions, weight_round=None):
    """Fused QKV projection + head split + RoPE (``src/spark_qkv_rope.cpp:83-101``).

    ``x[B, L, H]``; ``positions[B, L]`` integers. The projection is rounded to
    bf16 (the reference materialises ``quantized_matmul`` in the activation
    dtype), split at ``[q_size, q_size + kv_size]``, reshaped to
    ``[B, heads, L, head_dim]``; Q and K are rotated and rounded to bf16 again.
    Returns bf16-valued float32 ``(q, k, v)``.
    """
    x = np.asarray(x, dtype=np.float32)
    bsz, length, _ = x.shape
    qkv = round_bf16(affine_linear(x, packed, scales, biases, group_size, bits, weight_round))
    q_size, kv_size = n_heads * head_dim, n_kv_heads * head_dim

    def heads(part, n):
        return part.reshape(bsz, length, n, head_dim).transpose(0, 2, 1, 3)

    q = heads(qkv[..., :q_size], n_heads)
    k = heads(qkv[..., q_size:q_size + kv_size], n_kv_heads)
    v = heads(qkv[..., q_size + kv_size:], n_kv_heads)
    pos = np.asarray(positions).reshape(bsz, 1, length)
    q = round_bf16(rope(q, pos, rope_dims, rope_base))
    k = round_bf16(rope(k, pos, rope_dims, rope_base))
    return q, k, np.ascontiguousarray(v)


def _attend(q, k, v, scale, causal):
    """Softmax attention in float64; ``q[B,H,L,D]``, ``k/v[B,KH,N,D]`` (GQA)."""
    bsz, heads, length, dim = q.shape
    kv_heads, n = k.shape[1], k.shape[2]
    rep = heads // kv_heads
    k = np.repeat(k, rep, axis=1)
    v = np.repeat(v, rep, axis=1)
    scores = np.einsum("bhld,bhnd->bhln", q * scale, k)
    if causal:
        # bottom-right aligned causal mask (int8_quantized_sdpa.py:139-140)
        rows = np.arange(n - length, n)[:, None]
        scores = np.where(rows >= np.arange(n)[None, :], scores, -np.inf)
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhln,bhnd->bhld", p, v)


def sdpa_masked(q, k, v, scale, causal=False, window=0, mask=None):
    """Softmax attention in float64 with the masks of ``mx.fast.scaled_dot_product_attention``
    as ``bf16_sdpa_multiquery`` uses them (``bf16_sdpa_multiquery.py:155-189``):
    bottom-right causal, a sliding window of the last ``window`` keys up to the
    query's position, and a boolean ``mask[L, N]`` (True = visible). A query
    with no visible key returns zeros. ``q[B,H,L,D]``, ``k/v[B,KH,N,D]``."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    bsz, heads, length, dim = q.shape
    kv_heads, n = k.shape[1], k.shape[2]
    rep = heads // kv_heads
    k = np.repeat(k, rep, axis=1)
    v = np.repeat(v, rep, axis=1)
    scores = np.einsum("bhld,bhnd->bhln", q * scale, k)
    pos = np.arange(n - length, n)[:, None]
    keys = np.arange(n)[None, :]
    visible = np.ones((length, n), bool)
    if causal:
        visible &= keys <= pos
    if window > 0:
        visible &= keys > pos - window
    if mask is not None:
        visible &= np.asarray(mask, bool)
    scores = np.where(visible, scores, -np.inf)
    m = scores.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(scores - m)
    s = p.sum(axis=-1, keepdims=True)
    return np.einsum("bhln,bhnd->bhld", p / np.where(s > 0, s, 1.0), v)


def sdpa_int8(q, k_int8, k_scale, v_int8, v_scale, scale, causal=False):
    """INT8-KV attention (symmetric per token per head, fp16 scales).

    The staged recipe of ``spark_mlx_ext/int8_quantized_sdpa.py:122-153``
    (scaled scores, bottom-right causal mask, precise softmax, ``P @ V``)
    over ``K = k_int8 * k_scale``, ``V = v_int8 * v_scale`` in float64.
    ``q[B,H,L,D]``, ``k_int8/v_int8[B,KH,N,D]``, scales ``[B,KH,N]``.
    Returns float64 ``[B,H,L,D]``.
    """
    k = np.asarray(k_int8, np.float64) * np.asarray(k_scale, np.float64)[..., None]
    v = np.asarray(v_int8, np.float64) * np.asarray(v_scale, np.float64)[..., None]
    return _attend(np.asarray(q, np.float64), k, v, scale, causal)


def sdpa_affine(q, keys, values, scale, group_size, bits, causal=False):
    """Attention over MLX affine KV tuples ``(packed, scales, biases)``.

    ``int8_quantized_sdpa.py:156-166`` inputs: packed ``[B,KH,N,D*bits/32]``
    uint32, scales/biases ``[B,KH,N,D/G]``. Dequantized per group in float64.
    """
    def deq(t):
        packed, s, b = t
        codes = unpack_codes(packed, bits).astype(np.float64)
        s = np.repeat(np.asarray(s, np.float64), group_size, axis=-1)
        b = np.repeat(np.asarray(b, np.float64), group_size, axis=-1)
        return s * codes + b

    return _attend(np.asarray(q, np.float64), deq(keys), deq(values), scale, causal)


def rms_norm(x, weight, eps):
    """``x * rsqrt(mean(x^2) + eps) * weight`` in float64 (``mx.fast.rms_norm``,
    ``spark_mlx_llm/ops/ffn.py:99``). Returns float64."""
    x = np.asarray(x, dtype=np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * r * np.asarray(weight, dtype=np.float64)


def gelu(x):
    """Exact GELU ``0.5 x (1 + erf(x / sqrt 2))`` (``nn.gelu`` of the reference's
    Spark2_5 FFN, ``spark_mlx_llm/ops/ffn.py:102``), float64."""
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * x * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))


def gelu_glu(gate, up):
    """``gelu(gate) * up`` in float64 from bf16 gate/up (``ops/ffn.py:98-103``)."""
    return gelu(gate) * np.asarray(up, dtype=np.float64)


def head_gate(x, gate_weight, attn):
    """Attention-output head gate (``spark_mlx_llm/ops/attention_output.py:91-95``):
    ``gate = bf16(sigmoid(float32(bf16(x @ gate_weight.T))))`` per row and head,
    ``attn[m, h, :] * gate`` in float64. ``x[M, hidden]``, ``gate_weight[H, hidden]``,
    ``attn[M, H, D]``."""
    d = round_bf16((np.asarray(x, np.float64) @ np.asarray(gate_weight, np.float64).T).astype(np.float32))
    g = round_bf16((1.0 / (1.0 + np.exp(-d.astype(np.float64)))).astype(np.float32))
    return np.asarray(attn, np.float64) * g.astype(np.float64)[:, :, None]


def swiglu(gate, up):
    """``silu(gate) * up`` in float64 from bf16 gate/up (the synthetic model's
    activation; the reference Spark2_5 uses ``gelu`` at ``ops/ffn.py:102``)."""
    g = np.asarray(gate, dtype=np.float64)
    return g / (1.0 + np.exp(-g)) * np.asarray(up, dtype=np.float64)
