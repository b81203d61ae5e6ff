"""Quantizers that define the data formats on the hot path (oracle, test only).

Every function returns the exact integer codes / coefficient bit patterns the
CUDA kernels consume, so GPU and oracle see byte-identical inputs.
"""

import numpy as np

from .formats import bf16_bits, bf16_from_bits, pack_codes, round_bf16, unpack_codes

__all__ = [
    "quantize_affine_minmax",
    "conversion_rows",
    "quantize_w8_per_channel",
    "int8_to_affine_w8",
    "unpack_affine_w8",
    "quantize_per_token",
    "quantize_kv_symmetric",
    "dequantize_affine",
]


def quantize_affine_minmax(w, group_size, bits):
    """MLX-affine quantization with per-group min/max.

    For each group of ``group_size`` along the last axis:
    ``scale = bf16((max - min) / (2**bits - 1))``, ``bias = bf16(min)``,
    ``q = clip(rint((w - bias) / scale), 0, 2**bits - 1)`` in float32. A group
    whose rounded scale is zero (constant group) uses scale 1, so every code is
    0 and the group decodes to ``bias``. Returns ``(packed uint32 [N, K*bits/32],
    scales bf16 bits uint16 [N, K/G], biases bf16 bits uint16 [N, K/G])``.
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    if k % group_size:
        raise ValueError("K must be a multiple of group_size")
    levels = np.float32((1 << bits) - 1)
    grouped = w.reshape(n, k // group_size, group_size)
    lo = grouped.min(axis=-1)
    hi = grouped.max(axis=-1)
    scale = round_bf16((hi - lo) / levels)
    scale = np.where(scale == 0, np.float32(1), scale).astype(np.float32)
    bias = round_bf16(lo)
    q = np.rint((grouped - bias[..., None]) / scale[..., None])
    q = np.clip(q, 0, levels).astype(np.uint32).reshape(n, k)
    return pack_codes(q, bits), bf16_bits(scale), bf16_bits(bias)


def conversion_rows(values, kind, coefficient_dtype="BF16", channel_scales=None):
    """Restatement of the reference CPU quantizer ``_rows``.

    Follows ``spark_mlx_llm/conversion.py:551-608``:

    * ``"bf16-int4"``: asymmetric 4-bit, group 32, zero point clipped to 0..15,
      ``scale = (max(max,0) - min(min,0)) / 15`` (1 when zero), stored bf16;
      ``bias = -zero * scale``.
    * ``"bf16-int8"``: symmetric per-row int8 ``absmax / 127`` as 8-bit affine
      codes ``int8 + 128``, ``bias = -128 * scale``, both repeated per 32
      columns.
    * ``"channel-int8"``: existing int8 codes ``values`` with per-row
      ``channel_scales`` in the same affine form.

    ``coefficient_dtype`` is ``"BF16"`` (rounded, returned as uint16 bits) or
    ``"F32"`` (returned as float32), as ``conversion.py:436-441`` does for
    ``lm_head``. Returns ``(packed uint32, scales, biases)``.
    """
    values = np.asarray(values)
    rows = values.shape[0]

    def coefficient(x):
        x = np.asarray(x, dtype=np.float32)
        if coefficient_dtype == "BF16":
            bits = bf16_bits(x)
            return bits, bf16_from_bits(bits)
        return x, x

    if kind == "channel-int8":
        scales = np.asarray(channel_scales, dtype=np.float32).reshape(rows, -1)
        codes = values.astype(np.int32).reshape(rows, -1) + 128
    else:
        values = values.astype(np.float32)
        if kind == "bf16-int4":
            grouped = values.reshape(rows, -1, 32)
            lower = np.minimum(grouped.min(axis=-1), np.float32(0))
            upper = np.maximum(grouped.max(axis=-1), np.float32(0))
            scales = (upper - lower) / np.float32(15)
        elif kind == "bf16-int8":
            scales = np.max(np.abs(values), axis=-1, keepdims=True) / np.float32(127)
        else:
            raise ValueError(f"unknown kind {kind!r}")
        scales = np.where(scales == 0, np.float32(1), scales).astype(np.float32)
    scale_data, rounded = coefficient(scales)
    if kind == "bf16-int4":
        zeros = np.clip(np.rint(-lower / rounded), 0, 15).astype(np.float32)
        codes = np.clip(np.rint(grouped / rounded[..., None]) + zeros[..., None], 0, 15)
        codes = codes.reshape(values.shape)
        offsets = -zeros * rounded
        bits = 4
    else:
        if kind == "bf16-int8":
            codes = np.clip(np.rint(values / rounded), -127, 127).astype(np.int32) + 128
        offsets = -np.float32(128) * rounded
        repeat = codes.shape[1] // 32
        scale_data = np.repeat(scale_data, repeat, axis=1)
        bits = 8
    bias_data, _ = coefficient(offsets)
    if bits == 8:
        bias_data = np.repeat(bias_data, codes.shape[1] // 32, axis=1)
    return pack_codes(np.asarray(codes, dtype=np.uint32), bits), scale_data, bias_data


def quantize_w8_per_channel(w, scale_to_bf16=True):
    """Symmetric per-output-channel int8: ``scale = absmax / 127`` per row.

    The scale is optionally rounded to bf16 first (as a bf16 MLX checkpoint
    stores it, ``conversion.py:576-590``); codes are
    ``clip(rint(w / scale), -127, 127)``. Zero rows use scale 1. Returns
    ``(int8 [N, K], float32 scales [N])``.
    """
    w = np.asarray(w, dtype=np.float32)
    scale = np.max(np.abs(w), axis=1) / np.float32(127)
    scale = np.where(scale == 0, np.float32(1), scale).astype(np.float32)
    if scale_to_bf16:
        scale = round_bf16(scale)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale.astype(np.float32)


def int8_to_affine_w8(w_int8, scales, group_size):
    """Store per-channel int8 weights as MLX 8-bit affine tensors.

    Codes are ``int8 + 128`` (uint8), ``scales`` is repeated for every group
    and ``biases = -128 * scales``: the symmetric-in-affine form of
    ``conversion.py:585-592``. ``scales`` must already be bf16 values.
    Returns ``(packed uint32 [N, K/4], scales bits uint16, biases bits uint16)``.
    """
    w_int8 = np.asarray(w_int8, dtype=np.int8)
    n, k = w_int8.shape
    scales = np.asarray(scales, dtype=np.float32)
    if not np.array_equal(round_bf16(scales), scales):
        raise ValueError("scales must be bf16-representable")
    codes = (w_int8.astype(np.int32) + 128).astype(np.uint32)
    s = np.repeat(scales[:, None], k // group_size, axis=1)
    return pack_codes(codes, 8), bf16_bits(s), bf16_bits(-np.float32(128) * s)


def unpack_affine_w8(packed, scales, biases):
    """Affine W8 -> (int8 [N, K], float32 [N]); restates ``ops/linear.py:299-324``.

    Requires finite positive scales equal across a row and
    ``biases == -128 * scales``; raises ``ValueError`` otherwise. The int8
    weight is the packed word XOR ``0x80808080`` viewed as int8.
    """
    s = np.asarray(scales, dtype=np.float32)
    b = np.asarray(biases, dtype=np.float32)
    if not (
        np.all(np.isfinite(s) & (s > 0))
        and np.all(s == s[:, :1])
        and np.all(b == -128 * s)
    ):
        raise ValueError(
            "QMV requires repeated positive per-channel scales and "
            "affine biases=-128*scales"
        )
    words = np.asarray(packed, dtype=np.uint32) ^ np.uint32(0x80808080)
    return np.ascontiguousarray(words).view(np.int8), np.ascontiguousarray(s[:, 0])


def quantize_per_token(x):
    """Per-row symmetric INT8 activation quantization.

    Restates ``extensions/spark-mlx-ext/src/kernels/w8a8_quantize.metal:11-27``:
    ``amax = max|x|``; ``scale = amax / 127`` (IEEE float32 divide) or 1 when
    ``amax == 0``; ``q = clamp(rint(x / scale), -127, 127)`` with round half to
    even. Returns ``(int8 [M, K], float32 [M])``.
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1)
    scale = np.where(amax > 0, amax / np.float32(127), np.float32(1)).astype(np.float32)
    q = np.clip(np.rint(x / scale[..., None]), -127, 127).astype(np.int8)
    return q, scale


def quantize_kv_symmetric(x):
    """Symmetric INT8 per token per head with an fp16 scale.

    ``x[..., D]``: ``scale = fp16(absmax / 127)`` (fp16 1.0 when absmax is 0);
    ``q = clip(rint(x / scale), -127, 127)`` using the fp16 scale's value, so
    dequantization ``q * scale`` uses exactly the stored scale. Returns
    ``(int8 [..., D], float16 [...])``.
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1)
    s16 = (amax / np.float32(127)).astype(np.float16)
    s16 = np.where(s16 == 0, np.float16(1), s16)
    s = s16.astype(np.float32)
    q = np.clip(np.rint(x / s[..., None]), -127, 127).astype(np.int8)
    return q, s16


def dequantize_affine(packed, scales, biases, group_size, bits):
    """``W[n, k] = scale[n, k/G] * q[n, k] + bias[n, k/G]`` in float64.

    ``scales``/``biases`` are float arrays (values, not bits).
    """
    q = unpack_codes(packed, bits).astype(np.float64)
    s = np.repeat(np.asarray(scales, dtype=np.float64), group_size, axis=-1)
    b = np.repeat(np.asarray(biases, dtype=np.float64), group_size, axis=-1)
    return s * q + b
