"""bf16 / fp16 rounding and MLX affine bit packing (oracle, test infrastructure).

bf16 rounding follows ``spark_mlx_llm/conversion.py:154-160``: add
``0x7FFF + lsb`` to the float32 word and keep the high half (round to nearest,
ties to even). Packing follows ``spark_mlx_llm/conversion.py:429-433``: element
``j`` of a little-endian uint32 word occupies bits ``[j*bits, (j+1)*bits)``.
"""

import numpy as np

__all__ = [
    "bf16_bits",
    "bf16_from_bits",
    "round_bf16",
    "round_fp16",
    "pack_codes",
    "unpack_codes",
]


def bf16_bits(values):
    """float32 -> bf16 bit pattern (uint16), round to nearest even.

    Restates ``conversion.py:154-160``. NaN inputs map to the canonical quiet
    NaN 0x7FC0 (the reference requires finite inputs and never reaches it).
    """
    words = np.ascontiguousarray(values, dtype="<f4").view(np.uint32)
    rounded = ((words.astype(np.uint64) + 0x7FFF + ((words >> 16) & 1)) >> 16).astype(
        np.uint16
    )
    nan = np.isnan(np.asarray(values, dtype=np.float32))
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


def bf16_from_bits(bits):
    """bf16 bit pattern (uint16) -> float32 value."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(values):
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return bf16_from_bits(bf16_bits(np.asarray(values, dtype=np.float32)))


def round_fp16(values):
    """Round float32 values to IEEE fp16 (round to nearest even), as float32."""
    return np.asarray(values, dtype=np.float32).astype(np.float16).astype(np.float32)


def pack_codes(codes, bits):
    """Pack unsigned codes along the last axis into little-endian uint32 words.

    ``codes[..., K]`` with ``K * bits % 32 == 0`` becomes ``[..., K*bits/32]``;
    restates ``conversion.py:429-433``.
    """
    if bits not in (2, 4, 8):
        raise ValueError("bits must be 2, 4 or 8")
    codes = np.asarray(codes, dtype=np.uint32)
    per_word = 32 // bits
    if codes.shape[-1] % per_word:
        raise ValueError("last dimension must fill whole uint32 words")
    if (codes >> bits).any():
        raise ValueError("code out of range for the bit width")
    shifts = np.arange(per_word, dtype=np.uint32) * bits
    groups = codes.reshape(*codes.shape[:-1], -1, per_word)
    return np.bitwise_or.reduce(groups << shifts, axis=-1).astype("<u4")


def unpack_codes(words, bits):
    """Inverse of :func:`pack_codes`: ``[..., W]`` uint32 -> ``[..., W*32/bits]``."""
    words = np.asarray(words, dtype=np.uint32)
    per_word = 32 // bits
    shifts = np.arange(per_word, dtype=np.uint32) * bits
    codes = (words[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return codes.reshape(*words.shape[:-1], -1).astype(np.uint32)
