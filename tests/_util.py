"""Helpers shared by the tests: numpy <-> torch conversions with exact bits."""

import numpy as np
import torch

from oracle import formats


def bf16_tensor(values_f32, device="cuda"):
    """float32 values (already bf16-representable or not) -> torch bf16 (RNE)."""
    bits = formats.bf16_bits(np.asarray(values_f32, dtype=np.float32))
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)


def bf16_bits_tensor(bits_u16, device="cuda"):
    return torch.from_numpy(np.asarray(bits_u16, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16).to(device)


def to_f32(t):
    return t.detach().float().cpu().numpy()


def u32_tensor(words, device="cuda"):
    return torch.from_numpy(np.asarray(words, dtype=np.uint32).view(np.int32).copy()).to(device)


def assert_close(actual, expected, rtol=1e-2, atol=2e-2, what=""):
    """The north-star tolerance: |a - e| <= atol + rtol * |e| elementwise."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    err = np.abs(a - e)
    bound = atol + rtol * np.abs(e)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} of {bad.size} outside rtol={rtol} atol={atol}; worst at {i}: "
            f"actual {a[i]!r} expected {e[i]!r}"
        )
