"""The device-side quantizers produce the oracle's bytes (checked on CPU)."""

import numpy as np
import pytest
import torch

from oracle import formats, quant
from spark_b200 import quantize


@pytest.mark.parametrize("bits,group", [(4, 64), (4, 32), (8, 64), (4, 128)])
def test_affine_minmax_matches_oracle(bits, group):
    rng = np.random.default_rng(bits * 100 + group)
    w = (rng.standard_normal((24, 512)) * 0.02).astype(np.float32)
    w[3, :group] = 0.25  # constant group -> scale 1
    packed, s, b = quantize.quantize_affine_minmax(torch.from_numpy(w), group, bits)
    p_ref, s_ref, b_ref = quant.quantize_affine_minmax(w, group, bits)
    np.testing.assert_array_equal(packed.numpy().view(np.uint32), p_ref)
    np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), s_ref)
    np.testing.assert_array_equal(b.view(torch.int16).numpy().view(np.uint16), b_ref)


@pytest.mark.parametrize("to_bf16", [True, False])
def test_w8_per_channel_matches_oracle(to_bf16):
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    w[5] = 0
    q, s = quantize.quantize_w8_per_channel(torch.from_numpy(w), scale_to_bf16=to_bf16)
    q_ref, s_ref = quant.quantize_w8_per_channel(w, scale_to_bf16=to_bf16)
    np.testing.assert_array_equal(q.numpy(), q_ref)
    np.testing.assert_array_equal(s.numpy().view(np.uint32), s_ref.view(np.uint32))


def test_pack_codes_matches_reference_layout():
    codes = np.arange(64, dtype=np.uint32).reshape(2, 32) % 16
    got = quantize.pack_codes(torch.from_numpy(codes.astype(np.int32)), 4).numpy().view(np.uint32)
    np.testing.assert_array_equal(got, formats.pack_codes(codes, 4))
