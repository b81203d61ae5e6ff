"""The oracle against the reference's own conversion code (golden vectors).

``tests/golden/conversion_vectors.npz`` was produced by importing the
reference's ``spark_mlx_llm/conversion.py`` (``tests/golden/make_golden.py``).
"""

import os

import numpy as np
import pytest

from oracle import formats, ops, quant

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "conversion_vectors.npz")


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as data:
        return {k: data[k] for k in data.files}


def test_bf16_rounding_matches_reference(golden):
    bits = formats.bf16_bits(golden["bf16_in"])
    np.testing.assert_array_equal(bits, golden["bf16_bits"])
    np.testing.assert_array_equal(
        formats.bf16_from_bits(bits).view(np.uint32),
        golden["bf16_decoded"].view(np.uint32),
    )


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_packing_matches_reference(golden, bits):
    codes = golden[f"pack{bits}_codes"]
    words = formats.pack_codes(codes, bits)
    np.testing.assert_array_equal(words, golden[f"pack{bits}_words"])
    np.testing.assert_array_equal(formats.unpack_codes(words, bits), codes)


@pytest.mark.parametrize(
    "tag,kind,coef",
    [("w4", "bf16-int4", "BF16"), ("w8", "bf16-int8", "BF16"), ("w8f32", "bf16-int8", "F32")],
)
def test_reference_quantizer_rows(golden, tag, kind, coef):
    w = formats.bf16_from_bits(golden["rows_w_bf16_bits"])
    weight, scales, biases = quant.conversion_rows(w, kind, coef)
    np.testing.assert_array_equal(weight, golden[f"rows_{tag}_weight"])
    if coef == "F32":
        np.testing.assert_array_equal(scales.view(np.uint32), golden[f"rows_{tag}_scales"].view(np.uint32))
        np.testing.assert_array_equal(biases.view(np.uint32), golden[f"rows_{tag}_biases"].view(np.uint32))
    else:
        np.testing.assert_array_equal(scales, golden[f"rows_{tag}_scales"])
        np.testing.assert_array_equal(biases, golden[f"rows_{tag}_biases"])


def test_reference_quantizer_channel_int8(golden):
    scale = formats.bf16_from_bits(golden["chan_scale_bf16_bits"])
    weight, scales, biases = quant.conversion_rows(
        golden["chan_codes"], "channel-int8", "BF16", channel_scales=scale
    )
    np.testing.assert_array_equal(weight, golden["rows_chan_weight"])
    np.testing.assert_array_equal(scales, golden["rows_chan_scales"])
    np.testing.assert_array_equal(biases, golden["rows_chan_biases"])


def test_affine_w8_roundtrip_through_reference_layout(golden):
    """``ops/linear.py:299-324`` unpacks the reference's W8 rows back to int8."""
    w = formats.bf16_from_bits(golden["rows_w_bf16_bits"])
    weight, s_bits, b_bits = quant.conversion_rows(w, "bf16-int8", "BF16")
    w_int8, scale = quant.unpack_affine_w8(
        weight, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits)
    )
    codes = formats.unpack_codes(weight, 8).astype(np.int32) - 128
    np.testing.assert_array_equal(w_int8.astype(np.int32), codes)
    np.testing.assert_array_equal(scale, formats.bf16_from_bits(s_bits)[:, 0])


def test_unpack_affine_w8_rejects_groupwise():
    packed = np.zeros((2, 16), np.uint32)
    s = np.ones((2, 2), np.float32)
    s[0, 1] = 2.0
    with pytest.raises(ValueError):
        quant.unpack_affine_w8(packed, s, -128 * s)


def test_readme_known_answer_w8a16():
    """``extensions/spark-mlx-ext/README.md:32-48``: ones x ones -> 32."""
    y = ops.w8a16_per_channel(np.ones(32, np.float32), np.ones((4, 32), np.int8), np.ones(4, np.float32))
    np.testing.assert_array_equal(formats.round_bf16(y), np.full(4, 32.0, np.float32))


def test_affine_minmax_roundtrip_error_bound():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize_affine_minmax(w, 64, 4)
    deq = quant.dequantize_affine(packed, formats.bf16_from_bits(s), formats.bf16_from_bits(b), 64, 4)
    step = np.repeat(formats.bf16_from_bits(s), 64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + 2e-3 * np.abs(w).max())


def test_per_token_quantizer_rounding():
    x = np.array([[127.0, 0.5, -0.5, 1.5, -63.5], [0, 0, 0, 0, 0]], np.float32)
    q, s = quant.quantize_per_token(x)
    assert s[0] == np.float32(1.0) and s[1] == np.float32(1.0)
    np.testing.assert_array_equal(q[0], [127, 0, 0, 2, -64])  # half to even
    np.testing.assert_array_equal(q[1], 0)


def test_int8_matmul_exact():
    rng = np.random.default_rng(1)
    a = rng.integers(-127, 128, (3, 64), dtype=np.int8)
    b = rng.integers(-128, 128, (5, 64), dtype=np.int8)
    ref = a.astype(np.int64) @ b.astype(np.int64).T
    np.testing.assert_array_equal(ops.int8_matmul_int32(a, b), ref)


def test_rope_half_split_rotation():
    x = np.zeros((1, 1, 1, 8))
    x[..., 0] = 1.0
    out = ops.rope(x, np.array([[[1]]]), 8, 10000.0)
    assert np.isclose(out[..., 0], np.cos(1.0)).all() and np.isclose(out[..., 4], np.sin(1.0)).all()


def test_sdpa_int8_matches_affine_form():
    """Symmetric int8 is the affine 8-bit form with code = q + 128, bias = -128*s."""
    rng = np.random.default_rng(2)
    q = rng.standard_normal((1, 4, 1, 64)).astype(np.float32)
    k = rng.standard_normal((1, 2, 9, 64)).astype(np.float32)
    v = rng.standard_normal((1, 2, 9, 64)).astype(np.float32)
    kq, ks = quant.quantize_kv_symmetric(k)
    vq, vs = quant.quantize_kv_symmetric(v)
    ref = ops.sdpa_int8(q, kq, ks, vq, vs, 0.125)

    def affine(codes, s):
        packed = formats.pack_codes((codes.astype(np.int32) + 128).astype(np.uint32), 8)
        sf = s.astype(np.float32)[..., None]
        return packed, sf, -128 * sf

    alt = ops.sdpa_affine(q, affine(kq, ks), affine(vq, vs), 0.125, 64, 8)
    np.testing.assert_allclose(ref, alt, rtol=1e-12, atol=1e-12)
