"""Tensor-core (tcgen05 + TMEM) linear kernel, M >= 9 activation rows, against the
CPU oracle on a B200.

Shapes follow the linear batch sweep (M in {16, 64, 256} over the projection
shapes (K, N) in {(2560, 9728), (9728, 2560), (2560, 6144), (4096, 2560)}) and
the fused QKV + RoPE prefill case (1 x 1024 tokens), plus ragged M / N / K and
shapes that split K over a thread-block cluster.

Tolerances: bf16 / fp16 outputs |gpu - ref| <= 2e-2 + 1e-2 * |ref| against the
float64 reference with the dequantized weights rounded to the activation dtype
(this kernel, like MLX's multi-row GEMM path, dequantizes each weight tile
into the activation type before the MMA); the plain float64 dequantized
reference is checked as well for the linear layers. INT32 accumulators and the
W8A8 fp32 epilogue are bit-exact.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, ops as ref, quant  # noqa: E402

from _util import assert_close, bf16_bits_tensor, bf16_tensor, to_f32, u32_tensor  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sb():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import spark_b200.ops as sb_ops

    return sb_ops


def make_affine(rng, n, k, group, bits):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    return quant.quantize_affine_minmax(w, group, bits)


@pytest.mark.parametrize(
    "m,k,n,group,bits",
    [
        (16, 2560, 9728, 64, 4),
        (64, 9728, 2560, 64, 4),
        (256, 2560, 6144, 64, 4),
        (64, 4096, 2560, 64, 4),
        (37, 576, 200, 32, 4),    # ragged M and N, 9 K stages
        (9, 1024, 130, 128, 4),
        (48, 2560, 512, 64, 8),
        (300, 512, 256, 64, 4),   # two activation tiles
    ],
)
def test_tc_affine_linear(sb, m, k, n, group, bits):
    rng = np.random.default_rng(m * 7 + n + bits)
    packed, s_bits, b_bits = make_affine(rng, n, k, group, bits)
    x = formats.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    s, b = formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits)
    expected = ref.affine_linear(x, packed, s, b, group, bits, weight_round="bf16")
    y = sb.affine_linear(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits),
                         group, bits)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (m, n)
    assert_close(to_f32(y), expected, what="tc affine_linear")
    assert_close(to_f32(y), ref.affine_linear(x, packed, s, b, group, bits), what="tc affine_linear vs fp64")


def test_tc_affine_linear_fp16(sb):
    rng = np.random.default_rng(21)
    m, n, k, group = 32, 384, 2048, 64
    packed, s_bits, b_bits = make_affine(rng, n, k, group, 4)
    s = formats.bf16_from_bits(s_bits).astype(np.float16)
    b = formats.bf16_from_bits(b_bits).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float16)
    expected = ref.affine_linear(x.astype(np.float32), packed, s.astype(np.float32), b.astype(np.float32), group, 4,
                                 weight_round="f16")
    y = sb.affine_linear(torch.from_numpy(x).cuda(), u32_tensor(packed), torch.from_numpy(s).cuda(),
                         torch.from_numpy(b).cuda(), group, 4)
    assert y.dtype == torch.float16
    assert_close(to_f32(y), expected, what="tc affine fp16")


@pytest.mark.parametrize("m,k,n,dtype", [(16, 2560, 6144, "bfloat16"), (64, 4096, 2560, "float16"),
                                         (24, 640, 200, "bfloat16")])
def test_tc_w8a16_per_channel(sb, m, k, n, dtype):
    rng = np.random.default_rng(m + k)
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x32 = rng.standard_normal((m, k)).astype(np.float32)
    if dtype == "bfloat16":
        x = formats.round_bf16(x32)
        xt = bf16_tensor(x)
    else:
        x = x32.astype(np.float16).astype(np.float32)
        xt = torch.from_numpy(x.astype(np.float16)).cuda()
    expected = ref.w8a16_per_channel(x, wq, ws)
    y = sb.w8a16_per_channel(xt, torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda())
    assert_close(to_f32(y), expected, what="tc w8a16")


@pytest.mark.parametrize("m,k,n", [(16, 2560, 9728), (64, 9728, 2560), (256, 2560, 6144), (40, 192, 136)])
def test_tc_int8_matmul_int32_bit_exact(sb, m, k, n):
    rng = np.random.default_rng(m * 3 + n)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (n, k), dtype=np.int8)
    out = sb.int8_matmul_int32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    np.testing.assert_array_equal(out.cpu().numpy(), ref.int8_matmul_int32(a, b))


@pytest.mark.parametrize("m,k,n,with_bias", [(16, 2560, 9728, False), (64, 9728, 2560, True),
                                             (256, 4096, 2560, False), (33, 2560, 6144, True)])
def test_tc_w8a8_linear_exact(sb, m, k, n, with_bias):
    rng = np.random.default_rng(5 * m + k)
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32),
                                           scale_to_bf16=False)
    x = formats.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    bias = formats.round_bf16(rng.standard_normal(n).astype(np.float32)) if with_bias else None
    y32, _, _ = ref.w8a8_linear(x, wq, ws, bias)
    y = sb.w8a8_linear(bf16_tensor(x), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(),
                       None if bias is None else bf16_tensor(bias))
    np.testing.assert_array_equal(to_f32(y), formats.round_bf16(y32))


@pytest.mark.parametrize("bsz,length,bits", [(1, 1024, 4), (4, 16, 4), (2, 24, 8)])
def test_tc_qkv_rope(sb, bsz, length, bits):
    """QKV projection + head split + RoPE for B*L > 8 tokens (config 2's 1 x 1024)."""
    rng = np.random.default_rng(bsz * 100 + length)
    hidden, hq, hkv, d, group = 2560, 32, 8, 128, 64
    n = (hq + 2 * hkv) * d
    packed, s_bits, b_bits = make_affine(rng, n, hidden, group, bits)
    x = formats.round_bf16(rng.standard_normal((bsz, length, hidden)).astype(np.float32))
    pos = rng.integers(0, 32768, (bsz, length)).astype(np.int32)
    q_ref, k_ref, v_ref = ref.qkv_rope(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits),
                                       group, bits, hq, hkv, d, d, 1e6, pos, weight_round="bf16")
    q, k, v = sb.qkv_rope(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits),
                          torch.from_numpy(pos).cuda(), hq, hkv, d, d, 1e6, group, bits)
    assert tuple(q.shape) == (bsz, hq, length, d) and tuple(v.shape) == (bsz, hkv, length, d)
    assert_close(to_f32(q), q_ref, what="tc q")
    assert_close(to_f32(k), k_ref, what="tc k")
    assert_close(to_f32(v), v_ref, what="tc v")
