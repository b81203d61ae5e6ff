"""GPU parity of every operator against the CPU oracle (runs on a B200).

Tolerance for bf16 outputs: |gpu - ref| <= 2e-2 + 1e-2 * |ref| against the
float64 dequantized reference. Integer outputs
(INT8 quantizer, INT32 accumulators) and the W8A8 fp32 epilogue are exact.
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
    packed, s_bits, b_bits = quant.quantize_affine_minmax(w, group, bits)
    return packed, s_bits, b_bits


@pytest.mark.parametrize(
    "m,k,n,group,bits",
    [
        (1, 2560, 9728, 64, 4),  # config 0
        (4, 9728, 2560, 64, 4),
        (8, 2560, 6144, 64, 4),
        (3, 4096, 2560, 64, 4),
        (1, 2560, 1000, 32, 4),
        (2, 2048, 512, 128, 4),
        (1, 2560, 6144, 64, 8),
        (5, 1024, 96, 32, 8),
        (7, 512, 64, 128, 8),
        (16, 1024, 256, 64, 4),  # M > 8: tensor-core kernel
    ],
)
def test_affine_linear_matches_oracle(sb, m, k, n, group, bits):
    rng = np.random.default_rng(1000 + m + n + bits)
    packed, s_bits, b_bits = make_affine(rng, n, k, group, bits)
    x = formats.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    expected = ref.affine_linear(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits), group, bits)
    y = sb.affine_linear(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits),
                         group, bits)
    torch.cuda.synchronize()
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (m, n)
    assert_close(to_f32(y), expected, what="affine_linear")
    if m <= 8:
        # the weight-streaming kernel multiplies the exact codes: almost every
        # output equals the correctly rounded bf16 value (M > 8 runs the
        # tensor-core kernel, which rounds the dequantized weights to bf16)
        exact = np.mean(to_f32(y) == formats.round_bf16(expected.astype(np.float32)))
        assert exact > 0.97, exact


def test_affine_linear_fp16_activations(sb):
    rng = np.random.default_rng(7)
    n, k, group = 512, 1024, 64
    packed, s_bits, b_bits = make_affine(rng, n, k, group, 4)
    s = formats.bf16_from_bits(s_bits).astype(np.float16)
    b = formats.bf16_from_bits(b_bits).astype(np.float16)
    x = rng.standard_normal((3, k)).astype(np.float16)
    expected = ref.affine_linear(x.astype(np.float32), packed, s.astype(np.float32), b.astype(np.float32), group, 4)
    y = sb.affine_linear(torch.from_numpy(x).cuda(), u32_tensor(packed), torch.from_numpy(s).cuda(),
                         torch.from_numpy(b).cuda(), group, 4)
    assert y.dtype == torch.float16
    assert_close(to_f32(y), expected, what="affine fp16")


@pytest.mark.parametrize("m,k,n,group,bits", [(1, 2496, 300, 64, 4), (2, 1088, 130, 64, 8), (6, 1216, 72, 64, 4),
                                              (1, 576, 40, 32, 4), (3, 1280, 48, 128, 4)])
def test_affine_linear_ragged_k_wide_range(sb, m, k, n, group, bits):
    """K ending inside a 128-byte weight stage, partial row blocks, and activation
    groups spread over nine decades (plus an all-zero group): the staged operands
    are scaled per group by a power of two, which must stay exact."""
    rng = np.random.default_rng(50 + m + k + n)
    packed, s_bits, b_bits = make_affine(rng, n, k, group, bits)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= np.repeat(10.0 ** rng.uniform(-6, 3, size=(m, k // group)), group, axis=1).astype(np.float32)
    x[:, :group] = 0.0
    x = formats.round_bf16(x)
    expected = ref.affine_linear(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits), group, bits)
    y = sb.affine_linear(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits),
                         group, bits)
    assert_close(to_f32(y), expected, what="affine ragged/wide")


def test_w8a16_wide_range(sb):
    rng = np.random.default_rng(77)
    m, k, n = 2, 1088, 100
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= np.repeat(10.0 ** rng.uniform(-5, 3, size=(m, k // 64)), 64, axis=1).astype(np.float32)
    x = formats.round_bf16(x)
    expected = ref.w8a16_per_channel(x, wq, ws)
    y = sb.w8a16_per_channel(bf16_tensor(x), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda())
    assert_close(to_f32(y), expected, what="w8a16 wide")


def test_w8a16_known_answer(sb):
    """extensions/spark-mlx-ext/README.md:32-48: ones x ones -> 32."""
    x = torch.ones(64, dtype=torch.bfloat16, device="cuda")
    w = torch.ones((4, 64), dtype=torch.int8, device="cuda")
    s = torch.ones(4, dtype=torch.float32, device="cuda")
    y = sb.w8a16_per_channel(x, w, s)
    assert y.tolist() == [64.0] * 4


@pytest.mark.parametrize("m,k,n", [(1, 2560, 6144), (1, 4096, 2560), (8, 2560, 6144), (3, 640, 200)])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_w8a16_per_channel(sb, m, k, n, dtype):
    rng = np.random.default_rng(m * 31 + n)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, ws = quant.quantize_w8_per_channel(w)
    x32 = rng.standard_normal((m, k)).astype(np.float32)
    if dtype == "bfloat16":
        x = formats.round_bf16(x32)
        xt = bf16_tensor(x)
    else:
        x = x32.astype(np.float16).astype(np.float32)
        xt = torch.from_numpy(x.astype(np.float16)).cuda()
    expected = ref.w8a16_per_channel(x, wq, ws)
    y = sb.w8a16_per_channel(xt, torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda())
    assert_close(to_f32(y), expected, what="w8a16")


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_quantize_per_token_exact(sb, dtype):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, 2560)) * 3).astype(np.float32)
    x[2] = 0.0
    x[3, :5] = [127.0, 0.5, -0.5, 1.5, -63.5]
    x[3, 5:] = 0.0
    if dtype == "bfloat16":
        x = formats.round_bf16(x)
        xt = bf16_tensor(x)
    else:
        xt = torch.from_numpy(x).cuda()
    q_ref, s_ref = quant.quantize_per_token(x)
    q, s = sb.quantize_per_token(xt)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(1, 2560, 9728), (4, 9728, 2560), (8, 2560, 6144), (13, 4096, 2560),
                                   (2, 64, 33), (256, 256, 96)])
def test_int8_matmul_int32_bit_exact(sb, m, k, n):
    rng = np.random.default_rng(m + k + n)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (n, k), dtype=np.int8)
    out = sb.int8_matmul_int32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    np.testing.assert_array_equal(out.cpu().numpy(), ref.int8_matmul_int32(a, b))


@pytest.mark.parametrize("m,k,n,with_bias", [(1, 2560, 9728, False), (4, 2560, 6144, True), (8, 4096, 2560, False),
                                             (16, 2560, 256, True)])
def test_w8a8_linear_exact_epilogue(sb, m, k, n, with_bias):
    """W8A8 (config 1): per-channel int8 weights N(0,0.02), per-token int8 activations."""
    rng = np.random.default_rng(11 + m)
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32),
                                           scale_to_bf16=False)
    x = formats.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    bias = formats.round_bf16(rng.standard_normal(n).astype(np.float32)) if with_bias else None
    y32, acc, _ = ref.w8a8_linear(x, wq, ws, bias)
    y = sb.w8a8_linear(bf16_tensor(x), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(),
                       None if bias is None else bf16_tensor(bias))
    np.testing.assert_array_equal(to_f32(y), formats.round_bf16(y32))


@pytest.mark.parametrize("bsz,length,bits", [(1, 1, 4), (8, 1, 4), (2, 3, 8)])
def test_qkv_rope_matches_oracle(sb, bsz, length, bits):
    """Config 2: hidden 2560, 32 q / 8 kv heads, head_dim 128, theta 1e6, positions in [0, 32768)."""
    rng = np.random.default_rng(bsz * 10 + length)
    hidden, hq, hkv, d, group = 2560, 32, 8, 128, 64
    n = (hq + 2 * hkv) * d
    packed, s_bits, b_bits = make_affine(rng, n, hidden, group, bits)
    x = formats.round_bf16(rng.standard_normal((bsz, length, hidden)).astype(np.float32))
    pos = rng.integers(0, 32768, (bsz, length)).astype(np.int32)
    q_ref, k_ref, v_ref = ref.qkv_rope(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits),
                                       group, bits, hq, hkv, d, d, 1e6, pos)
    q, k, v = sb.qkv_rope(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits),
                          torch.from_numpy(pos).cuda(), hq, hkv, d, d, 1e6, group, bits)
    assert tuple(q.shape) == (bsz, hq, length, d) and tuple(k.shape) == (bsz, hkv, length, d)
    assert_close(to_f32(q), q_ref, what="q")
    assert_close(to_f32(k), k_ref, what="k")
    assert_close(to_f32(v), v_ref, what="v")


def make_kv(rng, bsz, kvh, n, d, capacity=None):
    capacity = capacity or n
    k = rng.standard_normal((bsz, kvh, n, d)).astype(np.float32)
    v = rng.standard_normal((bsz, kvh, n, d)).astype(np.float32)
    kq, ks = quant.quantize_kv_symmetric(k)
    vq, vs = quant.quantize_kv_symmetric(v)
    pad = capacity - n

    def cache(a, fill):
        if pad == 0:
            return a
        widths = [(0, 0)] * a.ndim
        widths[2] = (0, pad)
        return np.pad(a, widths, constant_values=fill)

    return kq, ks, vq, vs, cache(kq, 7), cache(ks, np.float16(3.0)), cache(vq, -5), cache(vs, np.float16(2.0))


@pytest.mark.parametrize(
    "bsz,n,capacity",
    [(1, 512, 512), (8, 4096, 4096), (1, 32768, 32768), (32, 512, 528), (2, 1, 16), (1, 17, 40), (3, 1000, 1024)],
)
def test_int8_sdpa_decode_matches_oracle(sb, bsz, n, capacity):
    """Config 3: 32 q heads, 8 kv heads, head_dim 128, scale 1/sqrt(128)."""
    rng = np.random.default_rng(bsz * 7 + n)
    hq, hkv, d = 32, 8, 128
    q = formats.round_bf16(rng.standard_normal((bsz, hq, 1, d)).astype(np.float32))
    kq, ks, vq, vs, kc, ksc, vc, vsc = make_kv(rng, bsz, hkv, n, d, capacity)
    scale = 1.0 / np.sqrt(d)
    expected = ref.sdpa_int8(q, kq, ks, vq, vs, scale, causal=True)
    out = sb.int8_sdpa_decode(bf16_tensor(q), torch.from_numpy(kc).cuda(), torch.from_numpy(ksc).cuda(),
                              torch.from_numpy(vc).cuda(), torch.from_numpy(vsc).cuda(), n, float(scale))
    assert_close(to_f32(out), expected, what="int8 sdpa")


@pytest.mark.parametrize("g", [1, 2, 8])
def test_int8_sdpa_gqa_ratios(sb, g):
    rng = np.random.default_rng(g)
    hkv, d, n = 4, 128, 300
    q = formats.round_bf16(rng.standard_normal((2, hkv * g, 1, d)).astype(np.float32) * 4)
    kq, ks, vq, vs, *_ = make_kv(rng, 2, hkv, n, d)
    expected = ref.sdpa_int8(q, kq, ks, vq, vs, 0.1, causal=True)
    out = sb.int8_sdpa_decode(bf16_tensor(q), torch.from_numpy(kq).cuda(), torch.from_numpy(ks).cuda(),
                              torch.from_numpy(vq).cuda(), torch.from_numpy(vs).cuda(), n, 0.1)
    assert_close(to_f32(out), expected, what="gqa")


@pytest.mark.parametrize("bsz,n,capacity,g", [(1, 1000, 1008, 4), (4, 4096, 4096, 4), (2, 300, 304, 1),
                                             (1, 33, 48, 2), (3, 2048, 2048, 8), (1, 32768, 32768, 4)])
def test_int8_sdpa_decode_head_dim_256(sb, bsz, n, capacity, g):
    """head_dim 256 (the reference model's attention: 16 q / 4 kv heads x 256,
    ``int8_quantized_sdpa.py:226-230``): K/V rows as two 128-byte boxes."""
    rng = np.random.default_rng(256 + bsz * 7 + n + g)
    hkv, d = 4, 256
    q = formats.round_bf16(rng.standard_normal((bsz, hkv * g, 1, d)).astype(np.float32))
    kq, ks, vq, vs, kc, ksc, vc, vsc = make_kv(rng, bsz, hkv, n, d, capacity)
    scale = 1.0 / np.sqrt(d)
    expected = ref.sdpa_int8(q, kq, ks, vq, vs, scale, causal=True)
    out = sb.int8_sdpa_decode(bf16_tensor(q), torch.from_numpy(kc).cuda(), torch.from_numpy(ksc).cuda(),
                              torch.from_numpy(vc).cuda(), torch.from_numpy(vsc).cuda(), n, float(scale))
    assert_close(to_f32(out), expected, what="int8 sdpa d256")


def test_rms_norm(sb):
    rng = np.random.default_rng(5)
    x = formats.round_bf16(rng.standard_normal((3, 2560)).astype(np.float32))
    w = formats.round_bf16(1 + 0.1 * rng.standard_normal(2560).astype(np.float32))
    y = sb.rms_norm(bf16_tensor(x), bf16_tensor(w), 1e-6)
    assert_close(to_f32(y), ref.rms_norm(x, w, 1e-6), rtol=1e-2, atol=1e-2, what="rms_norm")


def test_cpu_tensor_raises(sb):
    with pytest.raises(ValueError):
        sb.rms_norm(torch.ones(4, 8, dtype=torch.bfloat16), torch.ones(8, dtype=torch.bfloat16), 1e-6)
