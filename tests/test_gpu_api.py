"""GPU parity of the reference-named entry points (spark_b200.ext / .dispatch)
against the CPU oracle, through the same kernels as the operators."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, ops as ref, quant  # noqa: E402

from _util import assert_close, bf16_bits_tensor, bf16_tensor, to_f32, u32_tensor  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200 import dispatch, ext

    return ext, dispatch


def affine(rng, n, k, group, bits):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    return quant.quantize_affine_minmax(w, group, bits)


def test_w4a16_qmv_and_dispatch_linear(api):
    ext, dispatch = api
    rng = np.random.default_rng(21)
    n, k = 2560, 2048
    packed, s_bits, b_bits = affine(rng, n, k, 32, 4)
    x = formats.round_bf16(rng.standard_normal((1, 1, k)).astype(np.float32))
    expected = ref.affine_linear(x.reshape(1, k), packed, formats.bf16_from_bits(s_bits),
                                 formats.bf16_from_bits(b_bits), 32, 4)
    y = ext.w4a16_qmv(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits))
    assert tuple(y.shape) == (1, 1, n)
    assert_close(to_f32(y).reshape(1, n), expected, what="w4a16_qmv")
    proj = dispatch.QuantizedLinear(u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits), 32, 4)
    y2 = dispatch.dispatch_linear(bf16_tensor(x), proj)
    np.testing.assert_array_equal(to_f32(y2), to_f32(y))


def test_multirow_entry_points(api):
    ext, _ = api
    rng = np.random.default_rng(22)
    n, k = 512, 1024
    packed, s_bits, b_bits = affine(rng, n, k, 32, 4)
    x = formats.round_bf16(rng.standard_normal((5, k)).astype(np.float32))
    expected = ref.affine_linear(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits), 32, 4)
    y = ext.w4a16_multirow(bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits))
    assert_close(to_f32(y), expected, what="w4a16_multirow")
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    y8 = ext.w8a16_multirow(bf16_tensor(x), torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda(),
                            output_dtype=torch.float32)
    assert y8.dtype == torch.float32
    assert_close(to_f32(y8), ref.w8a16_per_channel(x, wq, ws), what="w8a16_multirow")


def test_spark_qkv_rope_scalar_offset_and_dispatch_qkv(api):
    ext, dispatch = api
    rng = np.random.default_rng(23)
    hidden, hq, hkv, d, group = 2560, 32, 8, 128, 64
    packed, s_bits, b_bits = affine(rng, (hq + 2 * hkv) * d, hidden, group, 4)
    x = formats.round_bf16(rng.standard_normal((1, 1, hidden)).astype(np.float32))
    offset = 777
    pos = np.full((1, 1), offset, np.int32)
    q_ref, k_ref, v_ref = ref.qkv_rope(x, packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits),
                                       group, 4, hq, hkv, d, d, 1e6, pos)
    args = (bf16_tensor(x), u32_tensor(packed), bf16_bits_tensor(s_bits), bf16_bits_tensor(b_bits))
    q, k, v = ext.spark_qkv_rope(*args, hq * d, hkv * d, hq, hkv, d, d, 1e6, offset, group_size=group, bits=4)
    assert_close(to_f32(q), q_ref, what="q")
    assert_close(to_f32(k), k_ref, what="k")
    assert_close(to_f32(v), v_ref, what="v")
    proj = dispatch.QuantizedLinear(args[1], args[2], args[3], group, 4)
    q2, k2, v2 = dispatch.dispatch_qkv(args[0], proj, dispatch.RoPE(d, base=1e6), q_size=hq * d, kv_size=hkv * d,
                                       n_heads=hq, n_kv_heads=hkv, head_dim=d, offset=offset)
    for a, b in ((q, q2), (k, k2), (v, v2)):
        np.testing.assert_array_equal(to_f32(a), to_f32(b))


def affine_kv(rng, bsz, kvh, n, dim, group, bits):
    x = rng.standard_normal((bsz * kvh * n, dim)).astype(np.float32)
    packed, s_bits, b_bits = quant.quantize_affine_minmax(x, group, bits)
    shape = (bsz, kvh, n)
    return (packed.reshape(*shape, -1), formats.bf16_from_bits(s_bits).reshape(*shape, -1),
            formats.bf16_from_bits(b_bits).reshape(*shape, -1), s_bits.reshape(*shape, -1),
            b_bits.reshape(*shape, -1))


@pytest.mark.parametrize(
    "bsz,heads,kvh,length,n,dim,group,bits,mask",
    [
        (1, 32, 8, 1, 700, 256, 32, 8, None),      # the reference's fused decode shape (D256, G32, 8-bit)
        (2, 16, 4, 1, 5000, 128, 64, 4, None),     # several token splits
        (1, 8, 8, 3, 40, 128, 32, 8, "causal"),   # multi-token bottom-right causal
        (1, 4, 2, 1, 33, 64, 32, 2, "causal"),    # 2-bit codes
        # single-query decode on the KV-head-per-CTA kernel: the reference model's 16/4 x 256,
        # GQA 8 with group 128, GQA 1 at head_dim 64, a ragged short cache
        (1, 16, 4, 1, 4096, 256, 32, 8, None),
        (2, 8, 1, 1, 1000, 128, 128, 4, None),
        (3, 8, 8, 1, 300, 64, 32, 8, None),
        (1, 16, 4, 1, 37, 256, 32, 4, "causal"),
        # the tensor-core kernel (head_dim 128 / 256) at GQA 1 and 2, ragged tiles
        (1, 8, 8, 1, 333, 256, 64, 8, None),
        (2, 16, 8, 1, 2000, 128, 32, 8, None),
        (1, 32, 4, 1, 3001, 256, 32, 4, None),
    ],
)
def test_int8_quantized_sdpa_affine_tuples(api, bsz, heads, kvh, length, n, dim, group, bits, mask):
    ext, dispatch = api
    rng = np.random.default_rng(bsz + heads + n + bits)
    q = formats.round_bf16(rng.standard_normal((bsz, heads, length, dim)).astype(np.float32))
    kp, ks, kb, ks_bits, kb_bits = affine_kv(rng, bsz, kvh, n, dim, group, bits)
    vp, vs, vb, vs_bits, vb_bits = affine_kv(rng, bsz, kvh, n, dim, group, bits)
    scale = 1.0 / np.sqrt(dim)
    expected = ref.sdpa_affine(q, (kp, ks, kb), (vp, vs, vb), scale, group, bits, causal=mask == "causal")
    keys = (u32_tensor(kp), bf16_bits_tensor(ks_bits), bf16_bits_tensor(kb_bits))
    values = (u32_tensor(vp), bf16_bits_tensor(vs_bits), bf16_bits_tensor(vb_bits))
    out = ext.int8_quantized_sdpa(bf16_tensor(q), keys, values, scale=float(scale), group_size=group, bits=bits,
                                  mask=mask)
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == (bsz, heads, length, dim)
    assert_close(to_f32(out), expected, what="affine-tuple sdpa")

    class Cache:
        pass

    cache = Cache()
    cache.bits, cache.group_size = bits, group
    out2 = dispatch.dispatch_sdpa(bf16_tensor(q), keys, values, cache=cache, scale=float(scale), mask=mask)
    np.testing.assert_array_equal(to_f32(out2), to_f32(out))


def test_dispatch_sdpa_int8_pair(api):
    _, dispatch = api
    rng = np.random.default_rng(31)
    q = formats.round_bf16(rng.standard_normal((1, 32, 1, 128)).astype(np.float32))
    k = rng.standard_normal((1, 8, 300, 128)).astype(np.float32)
    v = rng.standard_normal((1, 8, 300, 128)).astype(np.float32)
    kq, ks = quant.quantize_kv_symmetric(k)
    vq, vs = quant.quantize_kv_symmetric(v)
    expected = ref.sdpa_int8(q, kq, ks, vq, vs, 0.088, causal=True)
    out = dispatch.dispatch_sdpa(bf16_tensor(q), (torch.from_numpy(kq).cuda(), torch.from_numpy(ks).cuda()),
                                 (torch.from_numpy(vq).cuda(), torch.from_numpy(vs).cuda()), cache=None, scale=0.088,
                                 mask=None)
    assert_close(to_f32(out), expected, what="dispatch int8 pair")


def test_w8a8_linear_layer(api):
    ext, _ = api
    rng = np.random.default_rng(41)
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((256, 512)) * 0.02).astype(np.float32),
                                           scale_to_bf16=False)
    x = formats.round_bf16(rng.standard_normal((3, 512)).astype(np.float32))
    y32, _, _ = ref.w8a8_linear(x, wq, ws, None)
    layer = ext.W8A8Linear(torch.from_numpy(wq).cuda(), torch.from_numpy(ws).cuda())
    np.testing.assert_array_equal(to_f32(layer(bf16_tensor(x))), formats.round_bf16(y32))
    assert ext.is_w8a8_available()
