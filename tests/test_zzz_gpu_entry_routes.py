"""GPU tests of the reference-facing entry points' routing, run after the rest
of the suite: fp16 inputs of the affine-tuple decode attention, the W8
projection adapters of ``spark_b200.dispatch`` (``ops/linear.py:413-562``),
the fused routes of ``dispatch_attention_output`` / ``dispatch_ffn``
(``ops/attention_output.py:16-101``, ``ops/ffn.py:17-118``) and the BF16 K/V
route of ``dispatch_sdpa``, each against the oracle or the entry point it
routes to."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, ops as ref, quant  # noqa: E402

from _util import assert_close, bf16_tensor, to_f32, u32_tensor  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200 import dispatch, ext

    return ext, dispatch


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _f32(t):
    return t.detach().float().cpu().numpy()


def _close(got, want):
    err = np.abs(got - want)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(want)), float((err / (2e-2 + 1e-2 * np.abs(want))).max())


def affine_kv(rng, bsz, kvh, n, dim, group, bits):
    x = rng.standard_normal((bsz * kvh * n, dim)).astype(np.float32)
    packed, s_bits, b_bits = quant.quantize_affine_minmax(x, group, bits)
    shape = (bsz, kvh, n)
    return (packed.reshape(*shape, -1), formats.bf16_from_bits(s_bits).reshape(*shape, -1),
            formats.bf16_from_bits(b_bits).reshape(*shape, -1), s_bits.reshape(*shape, -1),
            b_bits.reshape(*shape, -1))


@pytest.mark.parametrize("dim,bits,heads,kvh", [(256, 8, 16, 4), (128, 4, 8, 1), (64, 8, 4, 2)])
def test_int8_quantized_sdpa_affine_tuples_fp16(api, dim, bits, heads, kvh):
    """fp16 queries and fp16 scales / biases (the same values as the bf16 case:
    bf16 metadata converts to fp16 exactly) on the single-query decode kernels."""
    ext, _ = api
    rng = np.random.default_rng(dim + bits)
    n, group = 1500, 32
    q = formats.round_bf16(rng.standard_normal((1, heads, 1, dim)).astype(np.float32))
    kp, ks, kb, _, _ = affine_kv(rng, 1, kvh, n, dim, group, bits)
    vp, vs, vb, _, _ = affine_kv(rng, 1, kvh, n, dim, group, bits)
    scale = 1.0 / np.sqrt(dim)
    expected = ref.sdpa_affine(q, (kp, ks, kb), (vp, vs, vb), scale, group, bits)

    def f16(a):
        return torch.from_numpy(np.asarray(a, np.float32)).to(torch.float16).cuda()

    keys = (u32_tensor(kp), f16(ks), f16(kb))
    values = (u32_tensor(vp), f16(vs), f16(vb))
    out = ext.int8_quantized_sdpa(f16(q), keys, values, scale=float(scale), group_size=group, bits=bits)
    assert out.dtype == torch.float16
    assert_close(to_f32(out), expected, what="affine-tuple sdpa fp16")


def _w8_affine_layer(dispatch, rng, n, k, group):
    """An affine 8-bit layer in the reference's W8 checkpoint form (symmetric
    per-channel codes stored as code + 128 with bias = -128 * scale)."""
    wq, ws = quant.quantize_w8_per_channel((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    s_bf16 = formats.round_bf16(np.asarray(ws, np.float32))
    words = (np.asarray(wq, np.int16) + 128).astype(np.uint8).reshape(n, k // 4, 4)
    words = words.astype(np.uint32) @ np.array([1, 1 << 8, 1 << 16, 1 << 24], np.uint32)
    scales = np.repeat(s_bf16[:, None], k // group, axis=1)
    return dispatch.QuantizedLinear(u32_tensor(words), bf16_tensor(scales), bf16_tensor(-128 * scales),
                                    group_size=group, bits=8)


def test_w8a16_per_channel_linear_routes(api):
    """``dispatch.W8A16PerChannelLinear``: one BF16 row is ``ext.w8a16_per_channel``
    (bit-equal), several rows the affine layer's."""
    ext, dispatch = api
    rng = np.random.default_rng(53)
    layer = _w8_affine_layer(dispatch, rng, 512, 1024, 64)
    module = dispatch.W8A16PerChannelLinear.from_affine(layer, "o_proj")
    x = bf16_tensor(formats.round_bf16(rng.standard_normal((4, 1024)).astype(np.float32)))
    x1 = x[:1].contiguous()
    np.testing.assert_array_equal(to_f32(module(x1)), to_f32(ext.w8a16_per_channel(x1, module.weight,
                                                                                 module.scales)))
    np.testing.assert_array_equal(to_f32(module(x)), to_f32(layer(x)))


def test_w8_multirow_projection_routes(api):
    """``dispatch.W8MultirowProjection`` at the reference's out_proj geometry:
    8 BF16 rows give exactly ``ext.w8a16_multirow``'s result, one row the
    affine layer's."""
    ext, dispatch = api
    n, k = 2560, 4096
    rng = np.random.default_rng(51)
    layer = _w8_affine_layer(dispatch, rng, n, k, 64)
    proj = dispatch.W8MultirowProjection(layer, *dispatch.unpack_affine_w8(layer, "out_proj"))
    x8 = bf16_tensor(formats.round_bf16(rng.standard_normal((8, k)).astype(np.float32)))
    direct = ext.w8a16_multirow(x8, proj.weight, proj.scales)
    np.testing.assert_array_equal(to_f32(proj(x8)), to_f32(direct))
    x1 = x8[:1].contiguous()
    np.testing.assert_array_equal(to_f32(proj(x1)), to_f32(layer(x1)))


def test_w8a8_projection_routes(api):
    """``dispatch.W8A8Projection`` on the GPU is ``ext.W8A8Linear`` (bit-equal)."""
    ext, dispatch = api
    rng = np.random.default_rng(52)
    n, k = 256, 512
    layer = _w8_affine_layer(dispatch, rng, n, k, 64)
    weight, scales = dispatch.unpack_affine_w8(layer, "o_proj")
    proj = dispatch.W8A8Projection(layer, weight, scales)
    x = bf16_tensor(formats.round_bf16(rng.standard_normal((3, k)).astype(np.float32)))
    np.testing.assert_array_equal(to_f32(proj(x)), to_f32(ext.W8A8Linear(weight, scales)(x)))


def _qlinear(gen, n, k, group=32, bits=4):
    from spark_b200 import dispatch, quantize

    w, s, b = quantize.quantize_affine_minmax(torch.randn(n, k, generator=gen, device="cuda") * 0.05, group, bits)
    layer = dispatch.QuantizedLinear(w, s, b, group_size=group, bits=bits)
    host = (w.cpu().numpy().view(np.uint32), _f32(s), _f32(b), group, bits)
    return layer, host


def test_dispatch_attention_output_fused_route():
    """``dispatch.dispatch_attention_output`` with a bias-free BF16 gate Linear and
    an affine out_proj: ``sb_head_gate`` then the affine kernel, against the
    oracle's head gate and affine linear."""
    _need_cuda()
    from spark_b200 import dispatch

    gen = torch.Generator(device="cuda").manual_seed(11)
    b, l, hid, heads, d = 1, 3, 512, 4, 256
    x = torch.randn(b, l, hid, generator=gen, device="cuda").bfloat16()
    output = torch.randn(b, heads, l, d, generator=gen, device="cuda").bfloat16()
    gate = torch.nn.Linear(hid, heads, bias=False, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        gate.weight.copy_(torch.randn(heads, hid, generator=gen, device="cuda") * 0.05)
    out_proj, host = _qlinear(gen, hid, heads * d)
    got = _f32(dispatch.dispatch_attention_output(x, output, gate, out_proj))
    attn = _f32(output).transpose(0, 2, 1, 3).reshape(b * l, heads, d)
    gated = formats.round_bf16(ref.head_gate(_f32(x).reshape(b * l, hid), _f32(gate.weight), attn).astype(np.float32))
    want = ref.affine_linear(gated.reshape(b * l, heads * d), *host).reshape(b, l, hid)
    _close(got, want)


def test_dispatch_ffn_fused_route():
    """``dispatch.dispatch_ffn`` with an RMSNorm and affine gate/up/down: the
    residual, ``sb_rms_norm``, the affine kernels and the GELU gate, against the
    oracle step by step (bf16 at each of the reference's rounding points)."""
    _need_cuda()
    from spark_b200 import dispatch

    class MLP(torch.nn.Module):
        def __init__(self, gate_proj, up_proj, down_proj):
            super().__init__()
            self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    gen = torch.Generator(device="cuda").manual_seed(12)
    hid, inter = 512, 1024
    x = torch.randn(1, 3, hid, generator=gen, device="cuda").bfloat16()
    attn = torch.randn(1, 3, hid, generator=gen, device="cuda").bfloat16()
    norm = torch.nn.RMSNorm(hid, eps=1e-6, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(hid, generator=gen, device="cuda"))
    (gp, gh), (up, uh), (dp, dh) = (_qlinear(gen, inter, hid), _qlinear(gen, inter, hid), _qlinear(gen, hid, inter))
    got = _f32(dispatch.dispatch_ffn(x, attn, norm, MLP(gp, up, dp), mlp_type=MLP))

    def r(v):
        return formats.round_bf16(np.asarray(v, np.float32)).astype(np.float64)

    h = r(_f32(x) + _f32(attn))
    n = r(ref.rms_norm(h, _f32(norm.weight), 1e-6))
    a = r(ref.gelu_glu(r(ref.affine_linear(n, *gh)), r(ref.affine_linear(n, *uh))))
    want = r(h + r(ref.affine_linear(a, *dh)))
    _close(got, want)


def test_dispatch_sdpa_bf16_verification_route():
    """``dispatch_sdpa`` with BF16 K/V tensors and a boolean window mask - the
    reference's verification shape (16/4 heads x 256, 8 queries over 519 keys,
    scale 1/16) - against the float64 masked attention."""
    _need_cuda()
    from spark_b200 import dispatch

    gen = torch.Generator().manual_seed(21)
    q = torch.randn(1, 16, 8, 256, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, 4, 519, 256, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, 4, 519, 256, generator=gen).to(torch.bfloat16)
    pos = np.arange(519 - 8, 519)[:, None]
    keys = np.arange(519)[None, :]
    mask = (keys <= pos) & (keys > pos - 128)
    out = dispatch.dispatch_sdpa(q.cuda(), k.cuda(), v.cuda(), cache=None, scale=0.0625,
                                 mask=torch.from_numpy(mask).cuda(), is_sliding=True)
    ref = ref.sdpa_masked(_f32(q), _f32(k), _f32(v), 0.0625, mask=mask)
    np.testing.assert_allclose(_f32(out), ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())
