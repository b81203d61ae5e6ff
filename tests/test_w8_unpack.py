"""Load-time affine W8 -> per-channel INT8 unpack of the product
(``spark_b200.dispatch.unpack_affine_w8``, restating
``spark_mlx_llm/ops/linear.py:299-324``) against the reference's own W8
checkpoint rows (``tests/golden/conversion_vectors.npz``, written by the
reference's ``conversion.py``) and the oracle's unpack. CPU only: the unpack
is torch bit arithmetic that runs on whatever device holds the weights.
"""

import os
from types import SimpleNamespace

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, quant  # noqa: E402
from spark_b200 import dispatch  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "conversion_vectors.npz")


def _layer(words, s_bits, b_bits, group):
    def bf16(bits):
        return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16).copy()).view(torch.bfloat16)

    return SimpleNamespace(weight=torch.from_numpy(np.asarray(words, np.uint32).view(np.int32).copy()),
                           scales=bf16(s_bits), biases=bf16(b_bits), group_size=group, bits=8, mode="affine")


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as data:
        return {k: data[k] for k in data.files}


def test_unpack_matches_reference_channel_rows(golden):
    words = golden["rows_chan_weight"]
    k = words.shape[1] * 4
    group = k // golden["rows_chan_scales"].shape[1]
    layer = _layer(words, golden["rows_chan_scales"], golden["rows_chan_biases"], group)
    w_int8, scale = dispatch.unpack_affine_w8(layer, "o_proj")
    # the reference converter's input codes come back bit for bit
    np.testing.assert_array_equal(w_int8.numpy(), golden["chan_codes"])
    np.testing.assert_array_equal(scale.numpy(), formats.bf16_from_bits(golden["chan_scale_bf16_bits"])[:, 0])
    # and the oracle's restatement agrees
    ow, os_ = quant.unpack_affine_w8(words, formats.bf16_from_bits(golden["rows_chan_scales"]),
                                     formats.bf16_from_bits(golden["rows_chan_biases"]))
    np.testing.assert_array_equal(w_int8.numpy(), ow)
    np.testing.assert_array_equal(scale.numpy(), os_)


def test_unpack_rejects_groupwise_and_allows_fallback(golden):
    # the reference's W8 rows with one group's scale and bias changed: group-wise, not per-channel
    words = golden["rows_w8_weight"]
    group = words.shape[1] * 4 // golden["rows_w8_scales"].shape[1]
    s = formats.bf16_from_bits(golden["rows_w8_scales"]).copy()
    s[0, 1] *= 2
    layer = _layer(words, formats.bf16_bits(s), formats.bf16_bits(-128 * s), group)
    assert dispatch.unpack_affine_w8(_layer(words, golden["rows_w8_scales"], golden["rows_w8_biases"], group),
                                     "qkv_proj") is not None
    with pytest.raises(ValueError, match="groupwise/asymmetric"):
        dispatch.unpack_affine_w8(layer, "qkv_proj")
    assert dispatch.unpack_affine_w8(layer, "qkv_proj", allow_fallback=True) is None
    bad = SimpleNamespace(weight=layer.weight.view(torch.int8), scales=layer.scales, biases=layer.biases,
                          group_size=group, bits=8, mode="affine")
    with pytest.raises(ValueError, match="UINT32-packed affine W8"):
        dispatch.unpack_affine_w8(bad, "qkv_proj")


def test_prepared_w8_caches_by_source_identity(golden):
    words = golden["rows_chan_weight"]
    group = words.shape[1] * 4 // golden["rows_chan_scales"].shape[1]
    layer = _layer(words, golden["rows_chan_scales"], golden["rows_chan_biases"], group)
    prep = dispatch.PreparedW8()
    first = prep(layer)
    assert prep(layer) is first
    layer.weight = layer.weight.clone()  # new source tensor: unpacked again
    second = prep(layer)
    assert second is not first
    assert torch.equal(second[0], first[0])
    qlayer = dispatch.QuantizedLinear(layer.weight, layer.scales, layer.biases, group_size=layer.group_size, bits=8)
    module = dispatch.W8A16PerChannelLinear.from_affine(qlayer)
    assert module.weight.dtype == torch.int8 and module.scales.dtype == torch.float32
    assert module.fallback is qlayer


def _w8_layer(n, k, group=64, dtype=torch.bfloat16):
    words = torch.zeros(n, k // 4, dtype=torch.int32)
    scales = torch.full((n, k // group), 0.01, dtype=dtype)
    return dispatch.QuantizedLinear(words, scales, -128 * scales, group_size=group, bits=8)


def test_w8_multirow_projection_checks_its_inputs():
    """``W8MultirowProjection`` (``ops/linear.py:479-528``) accepts an affine
    8-bit layer with its per-channel INT8 form at the reference's measured
    out_proj geometry, and raises the reference's error for anything else."""
    n, k = 2560, 4096
    layer = _w8_layer(n, k)
    w, s = dispatch.unpack_affine_w8(layer, "out_proj")
    proj = dispatch.W8MultirowProjection(layer, w, s)
    assert proj.fallback is layer and proj.weight.dtype == torch.int8
    bad = [
        (SimpleNamespace(**vars(layer)), w, s),                 # not a QuantizedLinear
        (_w8_layer(n, k, dtype=torch.float16), w, s),           # scales dtype
        (layer, w.to(torch.int16), s),                          # weight dtype
        (layer, w, s.double()),                                 # scales dtype
        (layer, w, s[:-1]),                                     # scales shape
        (_w8_layer(1024, k), *dispatch.unpack_affine_w8(_w8_layer(1024, k), "p")),  # unmeasured geometry
    ]
    four = dispatch.QuantizedLinear(torch.zeros(n, k // 8, dtype=torch.int32), layer.scales, layer.biases,
                                    group_size=64, bits=4)
    bad.append((four, w, s))                                    # not 8-bit
    for args in bad:
        with pytest.raises(ValueError, match="measured out/head"):
            dispatch.W8MultirowProjection(*args)


def test_w8_multirow_projection_routes_only_eight_gpu_rows():
    layer = _w8_layer(2560, 4096)
    proj = dispatch.W8MultirowProjection(layer, *dispatch.unpack_affine_w8(layer, "out_proj"))
    calls = []

    class Recorder(torch.nn.Module):
        def forward(self, x):
            calls.append(tuple(x.shape))
            return x

    proj.fallback = Recorder()
    assert not proj.takes_multirow(torch.zeros(8, 4096, dtype=torch.bfloat16))   # CPU: affine layer
    for shape in ((1, 4096), (2, 4, 4096), (7, 4096)):
        x = torch.zeros(shape, dtype=torch.bfloat16)
        assert not proj.takes_multirow(x)
        proj(x)
    assert calls == [(1, 4096), (2, 4, 4096), (7, 4096)]
    meta = torch.empty(2, 4, 4096, dtype=torch.bfloat16, device="meta")
    assert not proj.takes_multirow(meta)  # 8 rows, but not on a GPU


def test_w8a8_projection_needs_the_gpu_kernels():
    """``W8A8Projection`` (``ops/linear.py:531-562``) refuses to build without
    the W8A8 kernels (here: no GPU), as the reference does without its extension."""
    layer = _w8_layer(256, 512)
    w, s = dispatch.unpack_affine_w8(layer, "o_proj")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: covered by the GPU tests")
    with pytest.raises(RuntimeError, match="w8a8"):
        dispatch.W8A8Projection(layer, w, s)


def test_w8a16_per_channel_linear_checks_and_routes():
    """``W8A16PerChannelLinear`` (``ops/linear.py:413-476``): the reference's
    checks and errors; only one BF16/FP16 row on a GPU leaves the affine layer."""
    layer = _w8_layer(64, 256)
    w, s = dispatch.unpack_affine_w8(layer, "o_proj")
    module = dispatch.W8A16PerChannelLinear(layer, w, s[:, None])
    assert tuple(module.scales.shape) == (64,)
    with pytest.raises(ValueError, match="bias-free affine W8"):
        dispatch.W8A16PerChannelLinear(SimpleNamespace(**vars(layer)), w, s)
    with pytest.raises(ValueError, match="bias-free affine W8"):
        dispatch.W8A16PerChannelLinear(dispatch.QuantizedLinear(layer.weight, layer.scales, layer.biases,
                                                                group_size=64, bits=4), w, s)
    for bad_w, bad_s in ((w[:, :128], s), (w.to(torch.int16), s), (w, s.double()), (w, s[:-1])):
        with pytest.raises(ValueError, match="matching signed INT8"):
            dispatch.W8A16PerChannelLinear(layer, bad_w, bad_s)
    assert dispatch.W8A16PerChannelLinear.supports_rows(1, torch.bfloat16)
    assert not dispatch.W8A16PerChannelLinear.supports_rows(2, torch.bfloat16)
    assert not dispatch.W8A16PerChannelLinear.supports_rows(1, torch.float32)
    assert not dispatch.W8A16PerChannelLinear.supports_rows(1, torch.bfloat16, "cpu")
    calls = []

    class Recorder(torch.nn.Module):
        def forward(self, x):
            calls.append(tuple(x.shape))
            return x

    module.fallback = Recorder()
    module(torch.zeros(1, 256, dtype=torch.bfloat16))  # one row, but on the CPU
    module(torch.zeros(4, 256, dtype=torch.bfloat16))
    assert calls == [(1, 256), (4, 256)]


def _model(out_layers, lm_head=None, backend="w8a16"):
    layers = [SimpleNamespace(self_attn=torch.nn.Module()) for _ in out_layers]
    for layer, out in zip(layers, out_layers):
        layer.self_attn.out_proj = out
    model = SimpleNamespace(layers=layers, lm_head=lm_head,
                            args=SimpleNamespace(tie_word_embeddings=lm_head is None, w8_qmv_backend=backend))
    return model


def test_quantized_projections_lifecycle():
    """``QuantizedProjections`` (``ops/linear.py:565-731``): w8a16 wraps every
    per-channel W8 out_proj and the untied head, skips group-wise W8 and W4,
    scale_paths names the fp32 scales, unwrap restores the affine layers;
    auto/native and an unknown backend leave the model alone or raise."""
    per_channel = _w8_layer(64, 256)
    grouped = _w8_layer(64, 256)
    grouped.scales = grouped.scales.clone()
    grouped.scales[0, 1] *= 2  # group-wise scales: not per-channel
    grouped.biases = -128 * grouped.scales
    four = dispatch.QuantizedLinear(torch.zeros(64, 32, dtype=torch.int32), grouped.scales, grouped.biases,
                                    group_size=64, bits=4)
    head = _w8_layer(128, 256)
    model = _model([per_channel, grouped, four], lm_head=head)
    for backend in ("auto", "native"):
        dispatch.QuantizedProjections.configure(model, backend)
        assert model.layers[0].self_attn.out_proj is per_channel
    with pytest.raises(ValueError):
        dispatch.QuantizedProjections.configure(model, "fast")
    dispatch.QuantizedProjections.prepare(model)  # args.w8_qmv_backend = "w8a16"
    outs = [layer.self_attn.out_proj for layer in model.layers]
    assert type(outs[0]) is dispatch.W8A16PerChannelLinear and outs[0].fallback is per_channel
    assert outs[1] is grouped and outs[2] is four
    assert type(model.lm_head) is dispatch.W8A16PerChannelLinear
    assert dispatch.QuantizedProjections.scale_paths(model) == {"model.layers.0.self_attn.out_proj.scales",
                                                                 "lm_head.scales"}
    dispatch.QuantizedProjections.unwrap(model)
    assert model.layers[0].self_attn.out_proj is per_channel and model.lm_head is head
    assert dispatch.QuantizedProjections.scale_paths(model) == set()


def test_quantized_projections_multirow_and_w8a8_selection():
    """multirow wraps only the measured out_proj geometry (2560 x 4096 here);
    w8a8 without its kernels (no GPU) changes nothing."""
    measured, other = _w8_layer(2560, 4096), _w8_layer(64, 256)
    model = _model([measured, other])
    if not torch.cuda.is_available():
        dispatch.QuantizedProjections.configure(model, "w8a8")
        assert model.layers[0].self_attn.out_proj is measured
    dispatch.QuantizedProjections.configure(model, "multirow")
    assert type(model.layers[0].self_attn.out_proj) is dispatch.W8MultirowProjection
    assert model.layers[1].self_attn.out_proj is other
    assert dispatch.QuantizedProjections.scale_paths(model) == {"model.layers.0.self_attn.out_proj.scales"}
