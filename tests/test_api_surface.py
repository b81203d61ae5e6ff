"""The reference-named entry points: signatures, argument validation, errors.

``spark_b200.ext`` mirrors ``spark_mlx_ext`` (_ext.pyi:1-44, w4a16_qmv.py:37-44,
w4a16_multirow.py:238-253, w8a16_multirow.py:43-54, int8_quantized_sdpa.py:
156-166, linear.py:9-55) and ``spark_b200.dispatch`` mirrors
``spark_mlx_llm.ops`` (linear.py:84-191, qkv.py:18-30, sdpa.py:39-49). These
run without a GPU: they check the Python surface and the validation that
happens before any kernel launch.
"""

import inspect

import pytest

torch = pytest.importorskip("torch")

from spark_b200 import dispatch, ext  # noqa: E402


def params(fn):
    sig = inspect.signature(fn)
    return [(p.name, p.kind.name, p.default) for p in sig.parameters.values()]


P, K = "POSITIONAL_OR_KEYWORD", "KEYWORD_ONLY"
E = inspect.Parameter.empty


@pytest.mark.parametrize(
    "fn,expected",
    [
        (ext.w8a16_per_channel, [("x", P, E), ("weight", P, E), ("scales", P, E), ("stream", K, None)]),
        (ext.int8_matmul_int32, [("x", P, E), ("weight", P, E), ("stream", K, None)]),
        (ext.w8a8_linear, [("x", P, E), ("weight", P, E), ("scales", P, E), ("bias", P, None), ("stream", K, None)]),
        (ext.spark_qkv_rope, [("x", P, E), ("weight", P, E), ("scales", P, E), ("biases", P, E), ("q_size", P, E),
                              ("kv_size", P, E), ("num_heads", P, E), ("num_key_value_heads", P, E),
                              ("head_dim", P, E), ("rope_dims", P, E), ("rope_base", P, E), ("offset", P, E),
                              ("group_size", P, 128), ("bits", P, 4), ("stream", K, None)]),
        (ext.w4a16_qmv, [("x", P, E), ("weight", P, E), ("scales", P, E), ("biases", P, E), ("stream", K, None)]),
        (ext.int8_quantized_sdpa, [("queries", P, E), ("keys", P, E), ("values", P, E), ("scale", K, E),
                                   ("group_size", K, 32), ("bits", K, 8), ("mask", K, None),
                                   ("single_pass_max_length", K, 1023)]),
        (dispatch.dispatch_linear, [("x", P, E), ("projection", P, E), ("config", K, None)]),
        (dispatch.dispatch_qkv, [("x", P, E), ("projection", P, E), ("rope", P, E), ("q_size", K, E),
                                 ("kv_size", K, E), ("n_heads", K, E), ("n_kv_heads", K, E), ("head_dim", K, E),
                                 ("offset", K, E), ("config", K, None)]),
        (dispatch.dispatch_sdpa, [("queries", P, E), ("keys", P, E), ("values", P, E), ("cache", K, E),
                                  ("scale", K, E), ("mask", K, E), ("config", K, None), ("is_sliding", K, False)]),
        (dispatch.dispatch_attention_output, [("x", P, E), ("output", P, E), ("gate_projection", P, E),
                                              ("output_projection", P, E)]),
        (dispatch.dispatch_ffn, [("x", P, E), ("attention_output", P, E), ("norm", P, E), ("mlp", P, E),
                                 ("mlp_type", K, E)]),
        (dispatch.W8A16PerChannelLinear.__init__, [("self", P, E), ("fallback", P, E), ("weight", P, E),
                                                   ("scales", P, E)]),
        (dispatch.W8MultirowProjection.__init__, [("self", P, E), ("fallback", P, E), ("weight", P, E),
                                                  ("scales", P, E)]),
        (dispatch.W8A8Projection.__init__, [("self", P, E), ("fallback", P, E), ("weight", P, E),
                                            ("scales", P, E)]),
        (dispatch.AffineParameters.resolve, [("layer", P, E), ("shape", P, E), ("dtype", P, E), ("config", P, E)]),
    ],
)
def test_reference_signatures(fn, expected):
    assert params(fn) == expected


def test_multirow_signatures_keep_reference_keywords():
    names = [p[0] for p in params(ext.w4a16_multirow)]
    assert names == ["x", "weight", "scales", "biases", "algorithm", "k_lanes", "splits", "simdgroups", "layout",
                     "static_layout", "multiply_mode", "static_slice", "contiguous_k", "stream"]
    names = [p[0] for p in params(ext.w8a16_multirow)]
    assert names == ["x", "weight", "scales", "output_dtype", "variant", "tile_rows", "k_lanes", "simdgroups",
                     "stream"]


def test_type_and_value_errors_before_launch():
    with pytest.raises(TypeError):
        ext.w8a16_per_channel([1.0], torch.zeros(4, 64, dtype=torch.int8), torch.ones(4))
    x = torch.zeros(1, 512, dtype=torch.bfloat16)
    w = torch.zeros(8, 64, dtype=torch.int32)
    s = torch.zeros(8, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="BF16"):
        ext.w4a16_qmv(x.float(), w, s, s)
    with pytest.raises(ValueError, match="divisible by 512"):
        ext.w4a16_qmv(torch.zeros(1, 256, dtype=torch.bfloat16), w, s, s)
    with pytest.raises(ValueError, match="exactly one activation row"):
        ext.w4a16_qmv(torch.zeros(2, 512, dtype=torch.bfloat16), w, s, s)
    with pytest.raises(ValueError, match="requires CUDA GPU execution"):
        ext.w4a16_qmv(x, w, s, s)  # valid descriptor, CPU tensors
    with pytest.raises(ValueError, match="single_pass_max_length"):
        ext.int8_quantized_sdpa(torch.zeros(1, 1, 1, 64), (), (), scale=1.0, single_pass_max_length=-1)
    with pytest.raises(ValueError, match="affine"):
        ext.int8_quantized_sdpa(torch.zeros(1, 1, 1, 64), (1, 2), (1, 2), scale=1.0)


def test_w8a8_linear_layer_validation():
    with pytest.raises(ValueError, match="INT8 matrix"):
        ext.W8A8Linear(torch.zeros(4, 64), torch.ones(4))
    with pytest.raises(ValueError, match="multiple of 32"):
        ext.W8A8Linear(torch.zeros(4, 40, dtype=torch.int8), torch.ones(4))
    with pytest.raises(ValueError, match="FP32"):
        ext.W8A8Linear(torch.zeros(4, 64, dtype=torch.int8), torch.ones(4, dtype=torch.float16))
    layer = ext.W8A8Linear(torch.zeros(4, 64, dtype=torch.int8), torch.ones(4, 1))
    assert (layer.input_dims, layer.output_dims) == (64, 4)


def test_configs_validate_choices():
    assert dispatch.LinearConfig().w4_qmv_backend == "native"
    with pytest.raises(ValueError):
        dispatch.LinearConfig(w4_qmv_backend="bogus")
    with pytest.raises(ValueError):
        dispatch.SDPAConfig(fused_quantized_sdpa="yes")
    proj = dispatch.QuantizedLinear(torch.zeros(8, 64, dtype=torch.int32), torch.zeros(8, 8), torch.zeros(8, 8), 64,
                                    4)
    assert dispatch.AffineParameters.accepts(proj)
    assert not dispatch.AffineParameters.accepts(torch.nn.Linear(4, 4))


def test_is_w8a8_available_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert ext.is_w8a8_available() is False


def test_operator_config_helpers():
    """``from_dict`` / ``choices`` / ``validate_values`` of the reference's
    ``OperatorConfig`` (``ops/base.py:14-53``) on the dispatch configs."""
    cfg = dispatch.LinearConfig.from_dict({"w8_qmv_backend": "multirow", "hidden_size": 2560})
    assert cfg.w8_qmv_backend == "multirow" and cfg.w4_qmv_backend == "native"
    assert dispatch.LinearConfig.choices("w4_qmv_backend") == ("native", "splitk", "multirow", "multirow_packed")
    dispatch.LinearConfig.validate_values({"w8_qmv_backend": "w8a8"})  # a partial mapping is fine
    with pytest.raises(ValueError, match="renamed to w8_qmv_backend"):
        dispatch.LinearConfig.validate_values({"qmv_backend": "w8a16"})
    with pytest.raises(ValueError, match="must be a boolean"):
        dispatch.SDPAConfig(tuned_bf16_sdpa=1)
    sd = dispatch.SDPAConfig.from_dict({"fused_quantized_sdpa_prefill": True, "other": 3})
    assert sd.fused_quantized_sdpa_prefill and sd.fused_quantized_sdpa
