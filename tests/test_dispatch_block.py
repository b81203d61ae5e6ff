"""The block-level dispatch entry points of the reference's ops package -
``dispatch_attention_output`` (``ops/attention_output.py:16-101``) and
``dispatch_ffn`` (``ops/ffn.py:17-118``). CPU: inputs off the GPU or custom
modules take the module route, which must compute the reference's formula;
the fused GPU routes are checked in ``tests/test_zzz_gpu_entry_routes.py``."""

import pytest

torch = pytest.importorskip("torch")

from spark_b200 import dispatch  # noqa: E402


def test_attention_output_module_route():
    g = torch.Generator().manual_seed(0)
    b, l, hid, heads, d = 2, 3, 64, 4, 16
    x = torch.randn(b, l, hid, generator=g)
    output = torch.randn(b, heads, l, d, generator=g)
    gate = torch.nn.Linear(hid, heads, bias=False)
    proj = torch.nn.Linear(heads * d, hid, bias=False)
    got = dispatch.dispatch_attention_output(x, output, gate, proj)
    want = proj((output.transpose(1, 2) * torch.sigmoid(gate(x))[..., None]).reshape(b, l, heads * d))
    torch.testing.assert_close(got, want)


def test_ffn_module_route():
    class MLP(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = torch.nn.Linear(32, 64, bias=False)
            self.up_proj = torch.nn.Linear(32, 64, bias=False)
            self.down_proj = torch.nn.Linear(64, 32, bias=False)

        def forward(self, x):
            return self.down_proj(torch.nn.functional.gelu(self.gate_proj(x)) * self.up_proj(x))

    g = torch.Generator().manual_seed(1)
    x, attn = torch.randn(1, 5, 32, generator=g), torch.randn(1, 5, 32, generator=g)
    norm, mlp = torch.nn.RMSNorm(32, eps=1e-6), MLP()
    got = dispatch.dispatch_ffn(x, attn, norm, mlp, mlp_type=MLP)
    h = x + attn
    torch.testing.assert_close(got, h + mlp(norm(h)))


def test_dispatch_sdpa_bf16_route_checks():
    """BF16 K/V tensors route to the multi-query kernel only in its format;
    everything else raises before any kernel call (here on the CPU)."""
    q = torch.zeros(1, 16, 8, 256, dtype=torch.bfloat16)
    k = torch.zeros(1, 4, 519, 256, dtype=torch.bfloat16)
    for bad_q, bad_k in ((q.float(), k.float()), (q[..., :64], k[..., :64]), (q[:, :12], k)):
        with pytest.raises(ValueError, match="BF16 K/V attention"):
            dispatch.dispatch_sdpa(bad_q, bad_k, bad_k, cache=None, scale=0.0625, mask=None)
    with pytest.raises(ValueError, match="mask must be"):
        dispatch.dispatch_sdpa(q, k, k, cache=None, scale=0.0625, mask="sliding")
    with pytest.raises(ValueError, match="serves"):
        dispatch.dispatch_sdpa(q, [k], [k], cache=None, scale=0.0625, mask=None)


def test_affine_backend_selection(monkeypatch):
    """``AffineParameters.resolve`` / ``select`` (``ops/linear.py:116-147``): the
    W4 backends are chosen under the reference's conditions (W4/G32 BF16 on the
    GPU; one row for split-K, eight for multirow) and every other input takes
    the native route."""
    from spark_b200.dispatch import AffineParameters, LinearConfig, QuantizedLinear

    n, k = 256, 1024
    layer = QuantizedLinear(torch.zeros(n, k // 8, dtype=torch.int32), torch.ones(n, k // 32, dtype=torch.bfloat16),
                            torch.zeros(n, k // 32, dtype=torch.bfloat16), group_size=32, bits=4)
    params = AffineParameters.from_module(layer)
    bf16 = torch.bfloat16
    # on the CPU every backend resolves to the native route
    for backend in ("native", "splitk", "multirow", "multirow_packed"):
        fn, _ = AffineParameters.resolve(layer, (8, k), bf16, LinearConfig(w4_qmv_backend=backend))
        assert fn == AffineParameters.native
    monkeypatch.setattr("spark_b200.dispatch._on_gpu", lambda t: True)
    cfg = LinearConfig
    assert params.select((1, 1, k), bf16, cfg(w4_qmv_backend="splitk")) == AffineParameters.splitk
    assert params.select((2, k), bf16, cfg(w4_qmv_backend="splitk")) == AffineParameters.native
    assert params.select((1, 8, k), bf16, cfg(w4_qmv_backend="multirow")) == AffineParameters.multirow
    assert params.select((4, k), bf16, cfg(w4_qmv_backend="multirow")) == AffineParameters.native
    assert params.select((8, k), torch.float16, cfg(w4_qmv_backend="multirow")) == AffineParameters.native
    fn, _ = AffineParameters.resolve(layer, (8, k), bf16, cfg(w4_qmv_backend="multirow_packed"))
    assert fn == AffineParameters.multirow_packed
    g64 = QuantizedLinear(layer.weight, torch.ones(n, k // 64, dtype=bf16), torch.zeros(n, k // 64, dtype=bf16),
                          group_size=64, bits=4)
    assert AffineParameters.from_module(g64).select((8, k), bf16, cfg(w4_qmv_backend="multirow")) == \
        AffineParameters.native
