"""The block-level dispatch entry points of the reference's ops package -
``dispatch_attention_output`` (``ops/attention_output.py:16-101``) and
``dispatch_ffn`` (``ops/ffn.py:17-118``). CPU: inputs off the GPU or custom
modules take the module route, which must compute the reference's formula;
the fused GPU routes are checked in ``tests/test_gpu_spark25.py``."""

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
