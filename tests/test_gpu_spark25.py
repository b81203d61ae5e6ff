"""Pieces of the reference's Spark2_5 block on the GPU against the oracle.

* the GELU-gated FFN (``spark_mlx_llm/ops/ffn.py:98-103``: ``nn.gelu(gate) * up``)
  as the paired gate/up GEMV epilogue (``sb_linear_ex`` activation 1) and as the
  elementwise form for prompt chunks; the SiLU form alongside;
* the attention-output head gate (``ops/attention_output.py:91-95``).
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, ops as ref  # noqa: E402

pytestmark = pytest.mark.gpu


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _f32(t):
    return t.detach().float().cpu().numpy()


def _close(got, want):
    err = np.abs(got - want)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(want)), float((err / (2e-2 + 1e-2 * np.abs(want))).max())


@pytest.mark.parametrize("activation", [0, 1])
@pytest.mark.parametrize("m", [1, 4, 8])
def test_gated_ffn_epilogue_matches_oracle(activation, m):
    _need_cuda()
    from spark_b200 import quantize
    from spark_b200._lib import check, lib, sb_linear_ex_desc

    n, k, grp = 1536, 2560, 64
    gen = torch.Generator(device="cuda").manual_seed(20 + m + activation)
    gw = quantize.quantize_affine_minmax(torch.randn(n, k, generator=gen, device="cuda") * 0.02, grp, 4)
    uw = quantize.quantize_affine_minmax(torch.randn(n, k, generator=gen, device="cuda") * 0.02, grp, 4)
    x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
    norm = (1.0 + 0.1 * torch.randn(k, generator=gen, device="cuda")).bfloat16()
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    d = sb_linear_ex_desc(x=x.data_ptr(), x_dtype=0, M=m, N=n, K=k, weight_format=0, weight=gw[0].data_ptr(),
                          scales=gw[1].data_ptr(), biases=gw[2].data_ptr(), weight2=uw[0].data_ptr(),
                          scales2=uw[1].data_ptr(), biases2=uw[2].data_ptr(), group_size=grp,
                          norm_weight=norm.data_ptr(), norm_eps=1e-6, epilogue=2, y=y.data_ptr(),
                          activation=activation)
    ws = torch.zeros(max(lib().sb_linear_ex_workspace_size(ctypes.byref(d)), 256), dtype=torch.uint8, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().sb_linear_ex(ctypes.byref(d), torch.cuda.current_stream().cuda_stream), "gated ffn")
    torch.cuda.synchronize()
    xn = formats.round_bf16(ref.rms_norm(_f32(x), _f32(norm), 1e-6).astype(np.float32))

    def proj(w):
        p, s, b = w
        return formats.round_bf16(ref.affine_linear(xn, p.cpu().numpy().view(np.uint32), _f32(s), _f32(b), grp,
                                                    4).astype(np.float32))

    g, u = proj(gw), proj(uw)
    want = ref.gelu_glu(g, u) if activation else ref.swiglu(g, u)
    _close(_f32(y), want)


@pytest.mark.parametrize("activation", [0, 1])
def test_gated_activation_elementwise(activation):
    _need_cuda()
    from spark_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(30 + activation)
    g = (torch.randn(3, 1003, generator=gen, device="cuda") * 2).bfloat16()  # ragged tail (not a multiple of 8)
    u = torch.randn(3, 1003, generator=gen, device="cuda").bfloat16()
    out = ops.gated_activation(g, u, activation)
    want = ref.gelu_glu(_f32(g), _f32(u)) if activation else ref.swiglu(_f32(g), _f32(u))
    _close(_f32(out), want)


def test_head_gate_matches_oracle():
    _need_cuda()
    from spark_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(40)
    m, hidden, heads, d = 5, 2560, 16, 128
    x = torch.randn(m, hidden, generator=gen, device="cuda").bfloat16()
    w = (torch.randn(heads, hidden, generator=gen, device="cuda") * 0.02).bfloat16()
    attn = torch.randn(m, heads, d, generator=gen, device="cuda").bfloat16()
    out = ops.head_gate(x, w, attn)
    _close(_f32(out), ref.head_gate(_f32(x), _f32(w), _f32(attn)))


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
