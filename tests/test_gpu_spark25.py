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
