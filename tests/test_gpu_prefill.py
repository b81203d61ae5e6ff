"""INT8-KV prefill attention and the chunked prompt path (GPU).

* ``sb_int8_sdpa_prefill`` against the float64 oracle (``oracle/ops.py``
  ``sdpa_int8``, the staged recipe of int8_quantized_sdpa.py:122-153 with the
  bottom-right causal mask) for GQA 1/2/4/8, causal and full, both layouts,
  ragged query counts and lengths; q_len = 1 against the decode kernel.
* The decoder's chunked prompt (tensor-core linears, RoPE + INT8 cache
  append, prefill attention) against its single-token prompt and against the
  NumPy decoder oracle: cache codes, the final residual stream and the first
  greedy token.
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import ops as oracle_ops  # noqa: E402
from oracle.model import OracleDecoder  # noqa: E402

from test_gpu_decoder import oracle_weights  # noqa: E402

pytestmark = pytest.mark.gpu


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _f32(t):
    return t.detach().float().cpu().numpy()


def _kv(rng, b, kh, cap, d):
    k = torch.from_numpy(rng.integers(-127, 128, (b, kh, cap, d)).astype(np.int8))
    v = torch.from_numpy(rng.integers(-127, 128, (b, kh, cap, d)).astype(np.int8))
    ks = torch.from_numpy(rng.uniform(0.002, 0.02, (b, kh, cap)).astype(np.float16))
    vs = torch.from_numpy(rng.uniform(0.002, 0.02, (b, kh, cap)).astype(np.float16))
    return k, ks, v, vs


CASES = [
    # batch, heads, kv_heads, q_len, length, causal, layout[, head_dim (default 128)]
    (1, 32, 8, 200, 200, True, 0),
    (2, 8, 8, 70, 150, True, 1),
    (1, 16, 2, 33, 600, True, 0),
    (1, 8, 4, 17, 90, False, 0),
    (2, 32, 8, 129, 129, True, 1),
    (1, 8, 8, 70, 150, False, 0),  # no mask: warps see keys past their own positions
    # head_dim 256: the reference model's 16 / 4 heads (int8_quantized_sdpa.py:226-230)
    (1, 16, 4, 200, 200, True, 0, 256),
    (2, 16, 4, 45, 301, True, 1, 256),
    (1, 8, 8, 37, 100, False, 0, 256),
    (1, 16, 2, 130, 513, True, 0, 256),
]


@pytest.mark.parametrize("case", CASES)
def test_prefill_attention_matches_oracle(case):
    _need_cuda()
    from spark_b200._lib import check, lib

    b, h, kh, ql, n, causal, layout, *rest = case
    d, cap = (rest[0] if rest else 128), ((n + 15) // 16) * 16 + 16
    rng = np.random.default_rng(sum(case[:5]))
    k, ks, v, vs = _kv(rng, b, kh, cap, d)
    q = torch.randn(b, h, ql, d, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    dev = [t.cuda() for t in (k, ks, v, vs)]
    q_dev = (q if layout == 0 else q.permute(0, 2, 1, 3)).contiguous().cuda()
    out = torch.empty_like(q_dev)
    scale = 1.0 / math.sqrt(d)
    check(lib().sb_int8_sdpa_prefill(q_dev.data_ptr(), dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(),
                                      dev[3].data_ptr(), out.data_ptr(), b, h, kh, ql, n, cap, d, scale,
                                      int(causal), layout, torch.cuda.current_stream().cuda_stream), "prefill")
    torch.cuda.synchronize()
    got = _f32(out if layout == 0 else out.permute(0, 2, 1, 3))
    ref = oracle_ops.sdpa_int8(_f32(q), k[:, :, :n].numpy(), ks[:, :, :n].numpy(), v[:, :, :n].numpy(),
                               vs[:, :, :n].numpy(), scale, causal=causal)
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())


WINDOW_CASES = [
    # batch, heads, kv_heads, q_len, length, window, layout, head_dim
    (2, 16, 4, 37, 48, 12, 1, 256),   # a prompt chunk of a sliding layer (window < chunk)
    (1, 16, 4, 8, 19, 12, 1, 256),    # chunk after the first: window - 1 earlier keys + the chunk
    (1, 32, 8, 130, 700, 64, 0, 128),
    (2, 8, 8, 70, 150, 200, 1, 128),  # a window longer than the context: plain causal
]


@pytest.mark.parametrize("case", WINDOW_CASES)
def test_int8_prefill_window_matches_oracle(case):
    """sb_int8_sdpa_prefill_window: bottom-right causal with a sliding window
    over the INT8 cache vs the float64 masked attention over the dequantized
    cache."""
    _need_cuda()
    from spark_b200._lib import check, lib

    b, h, kh, ql, n, window, layout, d = case
    cap = ((n + 15) // 16) * 16 + 16
    rng = np.random.default_rng(sum(case[:6]))
    k, ks, v, vs = _kv(rng, b, kh, cap, d)
    q = torch.randn(b, h, ql, d, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    dev = [t.cuda() for t in (k, ks, v, vs)]
    q_dev = (q if layout == 0 else q.permute(0, 2, 1, 3)).contiguous().cuda()
    out = torch.empty_like(q_dev)
    scale = 1.0 / math.sqrt(d)
    check(lib().sb_int8_sdpa_prefill_window(q_dev.data_ptr(), dev[0].data_ptr(), dev[1].data_ptr(),
                                             dev[2].data_ptr(), dev[3].data_ptr(), out.data_ptr(), b, h, kh, ql, n,
                                             cap, d, scale, window, layout, torch.cuda.current_stream().cuda_stream),
          "prefill window")
    torch.cuda.synchronize()
    got = _f32(out if layout == 0 else out.permute(0, 2, 1, 3))
    kd = k[:, :, :n].numpy().astype(np.float64) * ks[:, :, :n].numpy().astype(np.float64)[..., None]
    vd = v[:, :, :n].numpy().astype(np.float64) * vs[:, :, :n].numpy().astype(np.float64)[..., None]
    ref = oracle_ops.sdpa_masked(_f32(q), kd, vd, scale, causal=True, window=window)
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())


def test_prefill_attention_single_query_equals_decode_kernel():
    _need_cuda()
    from spark_b200 import ops

    rng = np.random.default_rng(7)
    b, h, kh, n, d = 2, 32, 8, 777, 128
    cap = 800
    k, ks, v, vs = (t.cuda() for t in _kv(rng, b, kh, cap, d))
    q = torch.randn(b, h, 1, d, device="cuda").to(torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    dec = ops.int8_sdpa_decode(q, k, ks, v, vs, n, scale)
    pre = ops.int8_sdpa_prefill(q, k, ks, v, vs, n, scale, True)
    torch.testing.assert_close(pre.float(), dec.float(), rtol=1e-2, atol=2e-3)


def test_dispatch_sdpa_routes_int8_prefill():
    _need_cuda()
    from spark_b200 import dispatch

    rng = np.random.default_rng(8)
    b, h, kh, n, d, ql = 1, 8, 2, 64, 128, 16
    k, ks, v, vs = (t.cuda() for t in _kv(rng, b, kh, n, d))
    q = torch.randn(b, h, ql, d, device="cuda").to(torch.bfloat16)
    out = dispatch.dispatch_sdpa(q, (k, ks), (v, vs), cache=None, scale=0.1, mask="causal")
    ref = oracle_ops.sdpa_int8(_f32(q), k.cpu().numpy(), ks.cpu().numpy(), v.cpu().numpy(), vs.cpu().numpy(), 0.1,
                               causal=True)
    np.testing.assert_allclose(_f32(out), ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())


def test_prefill_rejects_bad_shapes():
    _need_cuda()
    from spark_b200._lib import SB_EINVAL, lib

    z = torch.zeros(1024, dtype=torch.int8, device="cuda")
    p = z.data_ptr()
    s = torch.cuda.current_stream().cuda_stream
    # q_len > length, head_dim 64, G = 3
    assert lib().sb_int8_sdpa_prefill(p, p, p, p, p, p, 1, 8, 8, 10, 5, 16, 128, 0.1, 1, 0, s) == SB_EINVAL
    assert lib().sb_int8_sdpa_prefill(p, p, p, p, p, p, 1, 8, 8, 1, 5, 16, 64, 0.1, 1, 0, s) == SB_EINVAL
    assert lib().sb_int8_sdpa_prefill(p, p, p, p, p, p, 1, 6, 2, 1, 5, 16, 128, 0.1, 1, 0, s) == SB_EINVAL


# ------------------------------------------------------------------ decoder prompt
@pytest.fixture(scope="module")
def pair():
    _need_cuda()
    from spark_b200.decoder import DecoderConfig, SyntheticDecoder

    cfg = DecoderConfig.small(num_layers=2)
    mk = lambda: SyntheticDecoder(cfg, batch=2, capacity=160, seed=5, engine="launches")  # noqa: E731
    return mk(), mk()


def test_chunked_prompt_matches_single_token_prompt(pair):
    chunked, stepwise = pair
    rng = np.random.default_rng(11)
    prompt = torch.from_numpy(rng.integers(0, chunked.cfg.vocab, (2, 100)).astype(np.int32)).cuda()
    chunked.prefill(prompt, chunk=32)  # 3 full chunks and a ragged one
    stepwise.prefill_stepwise(prompt)
    torch.cuda.synchronize()
    assert torch.equal(chunked.positions, stepwise.positions)
    assert int(chunked.positions[0]) == 100
    for li in range(chunked.cfg.num_layers):
        a = chunked.k_cache[li][:, :, :100].int()
        b = stepwise.k_cache[li][:, :, :100].int()
        diff = (a - b).abs()
        # the two paths round the projections at different points (tensor-core
        # tiles vs the GEMV's split-K), so a code at a rounding boundary moves by
        # one; deeper layers inherit their inputs' differences
        assert diff.max() <= 2, li
        assert (diff > 0).float().mean() < 0.10, li
        deq_a = a.float() * chunked.k_scale[li][:, :, :100, None].float()
        deq_b = b.float() * stepwise.k_scale[li][:, :, :100, None].float()
        torch.testing.assert_close(deq_a, deq_b, rtol=2e-2, atol=2e-2 * float(deq_b.abs().max()))
        torch.testing.assert_close(chunked.v_scale[li][:, :, :100], stepwise.v_scale[li][:, :, :100], rtol=2e-2,
                                   atol=1e-4)
    np.testing.assert_allclose(_f32(chunked.x), _f32(stepwise.x), rtol=2e-2, atol=5e-2)
    # decoding continues from the chunked prompt
    toks = chunked.decode(4)
    assert toks.shape == (2, 4)
    chunked.check_status()


def test_chunked_prompt_matches_oracle():
    _need_cuda()
    from spark_b200.decoder import DecoderConfig, SyntheticDecoder

    cfg = DecoderConfig.small(num_layers=2)
    dec = SyntheticDecoder(cfg, batch=1, capacity=96, seed=6, engine="launches")
    orc = OracleDecoder(oracle_weights(dec), num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads,
                        head_dim=cfg.head_dim, rope_theta=cfg.rope_theta, eps=cfg.rms_eps, group=cfg.mlp_group,
                        capacity=dec.capacity, batch=1)
    rng = np.random.default_rng(12)
    prompt = rng.integers(0, cfg.vocab, (1, 80)).astype(np.int32)
    dec.prefill(torch.from_numpy(prompt).cuda(), chunk=64)
    torch.cuda.synchronize()
    for t in range(prompt.shape[1]):
        logits = orc.step(prompt[:, t], t)
    np.testing.assert_allclose(_f32(dec.x), orc.last_x, rtol=2e-2, atol=5e-2)
    top2 = np.sort(logits, axis=-1)[0, -2:]
    if top2[1] - top2[0] > 1e-2 * abs(top2[1]) + 1e-3:
        assert int(dec.tokens[0]) == int(orc.greedy(logits)[0])


# ------------------------------------------------------------ bf16 multi-query attention
BF16_CASES = [
    # batch, heads, kv_heads, q_len, length, causal, window, sliding mask (window of a boolean mask), layout[, head_dim]
    (1, 16, 4, 8, 519, False, 0, 128, 0),  # the reference's verification geometry at D = 128, boolean sliding mask
    (2, 8, 8, 33, 200, True, 64, 0, 1),
    (1, 32, 8, 1, 77, False, 0, 0, 0),
    (1, 8, 1, 70, 300, True, 0, 0, 0),
    # head_dim 256
    (1, 16, 4, 8, 519, False, 0, 128, 0, 256),
    (2, 16, 4, 33, 200, True, 64, 0, 1, 256),
    (1, 8, 2, 70, 300, True, 0, 0, 0, 256),
]


@pytest.mark.parametrize("case", BF16_CASES)
def test_bf16_multiquery_matches_oracle(case):
    _need_cuda()
    from spark_b200._lib import check, lib

    b, h, kh, ql, n, causal, window, mwin, layout, *rest = case
    d = rest[0] if rest else 128
    gen = torch.Generator().manual_seed(sum(case[:5]))
    q = torch.randn(b, h, ql, d, generator=gen).to(torch.bfloat16)
    k = torch.randn(b, kh, n, d, generator=gen).to(torch.bfloat16)
    v = torch.randn(b, kh, n, d, generator=gen).to(torch.bfloat16)
    mask = None
    if mwin:
        pos = np.arange(n - ql, n)[:, None]
        keys = np.arange(n)[None, :]
        mask = (keys <= pos) & (keys > pos - mwin)
        mask[3] = False  # one query sees nothing: zeros
    q_dev = (q if layout == 0 else q.permute(0, 2, 1, 3)).contiguous().cuda()
    out = torch.empty_like(q_dev)
    m_dev = torch.from_numpy(mask.astype(np.uint8)).cuda() if mask is not None else None
    scale = 1.0 / math.sqrt(d)
    k_dev, v_dev = k.cuda(), v.cuda()  # kept alive until the kernel has run
    check(lib().sb_bf16_sdpa_multiquery(q_dev.data_ptr(), k_dev.data_ptr(), v_dev.data_ptr(), out.data_ptr(),
                                        b, h, kh, ql, n, n, d, scale, int(causal), window,
                                        m_dev.data_ptr() if m_dev is not None else None, n, layout,
                                        torch.cuda.current_stream().cuda_stream), "bf16 multiquery")
    torch.cuda.synchronize()
    got = _f32(out if layout == 0 else out.permute(0, 2, 1, 3))
    ref = oracle_ops.sdpa_masked(_f32(q), _f32(k), _f32(v), scale, causal=causal, window=window, mask=mask)
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())


def test_ext_bf16_multiquery_masks():
    _need_cuda()
    from spark_b200 import ext

    gen = torch.Generator().manual_seed(9)
    q = torch.randn(1, 8, 8, 128, generator=gen).to(torch.bfloat16).cuda()
    k = torch.randn(1, 2, 100, 128, generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn(1, 2, 100, 128, generator=gen).to(torch.bfloat16).cuda()
    causal = ext.bf16_sdpa_multiquery(q, k, v, scale=0.08, mask="causal")
    ref = oracle_ops.sdpa_masked(_f32(q), _f32(k), _f32(v), 0.08, causal=True)
    np.testing.assert_allclose(_f32(causal), ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())
    band = np.zeros((8, 100), bool)
    band[:, 40:60] = True
    masked = ext.bf16_sdpa_multiquery(q, k, v, scale=0.08, mask=torch.from_numpy(band)[None, None].cuda())
    ref = oracle_ops.sdpa_masked(_f32(q), _f32(k), _f32(v), 0.08, mask=band)
    np.testing.assert_allclose(_f32(masked), ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())
    with pytest.raises(ValueError):
        ext.bf16_sdpa_multiquery(q, k, v, scale=0.08, mask=torch.ones(2, 8, 100, dtype=torch.bool).cuda())
