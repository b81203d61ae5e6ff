"""The multithreaded C restatement agrees with the NumPy oracle (CPU only)."""

import numpy as np
import pytest

from oracle import formats, ops, quant
from oracle.cpu_decoder import CDecoder, load_library
from oracle.model import OracleDecoder


@pytest.fixture(scope="module")
def lib():
    try:
        return load_library()
    except RuntimeError:
        import __graft_entry__

        __graft_entry__.build()
        return load_library()


def _p(a):
    import ctypes

    return a.ctypes.data_as(ctypes.c_void_p)


def test_affine_linear(lib):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((96, 512)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize_affine_minmax(w, 64, 4)
    x = formats.round_bf16(rng.standard_normal((3, 512)).astype(np.float32))
    y = np.empty((3, 96), np.float32)
    lib.oc_affine_linear(_p(x), 3, _p(packed), _p(s), _p(b), 96, 512, 64, 4, _p(y))
    ref = ops.affine_linear(x, packed, formats.bf16_from_bits(s), formats.bf16_from_bits(b), 64, 4)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)


def test_sdpa(lib):
    rng = np.random.default_rng(1)
    q = rng.standard_normal((2, 8, 128)).astype(np.float32)
    kq, ks = quant.quantize_kv_symmetric(rng.standard_normal((2, 2, 40, 128)).astype(np.float32))
    vq, vs = quant.quantize_kv_symmetric(rng.standard_normal((2, 2, 40, 128)).astype(np.float32))
    out = np.empty((2, 8, 128), np.float32)
    lib.oc_sdpa_int8(_p(q), _p(kq), _p(ks.view(np.uint16)), _p(vq), _p(vs.view(np.uint16)), 2, 8, 2, 33, 40, 128,
                     0.09, _p(out))
    ref = ops.sdpa_int8(q[:, :, None], kq[:, :, :33], ks[:, :, :33], vq[:, :, :33], vs[:, :, :33], 0.09)
    np.testing.assert_allclose(out, ref[:, :, 0], rtol=1e-4, atol=1e-5)


def test_decoder_step_matches_numpy_oracle(lib):
    rng = np.random.default_rng(2)
    hidden, hq, hkv, d, inter, vocab = 256, 4, 2, 128, 512, 300

    def aff(n, k):
        return quant.quantize_affine_minmax((rng.standard_normal((n, k)) * 0.02).astype(np.float32), 64, 4)

    layers_raw, layers_f = [], []
    for _ in range(2):
        qw, qs = quant.quantize_w8_per_channel((rng.standard_normal(((hq + 2 * hkv) * d, hidden)) * 0.02).astype(np.float32))
        ow, os_ = quant.quantize_w8_per_channel((rng.standard_normal((hidden, hq * d)) * 0.02).astype(np.float32))
        gate, up, down = aff(inter, hidden), aff(inter, hidden), aff(hidden, inter)
        norm = np.ones(hidden, np.float32)
        layers_raw.append(dict(qkv_w=qw, qkv_s=qs, o_w=ow, o_s=os_, gate=gate, up=up, down=down, in_norm=norm,
                               post_norm=norm))
        tof = lambda t: (t[0], formats.bf16_from_bits(t[1]), formats.bf16_from_bits(t[2]))  # noqa: E731
        layers_f.append(dict(qkv_w=qw, qkv_s=qs, o_w=ow, o_s=os_, gate=tof(gate), up=tof(up), down=tof(down),
                             in_norm=norm, post_norm=norm))
    embed = formats.bf16_bits(rng.standard_normal((vocab, hidden)).astype(np.float32))
    head = formats.bf16_bits((rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32))
    kw = dict(num_heads=hq, num_kv_heads=hkv, head_dim=d, rope_theta=1e6, eps=1e-6, group=64, capacity=8, batch=2)
    cdec = CDecoder(dict(layers=layers_raw, embed_bits=embed, head_bits=head, final_norm=np.ones(hidden, np.float32)),
                    **kw)
    ndec = OracleDecoder(dict(layers=layers_f, embed=formats.bf16_from_bits(embed), head=formats.bf16_from_bits(head),
                              final_norm=np.ones(hidden, np.float32)), **kw)
    toks = np.array([3, 7])
    for pos in range(4):
        c_next = cdec.step(toks, pos)
        logits = ndec.step(toks, pos)
        np.testing.assert_allclose(cdec.last_x, ndec.last_x, rtol=2e-2, atol=2e-2)
        top2 = np.sort(logits, axis=-1)[:, -2:]
        decisive = (top2[:, 1] - top2[:, 0]) > 1e-3
        assert np.all(c_next[decisive] == ndec.greedy(logits)[decisive])
        toks = c_next


def test_prefill_chunk_equals_sequential_steps(lib):
    """The oracle's chunked prompt pass (8 positions per weight pass) gives the
    same cache, hidden state and greedy token as one decode step per position."""
    rng = np.random.default_rng(5)
    hidden, hq, hkv, d, inter, vocab = 256, 4, 2, 128, 512, 300

    def aff(n, k):
        return quant.quantize_affine_minmax((rng.standard_normal((n, k)) * 0.02).astype(np.float32), 64, 4)

    layers = []
    for _ in range(2):
        qw, qs = quant.quantize_w8_per_channel((rng.standard_normal(((hq + 2 * hkv) * d, hidden)) * 0.02).astype(np.float32))
        ow, os_ = quant.quantize_w8_per_channel((rng.standard_normal((hidden, hq * d)) * 0.02).astype(np.float32))
        norm = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
        layers.append(dict(qkv_w=qw, qkv_s=qs, o_w=ow, o_s=os_, gate=aff(inter, hidden), up=aff(inter, hidden),
                           down=aff(hidden, inter), in_norm=norm, post_norm=norm))
    w = dict(layers=layers, embed_bits=formats.bf16_bits(rng.standard_normal((vocab, hidden)).astype(np.float32)),
             head_bits=formats.bf16_bits((rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)),
             final_norm=np.ones(hidden, np.float32))
    kw = dict(num_heads=hq, num_kv_heads=hkv, head_dim=d, rope_theta=1e6, eps=1e-6, group=64, capacity=32, batch=1)
    seq, chunked = CDecoder(w, **kw), CDecoder(w, **kw)
    prompt = rng.integers(0, vocab, 13)
    for t in range(13):
        tok = seq.step(prompt[t:t + 1], t)
    for start in range(0, 13, 8):
        got = chunked.prefill_chunk(prompt[start:start + 8], start, want_argmax=start + 8 >= 13)
    assert int(got) == int(tok[0])
    np.testing.assert_array_equal(chunked.last_x[-1], seq.last_x[0])
    np.testing.assert_array_equal(chunked.kq, seq.kq)
    np.testing.assert_array_equal(chunked.vs, seq.vs)
