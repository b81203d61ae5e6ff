"""The oracle's masked attention (``oracle.ops.sdpa_masked``) on the CPU."""

import numpy as np

from oracle import ops


def _qkv(rng, b=1, h=4, kh=2, l=5, n=9, d=8):
    return (rng.standard_normal((b, h, l, d)), rng.standard_normal((b, kh, n, d)), rng.standard_normal((b, kh, n, d)))


def test_causal_matches_the_staged_recipe():
    q, k, v = _qkv(np.random.default_rng(0))
    np.testing.assert_allclose(ops.sdpa_masked(q, k, v, 0.3, causal=True), ops._attend(q, k, v, 0.3, True))
    np.testing.assert_allclose(ops.sdpa_masked(q, k, v, 0.3), ops._attend(q, k, v, 0.3, False))


def test_window_equals_the_explicit_band_mask():
    q, k, v = _qkv(np.random.default_rng(1), l=6, n=20)
    pos = np.arange(20 - 6, 20)[:, None]
    keys = np.arange(20)[None, :]
    band = (keys <= pos) & (keys > pos - 4)
    np.testing.assert_allclose(ops.sdpa_masked(q, k, v, 0.5, causal=True, window=4),
                               ops.sdpa_masked(q, k, v, 0.5, mask=band))


def test_fully_masked_query_is_zero():
    q, k, v = _qkv(np.random.default_rng(2), l=3, n=4)
    mask = np.ones((3, 4), bool)
    mask[1] = False
    out = ops.sdpa_masked(q, k, v, 1.0, mask=mask)
    assert np.all(out[:, :, 1] == 0) and np.all(np.isfinite(out))
