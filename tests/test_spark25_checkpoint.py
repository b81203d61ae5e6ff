"""MLX-affine checkpoint loading (CPU): the safetensors reader/writer, the
Spark2_5 config checks of ``ModelArgs`` (``spark_mlx_llm/model.py:30-127``),
``Model.sanitize`` (``model.py:378-396``), and the NumPy oracle of the block
on a small checkpoint."""

import json
import os

import numpy as np
import pytest

from _spark25_ckpt import CONFIG, write_checkpoint


def test_safetensors_round_trip(tmp_path):
    from spark_b200.checkpoint import read_safetensors, write_safetensors

    rng = np.random.default_rng(0)
    t = {"a": ("BF16", rng.integers(0, 65535, (3, 5), dtype=np.uint16)),
         "b.weight": ("U32", rng.integers(0, 2**32, (4, 2), dtype=np.uint64).astype(np.uint32)),
         "c": ("F32", rng.standard_normal(7).astype(np.float32)),
         "d": ("I8", rng.integers(-128, 127, (2, 2, 2), dtype=np.int8))}
    path = tmp_path / "x.safetensors"
    write_safetensors(path, t, metadata={"format": "mlx"})
    back = read_safetensors(path)
    assert set(back) == set(t)
    for name, (dt, arr) in t.items():
        assert back[name][0] == dt
        np.testing.assert_array_equal(back[name][1], arr)
    # the header is JSON after an 8-byte little-endian length
    raw = path.read_bytes()
    n = int.from_bytes(raw[:8], "little")
    assert json.loads(raw[8:8 + n])["__metadata__"] == {"format": "mlx"}


def test_checkpoint_dir_and_sanitize(tmp_path):
    from spark_b200.checkpoint import load_checkpoint_dir
    from spark_b200.spark25 import Spark25Config, sanitize

    written = write_checkpoint(tmp_path, shards=3)
    config, weights = load_checkpoint_dir(tmp_path)
    assert config == json.loads(json.dumps(CONFIG))
    assert set(weights) == set(written)
    cfg = Spark25Config.from_dict(config)
    assert cfg.rope("sliding_attention") == (128, 10000.0) and cfg.rope("full_attention") == (256, 1e6)
    clean = sanitize(weights, cfg.tie_word_embeddings)
    assert "model.embedding.weight" in clean and "model.embed_tokens.weight" not in clean
    assert not any("rotary_emb" in k for k in clean)
    with pytest.raises(NotADirectoryError):
        load_checkpoint_dir(tmp_path / "missing")


@pytest.mark.parametrize("change,match", [
    ({"model_type": "llama"}, "spark2_5"),
    ({"hidden_act": "silu"}, "GELU"),
    ({"gate_attn_act_mode": "tanh"}, "sigmoid"),
    ({"layer_types": ["full_attention"]}, "layer_types length"),
    ({"rope_parameters": {"full_attention": {}}}, "Missing RoPE"),
    ({"num_key_value_heads": 3}, "divisible"),
    ({"head_dim": 96}, "head_dim"),
    ({"sliding_window": 0}, "positive"),
])
def test_config_checks(change, match):
    from spark_b200.spark25 import Spark25Config

    with pytest.raises(ValueError, match=match):
        Spark25Config.from_dict(dict(CONFIG, **change))


def test_default_layer_pattern():
    from spark_b200.spark25 import Spark25Config

    cfg = Spark25Config.from_dict({k: v for k, v in CONFIG.items() if k != "layer_types"})
    assert cfg.layer_types == ["sliding_attention"] * 3 + ["full_attention"]


def test_oracle_window_matters(tmp_path):
    """The oracle's sliding layers see only the last ``sliding_window`` keys: past
    the window the logits differ from a model whose layers are all full."""
    from oracle.spark25 import Spark25Oracle
    from spark_b200.checkpoint import load_checkpoint_dir
    from spark_b200.spark25 import Spark25Config, sanitize

    write_checkpoint(tmp_path)
    config, weights = load_checkpoint_dir(tmp_path)
    cfg = Spark25Config.from_dict(config)
    full = Spark25Config.from_dict(dict(config, layer_types=["full_attention"] * 4,
                                        rope_parameters={"full_attention": {"rope_theta": 1e6}}))
    w = sanitize(weights)
    tokens = np.random.default_rng(1).integers(0, 1000, 16)
    a, b = Spark25Oracle(cfg, w, 1), Spark25Oracle(full, w, 1)
    outs = [(a.step(t), b.step(t)) for t in tokens]
    assert np.all(np.isfinite(outs[-1][0]))
    assert not np.array_equal(outs[-1][0], outs[-1][1])


@pytest.mark.parametrize("window,chunk,prompt", [(12, 8, 37), (12, 4, 14), (5, 16, 70), (17, 1, 40)])
def test_mirrored_ring_keeps_every_window_contiguous(window, chunk, prompt):
    """Host logic of the rotating cache: position p written to ring slot p % R and
    to its mirror row p % R + R. After each prompt chunk (and each decode step
    after the prompt), the rows the attention reads - [start % R, start % R + n)
    with start the first position in the window - hold exactly the positions
    start .. start + n - 1 in order."""
    from spark_b200.spark25 import ring_slots

    r = ring_slots(window, chunk, 1 << 20)
    assert r >= window + chunk - 1 and r % 16 == 0
    assert ring_slots(window, chunk, 2 * r) == 0  # no smaller than the cache: linear
    rows = [None] * (2 * r)

    def append(p):
        rows[p % r] = rows[p % r + r] = p

    def check(c0, lc):
        start = max(0, c0 - window + 1)
        n = c0 + lc - start
        assert n <= r
        assert rows[start % r:start % r + n] == list(range(start, c0 + lc))

    for c0 in range(0, prompt, chunk):
        lc = min(chunk, prompt - c0)
        for p in range(c0, c0 + lc):
            append(p)
        check(c0, lc)
    for p in range(prompt, prompt + 3 * r):  # decode: one position per step
        append(p)
        check(p, 1)
