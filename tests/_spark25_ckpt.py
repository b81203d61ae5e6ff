"""A small random Spark2_5 checkpoint in the MLX-affine safetensors layout
(the tensor names of ``spark_mlx_llm/model.py``), written with the library's
own safetensors writer: head_dim 256, GQA 2:1, G32 4-bit projections with an
8-bit out_proj, a bf16 head gate, a 4-bit tied embedding, three sliding
layers and one full layer with partial rotary on the sliding ones."""

import json
import os

import numpy as np

from oracle import quant
from oracle.formats import bf16_bits

CONFIG = dict(model_type="spark2_5", hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
              num_attention_heads=4, num_key_value_heads=2, head_dim=256, vocab_size=1000, sliding_window=12,
              rope_parameters={"sliding_attention": {"rope_theta": 10000.0, "partial_rotary_factor": 0.5},
                               "full_attention": {"rope_theta": 1000000.0}},
              layer_types=["sliding_attention"] * 3 + ["full_attention"], rms_norm_eps=1e-6,
              max_position_embeddings=256, tie_word_embeddings=True, hidden_act="gelu",
              quantization={"group_size": 32, "bits": 4})


def make_weights(seed=0, cfg=CONFIG):
    rng = np.random.default_rng(seed)
    hid, inter = cfg["hidden_size"], cfg["intermediate_size"]
    hq, hkv, d = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    w = {}

    def affine(name, n, k, bits=4, group=32, std=0.02):
        packed, s, b = quant.quantize_affine_minmax(rng.standard_normal((n, k)).astype(np.float32) * std, group, bits)
        w[f"{name}.weight"] = ("U32", packed)
        w[f"{name}.scales"] = ("BF16", s)
        w[f"{name}.biases"] = ("BF16", b)

    def bf16(name, arr):
        w[name] = ("BF16", bf16_bits(np.asarray(arr, np.float32)))

    affine("model.embed_tokens", cfg["vocab_size"], hid, std=1.0)  # renamed to model.embedding on load
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        bf16(f"{p}.input_layernorm.weight", 1 + 0.1 * rng.standard_normal(hid))
        bf16(f"{p}.post_attention_layernorm.weight", 1 + 0.1 * rng.standard_normal(hid))
        affine(f"{p}.self_attn.q_k_v_proj", (hq + 2 * hkv) * d, hid, std=0.05)
        bf16(f"{p}.self_attn.g_proj.weight", 0.05 * rng.standard_normal((hq, hid)))
        affine(f"{p}.self_attn.out_proj", hid, hq * d, bits=8, group=64)
        affine(f"{p}.mlp.gate_proj", inter, hid)
        affine(f"{p}.mlp.up_proj", inter, hid)
        affine(f"{p}.mlp.down_proj", hid, inter)
        w[f"{p}.self_attn.rotary_emb.inv_freq"] = ("F32", np.arange(4, dtype=np.float32))  # dropped on load
    bf16("model.norm.weight", 1 + 0.1 * rng.standard_normal(hid))
    return w


def write_checkpoint(path, seed=0, shards=2):
    """config.json + model-0000i-of-0000n.safetensors; returns the weights dict."""
    from spark_b200.checkpoint import write_safetensors

    weights = make_weights(seed)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(CONFIG, f)
    names = sorted(weights)
    for s in range(shards):
        part = {n: weights[n] for n in names[s::shards]}
        write_safetensors(os.path.join(path, f"model-{s + 1:05d}-of-{shards:05d}.safetensors"), part)
    return weights
