"""Test infrastructure: a NumPy restatement of the reference Spark2_5 decoder step.

Only the tests import this module; it is the checker of
``spark_b200.spark25.Spark25Model``, never part of the product path. It
follows the reference block (``spark_mlx_llm/model.py:172-262``): RMSNorm,
the fused q/k/v projection (MLX-affine weights, ``ops/linear.py:180-191``),
non-traditional RoPE on the first ``dims`` features (``model.py:162-170``),
attention over the cache with a sliding window on sliding layers
(``model.py:313-320``, RotatingKVCache ``:362-370``), the sigmoid head gate
(``ops/attention_output.py:91-95``), ``h = x + out_proj(o)`` and
``x = h + down(gelu(gate(rms_norm(h))) * up(rms_norm(h)))`` (``ops/ffn.py:98-103``),
then the final norm and the tied lm_head (``model.py:326-333``). Values are
carried as float64 and rounded to bf16 where the reference's bf16 tensors are.
The KV cache uses the BASELINE symmetric INT8 format (``quant.quantize_kv_symmetric``)
because the runner does; the reference's own caches are bf16 or affine
uint8/G32.
"""

import numpy as np

from . import ops, quant
from .formats import bf16_from_bits, round_bf16

__all__ = ["Spark25Oracle"]


def _r(x):
    return round_bf16(np.asarray(x, dtype=np.float32)).astype(np.float64)


class Spark25Oracle:
    """``weights``: ``{name: (dtype, array)}`` as read from the checkpoint (BF16 as
    bits, U32 packed codes); ``cfg``: a ``Spark25Config``."""

    def __init__(self, cfg, weights, batch):
        self.cfg, self.batch = cfg, batch
        self.w = weights
        hkv, d = cfg.num_key_value_heads, cfg.head_dim
        self.kq = [np.zeros((batch, hkv, 0, d), np.int8) for _ in range(cfg.num_hidden_layers)]
        self.ks = [np.zeros((batch, hkv, 0), np.float16) for _ in range(cfg.num_hidden_layers)]
        self.vq = [np.zeros((batch, hkv, 0, d), np.int8) for _ in range(cfg.num_hidden_layers)]
        self.vs = [np.zeros((batch, hkv, 0), np.float16) for _ in range(cfg.num_hidden_layers)]
        self.pos = 0
        self.last_hidden = None

    def _bf(self, name):
        return bf16_from_bits(np.asarray(self.w[name][1])).astype(np.float64)

    def _lin(self, x, name):
        if f"{name}.scales" in self.w:
            packed = np.asarray(self.w[f"{name}.weight"][1]).view(np.uint32)
            s, b = self._bf(f"{name}.scales"), self._bf(f"{name}.biases")
            k = x.shape[-1]
            bits = packed.shape[1] * 32 // k
            return ops.affine_linear(x, packed, s, b, k // s.shape[1], bits)
        return np.asarray(x, np.float64) @ self._bf(f"{name}.weight").T

    def _embed(self, tokens):
        name = "model.embedding"
        if f"{name}.scales" in self.w:
            packed = np.asarray(self.w[f"{name}.weight"][1]).view(np.uint32)[tokens]
            s, b = self._bf(f"{name}.scales")[tokens], self._bf(f"{name}.biases")[tokens]
            hid = self.cfg.hidden_size
            bits = packed.shape[1] * 32 // hid
            return _r(quant.dequantize_affine(packed, s, b, hid // s.shape[1], bits))
        return self._bf(f"{name}.weight")[tokens]

    def step(self, tokens):
        """One position for every sequence; returns float64 logits (bf16 values)."""
        cfg, b = self.cfg, self.batch
        hq, hkv, d, eps = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rms_norm_eps
        tokens = np.asarray(tokens, np.int64).reshape(b)
        x = self._embed(tokens)
        pos = self.pos
        for li in range(cfg.num_hidden_layers):
            p = f"model.layers.{li}"
            xn = _r(ops.rms_norm(x, self._bf(f"{p}.input_layernorm.weight"), eps))
            qkv = _r(self._lin(xn, f"{p}.self_attn.q_k_v_proj"))
            q = qkv[:, :hq * d].reshape(b, hq, 1, d)
            k = qkv[:, hq * d:(hq + hkv) * d].reshape(b, hkv, 1, d)
            v = qkv[:, (hq + hkv) * d:].reshape(b, hkv, 1, d)
            dims, base = cfg.rope(cfg.layer_types[li])
            q = _r(ops.rope(q, np.full((b, 1, 1), pos), dims, base))
            k = _r(ops.rope(k, np.full((b, 1, 1), pos), dims, base))
            kq, ks = quant.quantize_kv_symmetric(k)
            vq, vs = quant.quantize_kv_symmetric(v)
            self.kq[li] = np.concatenate([self.kq[li], kq], axis=2)
            self.ks[li] = np.concatenate([self.ks[li], ks], axis=2)
            self.vq[li] = np.concatenate([self.vq[li], vq], axis=2)
            self.vs[li] = np.concatenate([self.vs[li], vs], axis=2)
            start = max(0, pos + 1 - cfg.sliding_window) if cfg.layer_types[li] == "sliding_attention" else 0
            o = ops.sdpa_int8(q, self.kq[li][:, :, start:], self.ks[li][:, :, start:], self.vq[li][:, :, start:],
                              self.vs[li][:, :, start:], d ** -0.5, causal=True)
            o = _r(o).reshape(b, hq, d)
            gated = _r(ops.head_gate(xn, self._bf(f"{p}.self_attn.g_proj.weight"), o)).reshape(b, hq * d)
            h = _r(x + _r(self._lin(gated, f"{p}.self_attn.out_proj")))
            hn = _r(ops.rms_norm(h, self._bf(f"{p}.post_attention_layernorm.weight"), eps))
            g = _r(self._lin(hn, f"{p}.mlp.gate_proj"))
            u = _r(self._lin(hn, f"{p}.mlp.up_proj"))
            a = _r(ops.gelu_glu(g, u))
            x = _r(h + _r(self._lin(a, f"{p}.mlp.down_proj")))
        self.last_hidden = x
        self.pos += 1
        return self.head(x)

    def head(self, x):
        """Final RMSNorm and the lm_head (the tied embedding) of hidden states ``x``."""
        xn = _r(ops.rms_norm(x, self._bf("model.norm.weight"), self.cfg.rms_norm_eps))
        return _r(self._lin(xn, "model.embedding" if self.cfg.tie_word_embeddings else "lm_head"))
