"""Synthetic decoder step in NumPy (oracle, test infrastructure only).

Mirrors the layer order of ``spark_mlx_llm/model.py:172-207,249-262`` and the
bf16 rounding points of the reference's MLX graph: every tensor the reference
materialises in the activation dtype (norm outputs, projections, RoPE output,
attention output, residual sums, the gated activation) is rounded to bf16
here too; arithmetic inside an operator is float64. The KV cache holds the
symmetric INT8 codes and fp16 scales of ``quant.quantize_kv_symmetric``.
Weights are passed in (the exact quantized tensors the GPU uses).
"""

import numpy as np

from . import ops
from .formats import round_bf16
from .quant import quantize_kv_symmetric

__all__ = ["OracleDecoder"]


class OracleDecoder:
    """``weights``: dict with per-layer lists of numpy arrays (float32 values):

    qkv_w int8 [N, H], qkv_s f32 [N], o_w int8 [H, Q], o_s f32 [H],
    gate/up/down = (packed uint32, scales f32, biases f32), in_norm/post_norm f32,
    and embed f32 [V, H], head f32 [V, H], final_norm f32 [H].
    """

    def __init__(self, weights, *, num_heads, num_kv_heads, head_dim, rope_theta, eps, group, capacity, batch):
        self.w = weights
        self.hq, self.hkv, self.d = num_heads, num_kv_heads, head_dim
        self.theta, self.eps, self.group = rope_theta, eps, group
        layers = len(weights["layers"])
        self.kq = np.zeros((layers, batch, num_kv_heads, capacity, head_dim), np.int8)
        self.vq = np.zeros_like(self.kq)
        self.ks = np.ones((layers, batch, num_kv_heads, capacity), np.float16)
        self.vs = np.ones_like(self.ks)

    def step(self, tokens, position):
        """One decode step for tokens [B] at position ``position``; returns fp64 logits [B, V]."""
        w = self.w
        x = w["embed"][np.asarray(tokens)]
        bsz = x.shape[0]
        d = self.d
        for li, layer in enumerate(w["layers"]):
            xn = round_bf16(ops.rms_norm(x, layer["in_norm"], self.eps))
            qkv = round_bf16(ops.w8a16_per_channel(xn, layer["qkv_w"], layer["qkv_s"]))
            q = qkv[:, : self.hq * d].reshape(bsz, self.hq, 1, d)
            k = qkv[:, self.hq * d:(self.hq + self.hkv) * d].reshape(bsz, self.hkv, 1, d)
            v = qkv[:, (self.hq + self.hkv) * d:].reshape(bsz, self.hkv, 1, d)
            pos = np.full((bsz, 1, 1), position)
            q = round_bf16(ops.rope(q, pos, d, self.theta))
            k = round_bf16(ops.rope(k, pos, d, self.theta))
            kq, ks = quantize_kv_symmetric(k[:, :, 0])
            vq, vs = quantize_kv_symmetric(v[:, :, 0])
            self.kq[li, :, :, position], self.ks[li, :, :, position] = kq, ks
            self.vq[li, :, :, position], self.vs[li, :, :, position] = vq, vs
            n = position + 1
            attn = ops.sdpa_int8(q, self.kq[li, :, :, :n], self.ks[li, :, :, :n], self.vq[li, :, :, :n],
                                 self.vs[li, :, :, :n], 1.0 / np.sqrt(d))
            attn = round_bf16(attn.reshape(bsz, self.hq * d))
            o = round_bf16(ops.w8a16_per_channel(attn, layer["o_w"], layer["o_s"]))
            x = round_bf16(x + o)
            xn = round_bf16(ops.rms_norm(x, layer["post_norm"], self.eps))
            g = round_bf16(ops.affine_linear(xn, *layer["gate"], self.group, 4))
            u = round_bf16(ops.affine_linear(xn, *layer["up"], self.group, 4))
            act = round_bf16(ops.swiglu(g, u))
            dn = round_bf16(ops.affine_linear(act, *layer["down"], self.group, 4))
            x = round_bf16(x + dn)
        self.last_x = x
        xn = round_bf16(ops.rms_norm(x, w["final_norm"], self.eps))
        return xn.astype(np.float64) @ w["head"].astype(np.float64).T

    @staticmethod
    def greedy(logits):
        """argmax with the lowest index on ties."""
        return np.argmax(logits, axis=-1)
