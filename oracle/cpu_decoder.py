"""Decoder step on the multithreaded C restatement (oracle/c/oracle_cpu.c).

TEST INFRASTRUCTURE / CPU BASELINE ONLY. Same layer order and bf16 rounding
points as ``oracle.model.OracleDecoder`` (spark_mlx_llm/model.py:172-207,
249-262), with the heavy operators (affine and per-channel int8 GEMV, INT8-KV
attention, the bf16 lm_head + argmax) in C over all host cores. Weights use
the raw formats of the GPU path: packed uint32 codes with bf16 scale/bias
bits, int8 codes with fp32 scales, bf16 bits for embedding and lm_head.
"""

import ctypes
import os

import numpy as np

from . import ops
from .formats import bf16_from_bits, round_bf16
from .quant import quantize_kv_symmetric

__all__ = ["CDecoder", "load_library", "LIB_PATH"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "liboracle_cpu.so")
_lib = None


def load_library():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle/c` (or __graft_entry__.build())")
        lib = ctypes.CDLL(LIB_PATH)
        p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        lib.oc_affine_linear.argtypes = [p, i, p, p, p, i, i, i, i, p]
        lib.oc_w8a16.argtypes = [p, i, p, p, i, i, p]
        lib.oc_sdpa_int8.argtypes = [p, p, p, p, p, i, i, i, i, i, i, f, p]
        lib.oc_bf16_argmax.argtypes = [p, i, p, i, i, p, p]
        lib.oc_bf16_logits.argtypes = [p, i, p, i, i, p]
        lib.oc_threads.restype = i
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class CDecoder:
    """``weights`` (raw formats): per layer qkv_w int8, qkv_s f32, o_w int8, o_s f32,
    gate/up/down = (packed uint32, scale bits uint16, bias bits uint16),
    in_norm/post_norm f32; embed_bits/head_bits uint16 [V, H]; final_norm f32."""

    def __init__(self, weights, *, num_heads, num_kv_heads, head_dim, rope_theta, eps, group, capacity, batch):
        self.lib = load_library()
        self.w = weights
        self.hq, self.hkv, self.d = num_heads, num_kv_heads, head_dim
        self.theta, self.eps, self.group = rope_theta, eps, group
        self.capacity = capacity
        layers = len(weights["layers"])
        self.kq = np.zeros((layers, batch, num_kv_heads, capacity, head_dim), np.int8)
        self.vq = np.zeros_like(self.kq)
        self.ks = np.ones((layers, batch, num_kv_heads, capacity), np.float16)
        self.vs = np.ones_like(self.ks)

    def _affine(self, x, tri):
        packed, s_bits, b_bits = tri
        n = packed.shape[0]
        k = x.shape[1]
        y = np.empty((x.shape[0], n), np.float32)
        self.lib.oc_affine_linear(_p(np.ascontiguousarray(x, np.float32)), x.shape[0], _p(packed), _p(s_bits),
                                  _p(b_bits), n, k, self.group, 4, _p(y))
        return y

    def _w8(self, x, w, s):
        y = np.empty((x.shape[0], w.shape[0]), np.float32)
        self.lib.oc_w8a16(_p(np.ascontiguousarray(x, np.float32)), x.shape[0], _p(w), _p(s), w.shape[0],
                          w.shape[1], _p(y))
        return y

    def prefill_chunk(self, tokens, start, *, want_argmax=False):
        """Feed consecutive tokens of sequence 0 at positions start..start+c-1
        (c <= 8) through the layers in one pass over the weights.

        Row r is the decode step of position start + r: the same arithmetic
        and bf16 rounding points as ``step`` (every GEMV row is computed
        independently), attention causal over positions <= start + r. Returns
        the greedy next token after the last row when ``want_argmax``."""
        w = self.w
        toks = np.asarray(tokens).reshape(-1)
        c = toks.shape[0]
        if not 1 <= c <= 8:
            raise ValueError("chunks of 1 to 8 tokens")
        x = bf16_from_bits(w["embed_bits"][toks])
        d = self.d
        pos = np.arange(start, start + c)
        for li, layer in enumerate(w["layers"]):
            xn = round_bf16(ops.rms_norm(x, layer["in_norm"], self.eps))
            qkv = round_bf16(self._w8(xn, layer["qkv_w"], layer["qkv_s"]))
            q = qkv[:, : self.hq * d].reshape(c, self.hq, 1, d)
            k = qkv[:, self.hq * d:(self.hq + self.hkv) * d].reshape(c, self.hkv, 1, d)
            v = qkv[:, (self.hq + self.hkv) * d:].reshape(c, self.hkv, 1, d)
            q = round_bf16(ops.rope(q, pos.reshape(c, 1, 1), d, self.theta))
            k = round_bf16(ops.rope(k, pos.reshape(c, 1, 1), d, self.theta))
            kq, ks = quantize_kv_symmetric(k[:, :, 0])
            vq, vs = quantize_kv_symmetric(v[:, :, 0])
            self.kq[li, 0, :, start:start + c] = kq.transpose(1, 0, 2)
            self.ks[li, 0, :, start:start + c] = ks.T
            self.vq[li, 0, :, start:start + c] = vq.transpose(1, 0, 2)
            self.vs[li, 0, :, start:start + c] = vs.T
            out = np.empty((c, self.hq, d), np.float32)
            for r in range(c):
                qr = np.ascontiguousarray(q[r, :, 0], np.float32)
                self.lib.oc_sdpa_int8(_p(qr), _p(self.kq[li]), _p(self.ks[li].view(np.uint16)), _p(self.vq[li]),
                                      _p(self.vs[li].view(np.uint16)), 1, self.hq, self.hkv, start + r + 1,
                                      self.capacity, d, float(1.0 / np.sqrt(d)), _p(out[r]))
            attn = round_bf16(out.reshape(c, self.hq * d))
            o = round_bf16(self._w8(attn, layer["o_w"], layer["o_s"]))
            x = round_bf16(x + o)
            xn = round_bf16(ops.rms_norm(x, layer["post_norm"], self.eps))
            g = round_bf16(self._affine(xn, layer["gate"]))
            u = round_bf16(self._affine(xn, layer["up"]))
            act = round_bf16(ops.swiglu(g, u))
            x = round_bf16(x + round_bf16(self._affine(act, layer["down"])))
        self.last_x = x
        if not want_argmax:
            return None
        return self._head(x[-1:])[0]

    def _head(self, x):
        """RMSNorm + bf16 lm_head of rows x: greedy tokens (lowest index on
        ties); the fp32 logits stay in ``last_logits`` for margin diagnostics."""
        w = self.w
        xn = np.ascontiguousarray(round_bf16(ops.rms_norm(x, w["final_norm"], self.eps)), np.float32)
        head = w["head_bits"]
        bsz = xn.shape[0]
        logits = np.empty((bsz, head.shape[0]), np.float32)
        self.lib.oc_bf16_logits(_p(xn), bsz, _p(head), head.shape[0], head.shape[1], _p(logits))
        self.last_logits = logits
        return np.argmax(logits, axis=-1).astype(np.int32)

    def layer(self, li, x, position):
        """Decoder layer ``li`` for hidden states x [B, H] (bf16 values) at
        ``position``: appends the new K/V rows to the cache and returns the
        layer's output residual stream (the loop body of ``step``)."""
        return self._layers(x, position, li, li + 1)

    def head(self, x):
        """Final RMSNorm + lm_head + greedy argmax of hidden states x [B, H]
        (logits kept in ``last_logits``)."""
        self.last_x = x
        return self._head(x)

    def step(self, tokens, position):
        """One decode step; returns the greedy next tokens [B]."""
        w = self.w
        x = bf16_from_bits(w["embed_bits"][np.asarray(tokens)])
        x = self._layers(x, position, 0, len(w["layers"]))
        self.last_x = x
        return self._head(x)

    def _layers(self, x, position, l0, l1):
        w = self.w
        bsz = x.shape[0]
        d = self.d
        for li in range(l0, l1):
            layer = w["layers"][li]
            xn = round_bf16(ops.rms_norm(x, layer["in_norm"], self.eps))
            qkv = round_bf16(self._w8(xn, layer["qkv_w"], layer["qkv_s"]))
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
            out = np.empty((bsz, self.hq, d), np.float32)
            self.lib.oc_sdpa_int8(_p(np.ascontiguousarray(q[:, :, 0], np.float32)), _p(self.kq[li]),
                                  _p(self.ks[li].view(np.uint16)), _p(self.vq[li]), _p(self.vs[li].view(np.uint16)),
                                  bsz, self.hq, self.hkv, position + 1, self.capacity, d,
                                  float(1.0 / np.sqrt(d)), _p(out))
            attn = round_bf16(out.reshape(bsz, self.hq * d))
            o = round_bf16(self._w8(attn, layer["o_w"], layer["o_s"]))
            x = round_bf16(x + o)
            xn = round_bf16(ops.rms_norm(x, layer["post_norm"], self.eps))
            g = round_bf16(self._affine(xn, layer["gate"]))
            u = round_bf16(self._affine(xn, layer["up"]))
            act = round_bf16(ops.swiglu(g, u))
            x = round_bf16(x + round_bf16(self._affine(act, layer["down"])))
        return x
