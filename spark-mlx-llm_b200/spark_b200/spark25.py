"""Spark2_5 checkpoints (MLX-affine safetensors) on this library's kernels.

The reference model (``spark_mlx_llm/model.py``) loaded from an MLX checkpoint
directory (``spark_mlx_llm/loader.py:65-120``) and run as a greedy decoder:

    x = embedding(token)                                   (model.py:291-294)
    per layer (TransformerBlock.__call__, model.py:249-262):
        xn  = rms_norm(x, input_layernorm)
        q, k, v = split(q_k_v_proj(xn)); RoPE on q, k      (ops/qkv.py:18-87; partial rotary)
        cache.update(k, v); o = sdpa(q, K, V)              (sliding layers: the last sliding_window keys)
        o  = o * sigmoid(xn @ g_proj^T) per head           (ops/attention_output.py:91-95)
        h  = x + out_proj(o)                               (ops/ffn.py:98)
        x  = h + down(gelu(gate(rms_norm(h))) * up(...))   (ops/ffn.py:98-103)
    logits = embedding.as_linear(rms_norm(x, norm))        (tied; model.py:326-333)

Per token and layer this runs ``sb_rms_norm``, the weight-streaming affine GEMV
(``sb_linear_ex``: 4- or 8-bit, groups 32/64/128, any projection shape),
``sb_rope_kv_append`` (RoPE on the first rope_dims features, K/V quantized into
the BASELINE INT8 cache; ``sb_rope_kv_append_ring`` for a sliding layer's
rotating cache), ``sb_int8_sdpa_decode`` (head_dim 128 or 256; a sliding layer
attends to its last ``sliding_window`` positions),
``sb_head_gate``, the residual epilogue of ``out_proj``, the paired gate/up GEMV
with the fused RMSNorm and GELU gate, ``down`` with its residual, and the
final RMSNorm fused into the (tied, quantized) lm_head GEMV. KV: the BASELINE
symmetric INT8 format (one fp16 scale per token and head) instead of the
reference's bf16 or affine uint8/G32 cache. Sliding layers keep a rotating
cache like the RotatingKVCache of ``model.py:362-370`` (``keep=0``): a ring of
R = sliding_window + chunk - 1 slots (rounded up to 16), position p in slot
p % R, and every slot written twice - at row p % R and at its mirror row
p % R + R - so the last ``n <= R`` positions are always one contiguous run of
rows, in position order: a decode query attends to rows
[(length - n) % R, ... + n) with n = min(length, sliding_window), and a prompt
chunk to the sliding_window - 1 positions before it plus itself. (The
reference's ring of exactly ``sliding_window`` slots is the case chunk = 1; a
ring that would not be smaller than the cache becomes a linear cache.
``rotating=False`` keeps every position and moves the attention start.)

``prefill`` runs a prompt in chunks of ``chunk`` positions (512, the reference's
prompt chunk, ``generation.py:78``) as one batched pass per layer: embedding
rows, ``sb_rms_norm``, ``sb_affine_linear`` at M = batch x chunk (the
tensor-core kernel beyond 8 rows), ``sb_rope_kv_append`` (ring) for the chunk,
``sb_int8_sdpa_prefill_window`` (bottom-right causal, the sliding window on
sliding layers), ``sb_head_gate``, the residual adds and ``sb_gated_activation``
(GELU); the lm_head runs on the last position only.
"""

import ctypes
import math
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ._lib import check, lib, sb_linear_ex_desc
from .checkpoint import load_checkpoint_dir, to_torch

__all__ = ["Spark25Config", "Spark25Model", "load", "ring_slots", "sanitize"]

BF16 = 0
AFFINE4, AFFINE8, BF16_W = 0, 1, 3
EPI_STORE, EPI_RESID, EPI_SWIGLU = 0, 1, 2


@dataclass
class Spark25Config:
    """``ModelArgs`` of the reference (``model.py:30-127``) with its checks."""
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    sliding_window: int
    rope_parameters: dict
    layer_types: Optional[list] = None
    rms_norm_eps: float = 1e-6
    max_position_embeddings: int = 8192
    attention_bias: bool = False
    mlp_bias: bool = False
    hidden_act: str = "gelu"
    gate_attn_act_mode: str = "sigmoid"
    headwise_attn_output_gate: bool = True
    tie_word_embeddings: bool = True
    extra: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, params):
        """Build and validate from a ``config.json`` dict (unknown keys kept in ``extra``)."""
        if params.get("model_type") != "spark2_5":
            raise ValueError(f"Expected model_type 'spark2_5', got {params.get('model_type')!r}")
        known = {f for f in cls.__dataclass_fields__ if f != "extra"}
        cfg = cls(**{k: v for k, v in params.items() if k in known},
                  extra={k: v for k, v in params.items() if k not in known})
        cfg.validate()
        return cfg

    def validate(self):
        for name in ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                     "num_key_value_heads", "head_dim", "vocab_size", "sliding_window", "max_position_embeddings"):
            value = getattr(self, name)
            if type(value) is not int or value <= 0:
                raise ValueError(f"{name} must be a positive integer")
        if self.layer_types is None:
            pattern = ["sliding_attention"] * 3 + ["full_attention"]
            self.layer_types = [pattern[i % 4] for i in range(self.num_hidden_layers)]
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("layer_types length must match num_hidden_layers: "
                             f"{len(self.layer_types)} != {self.num_hidden_layers}")
        unsupported = set(self.layer_types) - {"sliding_attention", "full_attention"}
        if unsupported:
            raise ValueError(f"Unsupported layer types: {sorted(unsupported)}")
        missing = set(self.layer_types) - set(self.rope_parameters)
        if missing:
            raise ValueError(f"Missing RoPE parameters for layer types: {sorted(missing)}")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        for layer_type in set(self.layer_types):
            dims = self.rope(layer_type)[0]
            if dims <= 0 or dims > self.head_dim or dims % 2:
                raise ValueError(f"Invalid rotary dimension {dims} for {layer_type} with head_dim={self.head_dim}")
        if self.hidden_act != "gelu":
            raise ValueError(f"Spark2_5 requires GELU, got {self.hidden_act!r}")
        if not self.headwise_attn_output_gate:
            raise ValueError("Spark2_5 requires head-wise attention output gates")
        if self.gate_attn_act_mode != "sigmoid":
            raise ValueError(f"Spark2_5 requires sigmoid attention gates, got {self.gate_attn_act_mode!r}")
        if self.attention_bias or self.mlp_bias:
            raise ValueError("projection biases are not supported by this runner")
        if self.head_dim not in (128, 256):
            raise ValueError("head_dim must be 128 or 256 (the INT8 attention kernel's sizes)")
        g = self.num_attention_heads // self.num_key_value_heads
        if g not in (1, 2, 4, 8):
            raise ValueError("query heads per KV head must be 1, 2, 4 or 8")

    def rope(self, layer_type):
        """``(rotary dims, base)`` of a layer type (``model.py:162-170``)."""
        params = self.rope_parameters[layer_type]
        dims = int(self.head_dim * float(params.get("partial_rotary_factor", 1.0)))
        return dims, float(params.get("rope_theta", 10000.0))


def sanitize(weights, tie_word_embeddings=True):
    """``Model.sanitize`` (``model.py:378-396``): ``embed_tokens`` renamed to
    ``embedding``, the tied ``lm_head`` and serialized RoPE buffers dropped."""
    weights = dict(weights)
    for suffix in ("weight", "scales", "biases"):
        old, new = f"model.embed_tokens.{suffix}", f"model.embedding.{suffix}"
        if old in weights and new not in weights:
            weights[new] = weights.pop(old)
    if tie_word_embeddings:
        for suffix in ("weight", "scales", "biases"):
            weights.pop(f"lm_head.{suffix}", None)
    return {k: v for k, v in weights.items() if "rotary_emb.inv_freq" not in k}


def _ptr(t):
    return t.data_ptr() if t is not None else None


def ring_slots(window, chunk, capacity):
    """Slots R of a sliding layer's ring for prompt chunks of up to ``chunk``
    positions: a chunk attends to the window - 1 positions before it and itself,
    so R >= window + chunk - 1 keeps all of them (rounded up to 16 rows). 0 (a
    linear cache) when the mirrored ring (2R rows) would not be smaller than
    ``capacity``."""
    r = (window + chunk - 1 + 15) // 16 * 16
    return r if 2 * r < capacity else 0


class _Proj:
    """One linear layer: MLX affine (packed uint32 + bf16 scales/biases) or bf16."""

    def __init__(self, weights, name, in_features, out_features, device):
        w = weights.get(f"{name}.weight")
        if w is None:
            raise ValueError(f"missing tensor {name}.weight")
        self.n, self.k = out_features, in_features
        if f"{name}.scales" in weights:
            dt, arr = w
            if dt not in ("U32", "I32") or arr.ndim != 2 or arr.shape[0] != out_features:
                raise ValueError(f"{name}.weight: expected packed uint32 [{out_features}, K*bits/32]")
            bits = arr.shape[1] * 32 // in_features
            sdt, sarr = weights[f"{name}.scales"]
            if bits not in (4, 8) or arr.shape[1] * 32 != bits * in_features:
                raise ValueError(f"{name}: unsupported affine bits (packed width {arr.shape[1]})")
            if sdt != "BF16" or weights[f"{name}.biases"][0] != "BF16":
                raise ValueError(f"{name}: scales and biases must be bfloat16")
            if sarr.shape != (out_features, sarr.shape[1]) or in_features % sarr.shape[1]:
                raise ValueError(f"{name}.scales: bad shape {sarr.shape}")
            self.group = in_features // sarr.shape[1]
            if self.group not in (32, 64, 128):
                raise ValueError(f"{name}: group size {self.group} is not 32, 64 or 128")
            self.bits = bits
            self.format = AFFINE4 if bits == 4 else AFFINE8
            self.weight = to_torch(w, device)
            self.scales = to_torch(weights[f"{name}.scales"], device)
            self.biases = to_torch(weights[f"{name}.biases"], device)
        else:
            dt, arr = w
            if dt != "BF16" or arr.shape != (out_features, in_features):
                raise ValueError(f"{name}.weight: expected bf16 [{out_features}, {in_features}] or an affine triple")
            self.bits, self.group, self.format = 16, 0, BF16_W
            self.weight, self.scales, self.biases = to_torch(w, device), None, None

    def desc(self, **kw):
        d = sb_linear_ex_desc(weight_format=self.format, weight=_ptr(self.weight), scales=_ptr(self.scales),
                              biases=_ptr(self.biases), group_size=self.group, N=self.n, K=self.k, x_dtype=BF16,
                              weights_constant=1)
        for key, value in kw.items():
            setattr(d, key, value)
        return d


class Spark25Model:
    """A loaded Spark2_5 checkpoint with its INT8 KV cache and decode buffers.
    ``prefill(prompt)`` runs a prompt in chunks of up to ``chunk`` positions
    (the sliding layers' rings are sized for it), ``step(tokens)`` one
    greedy-decode position for ``batch`` sequences."""

    def __init__(self, cfg, weights, *, batch=1, capacity=None, device="cuda", rotating=True, chunk=512):
        self.cfg, self.batch = cfg, batch
        self.rotating = rotating
        if chunk < 1:
            raise ValueError("chunk must be positive")
        self.chunk = int(chunk)
        self.device = torch.device(device)
        self.capacity = ((capacity or cfg.max_position_embeddings) + 15) // 16 * 16
        weights = sanitize(weights, cfg.tie_word_embeddings)
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        hid, inter = cfg.hidden_size, cfg.intermediate_size
        dev = self.device
        self.embed = _Proj(weights, "model.embedding", hid, cfg.vocab_size, dev)
        self.head = self.embed if cfg.tie_word_embeddings else _Proj(weights, "lm_head", hid, cfg.vocab_size, dev)

        def vec(name, n):
            dt, arr = weights[name]
            if dt != "BF16" or arr.shape != (n,):
                raise ValueError(f"{name}: expected bf16 [{n}]")
            return to_torch(weights[name], dev)

        self.final_norm = vec("model.norm.weight", hid)
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}"
            gdt, garr = weights[f"{p}.self_attn.g_proj.weight"]
            if gdt != "BF16" or garr.shape != (hq, hid):
                raise ValueError(f"{p}.self_attn.g_proj.weight: expected bf16 [{hq}, {hid}]")
            dims, base = cfg.rope(cfg.layer_types[i])
            self.layers.append(dict(
                in_norm=vec(f"{p}.input_layernorm.weight", hid),
                post_norm=vec(f"{p}.post_attention_layernorm.weight", hid),
                qkv=_Proj(weights, f"{p}.self_attn.q_k_v_proj", hid, (hq + 2 * hkv) * d, dev),
                g=to_torch(weights[f"{p}.self_attn.g_proj.weight"], dev),
                out=_Proj(weights, f"{p}.self_attn.out_proj", hq * d, hid, dev),
                gate=_Proj(weights, f"{p}.mlp.gate_proj", hid, inter, dev),
                up=_Proj(weights, f"{p}.mlp.up_proj", hid, inter, dev),
                down=_Proj(weights, f"{p}.mlp.down_proj", inter, hid, dev),
                sliding=cfg.layer_types[i] == "sliding_attention", rope_dims=dims, rope_base=base))
            lay = self.layers[-1]
            if not (lay["gate"].format == lay["up"].format and lay["gate"].group == lay["up"].group
                    and lay["gate"].format != BF16_W):
                raise ValueError(f"{p}.mlp: gate_proj and up_proj must share one affine format")
            for proj in ("qkv", "out", "down"):
                if lay[proj].format == BF16_W:
                    raise ValueError(f"{p}: {proj} must be affine-quantized (4 or 8 bit)")
        self._alloc()
        self.pos = 0

    # ------------------------------------------------------------------ state
    def _alloc(self):
        cfg, b, dev = self.cfg, self.batch, self.device
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(b, cfg.hidden_size, **bf)
        self.xn = torch.zeros_like(self.x)
        self.h = torch.zeros_like(self.x)
        self.qkv = torch.zeros(b, (hq + 2 * hkv) * d, **bf)
        self.q = torch.zeros(b, hq, 1, d, **bf)
        self.attn = torch.zeros(b, hq * d, **bf)
        self.gated = torch.zeros_like(self.attn)
        self.act = torch.zeros(b, cfg.intermediate_size, **bf)
        self.logits = torch.zeros(b, cfg.vocab_size, **bf)
        self.tokens = torch.zeros(b, dtype=torch.int32, device=dev)
        self.positions = torch.zeros(b, dtype=torch.int32, device=dev)
        # rows per head: a sliding layer's ring of R slots is stored twice (rows [0, R) and
        # the mirror [R, 2R)); a ring no smaller than the cache is a linear cache instead
        ring = ring_slots(cfg.sliding_window, self.chunk, self.capacity) if self.rotating else 0
        self.ring = [ring if lay["sliding"] else 0 for lay in self.layers]
        self.rows = [2 * r if r else self.capacity for r in self.ring]
        self.k_cache = [torch.zeros(b, hkv, r, d, dtype=torch.int8, device=dev) for r in self.rows]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.k_scale = [torch.ones(b, hkv, r, dtype=torch.float16, device=dev) for r in self.rows]
        self.v_scale = [torch.ones_like(s) for s in self.k_scale]
        ws = lib().sb_int8_sdpa_workspace_size(b, hq, hkv, self.capacity, d)
        descs = []
        for lay in self.layers:
            lay["qkv_d"] = lay["qkv"].desc(x=_ptr(self.xn), M=b, epilogue=EPI_STORE, y=_ptr(self.qkv))
            lay["out_d"] = lay["out"].desc(x=_ptr(self.gated), M=b, epilogue=EPI_RESID, y=_ptr(self.h),
                                           residual=_ptr(self.x))
            g, u = lay["gate"], lay["up"]
            lay["gu_d"] = g.desc(x=_ptr(self.h), M=b, epilogue=EPI_SWIGLU, y=_ptr(self.act),
                                 weight2=_ptr(u.weight), scales2=_ptr(u.scales), biases2=_ptr(u.biases),
                                 norm_weight=_ptr(lay["post_norm"]), norm_eps=self.cfg.rms_norm_eps, activation=1)
            lay["down_d"] = lay["down"].desc(x=_ptr(self.act), M=b, epilogue=EPI_RESID, y=_ptr(self.x),
                                             residual=_ptr(self.h))
            descs += [lay["qkv_d"], lay["out_d"], lay["gu_d"], lay["down_d"]]
        self.head_d = self.head.desc(x=_ptr(self.x), M=b, epilogue=EPI_STORE, y=_ptr(self.logits),
                                     norm_weight=_ptr(self.final_norm), norm_eps=self.cfg.rms_norm_eps)
        descs.append(self.head_d)
        sizes = [lib().sb_linear_ex_workspace_size(ctypes.byref(dd)) for dd in descs] + [ws]
        self.workspace = torch.zeros(max(sizes) + 256, dtype=torch.uint8, device=dev)
        for dd in descs:
            dd.workspace, dd.workspace_bytes = self.workspace.data_ptr(), self.workspace.numel()

    def reset(self):
        """Empty the cache (position 0)."""
        self.pos = 0

    # ------------------------------------------------------------------ decode
    def step(self, tokens):
        """Feed one token per sequence at the current position; returns the
        logits ``[batch, vocab]`` bf16 (device) and advances the position."""
        cfg, b, L = self.cfg, self.batch, lib()
        if self.pos >= self.capacity:
            raise ValueError("KV cache is full")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).to(self.device))
        self.positions.fill_(self.pos)
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        e = self.embed
        if e.format == BF16_W:
            check(L.sb_embed_rows(_ptr(e.weight), _ptr(self.tokens), _ptr(self.x), b, cfg.hidden_size,
                                  cfg.vocab_size, stream), "embedding")
        else:
            check(L.sb_embed_rows_affine(_ptr(e.weight), _ptr(e.scales), _ptr(e.biases), _ptr(self.tokens),
                                         _ptr(self.x), b, cfg.hidden_size, cfg.vocab_size, e.group, e.bits, stream),
                  "embedding")
        scale = 1.0 / math.sqrt(d)
        length = self.pos + 1
        for li, lay in enumerate(self.layers):
            check(L.sb_rms_norm(_ptr(self.x), _ptr(lay["in_norm"]), _ptr(self.xn), BF16, b, cfg.hidden_size,
                                cfg.rms_norm_eps, stream), "input_layernorm")
            check(L.sb_linear_ex(ctypes.byref(lay["qkv_d"]), stream), "q_k_v_proj")
            kc, vc, ks, vs = self.k_cache[li], self.v_cache[li], self.k_scale[li], self.v_scale[li]
            rows = self.rows[li]
            self._append(li, _ptr(self.qkv), self.qkv.shape[1], _ptr(self.positions), _ptr(self.q), 1, stream)
            # a sliding layer attends to its last sliding_window positions: one
            # contiguous run of rows (row stride unchanged)
            start = max(0, length - cfg.sliding_window) if lay["sliding"] else 0
            n, row0 = length - start, self._row(li, start)
            check(L.sb_int8_sdpa_decode(_ptr(self.q), kc.data_ptr() + row0 * d, ks.data_ptr() + 2 * row0,
                                        vc.data_ptr() + row0 * d, vs.data_ptr() + 2 * row0, _ptr(self.attn), b, hq,
                                        hkv, n, rows, d, scale, self.workspace.data_ptr(),
                                        self.workspace.numel(), stream), "attention")
            check(L.sb_head_gate(_ptr(self.xn), _ptr(lay["g"]), _ptr(self.attn), _ptr(self.gated), b,
                                 cfg.hidden_size, hq, d, stream), "head gate")
            check(L.sb_linear_ex(ctypes.byref(lay["out_d"]), stream), "out_proj + residual")
            check(L.sb_linear_ex(ctypes.byref(lay["gu_d"]), stream), "norm + gate/up + gelu")
            check(L.sb_linear_ex(ctypes.byref(lay["down_d"]), stream), "down_proj + residual")
        check(L.sb_linear_ex(ctypes.byref(self.head_d), stream), "norm + lm_head")
        self.pos += 1
        return self.logits

    def _row(self, li, position):
        """Cache row of ``position`` in layer ``li`` (its ring slot, or the position)."""
        r = self.ring[li]
        return position % r if r else position

    def _append(self, li, qkv, ld, positions, q_out, seq_len, stream):
        """RoPE + INT8 append of ``seq_len`` positions per sequence into layer
        ``li``'s cache: at the positions (linear) or at their ring slots and the
        slots' mirror rows (the same values written twice)."""
        cfg, L = self.cfg, lib()
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        lay, r = self.layers[li], self.ring[li]
        kc, vc, ks, vs = self.k_cache[li], self.v_cache[li], self.k_scale[li], self.v_scale[li]
        tail = (self.batch, seq_len, hq, hkv, d, self.rows[li], lay["rope_dims"], lay["rope_base"])
        if not r:
            check(L.sb_rope_kv_append(qkv, ld, positions, q_out, _ptr(kc), _ptr(ks), _ptr(vc), _ptr(vs), *tail,
                                      stream), "rope + cache append")
            return
        for m in (0, r):  # the ring rows, then their mirrors
            check(L.sb_rope_kv_append_ring(qkv, ld, positions, q_out, kc.data_ptr() + m * d, ks.data_ptr() + 2 * m,
                                           vc.data_ptr() + m * d, vs.data_ptr() + 2 * m, *tail, r, stream),
                  "rope + ring cache append")

    def _prefill_buffers(self, m):
        """Activation buffers for ``m`` prompt rows (kept; grown on demand)."""
        have = getattr(self, "_pf", None)
        if have is not None and have["rows"] >= m:
            return have
        cfg, dev = self.cfg, self.device
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        hid, inter = cfg.hidden_size, cfg.intermediate_size

        def buf(*shape):
            return torch.empty(shape, dtype=torch.bfloat16, device=dev)

        ws = 256
        for lay in self.layers:
            for proj in ("qkv", "out", "gate", "up", "down"):
                pr = lay[proj]
                ws = max(ws, lib().sb_affine_linear_workspace_size(m, pr.n, pr.k, pr.group, pr.bits))
        self._pf = dict(rows=m, x=buf(m, hid), xn=buf(m, hid), qkv=buf(m, (hq + 2 * hkv) * d), q=buf(m, hq * d),
                        attn=buf(m, hq * d), o=buf(m, hid), g=buf(m, inter), u=buf(m, inter), act=buf(m, inter),
                        ids=torch.empty(m, dtype=torch.int32, device=dev),
                        pos=torch.empty(m, dtype=torch.int32, device=dev),
                        ws=torch.zeros(ws, dtype=torch.uint8, device=dev))
        return self._pf

    def _linear(self, proj, x, y, m, t, stream, what):
        check(lib().sb_affine_linear(_ptr(x), BF16, _ptr(proj.weight), _ptr(proj.scales), _ptr(proj.biases),
                                     _ptr(y), m, proj.n, proj.k, proj.group, proj.bits, t["ws"].data_ptr(),
                                     t["ws"].numel(), stream), what)

    def _prefill_chunk(self, ids, c0, lc, t, stream):
        """Every layer for the tokens ``ids [batch, lc]`` at positions c0..c0+lc-1;
        returns the hidden rows [batch * lc, hidden] (a view of ``t``)."""
        cfg, b, L = self.cfg, self.batch, lib()
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        hid, inter, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
        m = b * lc
        x, xn, qkv, q, attn, o = (t[k][:m] for k in ("x", "xn", "qkv", "q", "attn", "o"))
        g, u, act, tok, pos = (t[k][:m] for k in ("g", "u", "act", "ids", "pos"))
        tok.copy_(ids.reshape(-1))
        pos.copy_(torch.arange(c0, c0 + lc, dtype=torch.int32).repeat(b))
        e = self.embed
        if e.format == BF16_W:
            check(L.sb_embed_rows(_ptr(e.weight), _ptr(tok), _ptr(x), m, hid, cfg.vocab_size, stream), "embedding")
        else:
            check(L.sb_embed_rows_affine(_ptr(e.weight), _ptr(e.scales), _ptr(e.biases), _ptr(tok), _ptr(x), m,
                                         hid, cfg.vocab_size, e.group, e.bits, stream), "embedding")
        scale = 1.0 / math.sqrt(d)
        for li, lay in enumerate(self.layers):
            check(L.sb_rms_norm(_ptr(x), _ptr(lay["in_norm"]), _ptr(xn), BF16, m, hid, eps, stream),
                  "input_layernorm")
            self._linear(lay["qkv"], xn, qkv, m, t, stream, "q_k_v_proj")
            self._append(li, _ptr(qkv), qkv.shape[1], _ptr(pos), _ptr(q), lc, stream)
            # keys: the sliding_window - 1 positions before the chunk (sliding) or
            # every earlier position, then the chunk; one contiguous run of rows
            start = max(0, c0 - cfg.sliding_window + 1) if lay["sliding"] else 0
            n, row0 = c0 + lc - start, self._row(li, start)
            kc, vc, ks, vs = self.k_cache[li], self.v_cache[li], self.k_scale[li], self.v_scale[li]
            check(L.sb_int8_sdpa_prefill_window(_ptr(q), kc.data_ptr() + row0 * d, ks.data_ptr() + 2 * row0,
                                                vc.data_ptr() + row0 * d, vs.data_ptr() + 2 * row0, _ptr(attn), b,
                                                hq, hkv, lc, n, self.rows[li], d, scale,
                                                cfg.sliding_window if lay["sliding"] else 0, 1, stream),
                  "prefill attention")
            check(L.sb_head_gate(_ptr(xn), _ptr(lay["g"]), _ptr(attn), _ptr(attn), m, hid, hq, d, stream),
                  "head gate")
            self._linear(lay["out"], attn, o, m, t, stream, "out_proj")
            check(L.sb_residual_add(_ptr(x), _ptr(o), m * hid, stream), "residual")
            check(L.sb_rms_norm(_ptr(x), _ptr(lay["post_norm"]), _ptr(xn), BF16, m, hid, eps, stream),
                  "post_attention_layernorm")
            self._linear(lay["gate"], xn, g, m, t, stream, "gate_proj")
            self._linear(lay["up"], xn, u, m, t, stream, "up_proj")
            check(L.sb_gated_activation(_ptr(g), _ptr(u), _ptr(act), m * inter, 1, stream), "gelu gate")
            self._linear(lay["down"], act, o, m, t, stream, "down_proj")
            check(L.sb_residual_add(_ptr(x), _ptr(o), m * hid, stream), "residual")
        return x

    def prefill(self, prompt, chunk=None):
        """Run ``prompt [batch, L]`` from the current position; returns the logits
        after its last position and advances the position by L. The prompt runs
        in chunks of ``chunk`` positions (default: the model's ``chunk``, at most
        it when a sliding layer has a ring); ``chunk=0`` feeds it position by
        position through ``step``."""
        prompt = torch.as_tensor(prompt, dtype=torch.int32)
        if prompt.ndim != 2 or prompt.shape[0] != self.batch or prompt.shape[1] < 1:
            raise ValueError("prompt must be [batch, L] with L >= 1")
        total = prompt.shape[1]
        if chunk == 0:
            logits = None
            for i in range(total):
                logits = self.step(prompt[:, i])
            return logits
        chunk = self.chunk if chunk is None else int(chunk)
        if chunk < 1 or (chunk > self.chunk and any(self.ring)):
            raise ValueError(f"chunk must be in [1, {self.chunk}] (the ring is sized for it)")
        if self.pos + total > self.capacity:
            raise ValueError("KV cache is full")
        b, hid = self.batch, self.cfg.hidden_size
        stream = torch.cuda.current_stream(self.device).cuda_stream
        prompt = prompt.to(self.device)
        t = self._prefill_buffers(b * min(chunk, total))
        for c0 in range(0, total, chunk):
            lc = min(chunk, total - c0)
            x = self._prefill_chunk(prompt[:, c0:c0 + lc], self.pos + c0, lc, t, stream)
        self.x.copy_(x.view(b, lc, hid)[:, lc - 1])
        check(lib().sb_linear_ex(ctypes.byref(self.head_d), stream), "norm + lm_head")
        self.pos += total
        return self.logits

    def generate(self, prompt, steps):
        """Greedy decode: the ``steps`` tokens after ``prompt`` ([batch, steps], host)."""
        logits = self.prefill(prompt)
        out = []
        for _ in range(steps):
            tok = torch.argmax(logits.float(), dim=-1).to(torch.int32)
            out.append(tok)
            logits = self.step(tok)
        return torch.stack(out, dim=1).cpu()


def load(path, *, batch=1, capacity=None, device="cuda", rotating=True, chunk=512,
         model_config: Optional[dict[str, Any]] = None):
    """Load a Spark2_5 MLX-affine checkpoint directory (``loader.load``,
    ``spark_mlx_llm/loader.py:65-120``: ``config.json`` + ``model*.safetensors``)."""
    config, weights = load_checkpoint_dir(path)
    config = dict(config, **(model_config or {}))
    cfg = Spark25Config.from_dict(config)
    return Spark25Model(cfg, weights, batch=batch, capacity=capacity, device=device, rotating=rotating,
                        chunk=chunk)
