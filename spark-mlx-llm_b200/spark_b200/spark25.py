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
rotating cache of ``sliding_window`` slots), ``sb_int8_sdpa_decode`` (head_dim
128 or 256; a sliding layer attends to its ring's filled slots),
``sb_head_gate``, the residual epilogue of ``out_proj``, the paired gate/up GEMV
with the fused RMSNorm and GELU gate, ``down`` with its residual, and the
final RMSNorm fused into the (tied, quantized) lm_head GEMV. KV: the BASELINE
symmetric INT8 format (one fp16 scale per token and head) instead of the
reference's bf16 or affine uint8/G32 cache. Sliding layers keep the
RotatingKVCache of ``model.py:362-370`` (``max_size=sliding_window, keep=0``):
position p lands in slot p % window, so the slots always hold the last
``window`` positions (``rotating=False`` instead keeps every position and moves
the attention start, the same keys in position order).
"""

import ctypes
import math
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ._lib import check, lib, sb_linear_ex_desc
from .checkpoint import load_checkpoint_dir, to_torch

__all__ = ["Spark25Config", "Spark25Model", "load", "sanitize"]

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
    """A loaded Spark2_5 checkpoint with its INT8 KV cache and decode buffers;
    ``step(tokens)`` runs one greedy-decode position for ``batch`` sequences."""

    def __init__(self, cfg, weights, *, batch=1, capacity=None, device="cuda", rotating=True):
        self.cfg, self.batch = cfg, batch
        self.rotating = rotating
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
        # rows per head: a sliding layer's ring holds sliding_window slots (rows rounded to 16)
        ring = (cfg.sliding_window + 15) // 16 * 16
        self.rows = [min(ring, self.capacity) if lay["sliding"] and self.rotating else self.capacity
                     for lay in self.layers]
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
            rotating = lay["sliding"] and self.rotating
            args = (_ptr(self.qkv), self.qkv.shape[1], _ptr(self.positions), _ptr(self.q), _ptr(kc), _ptr(ks),
                    _ptr(vc), _ptr(vs), b, 1, hq, hkv, d, rows, lay["rope_dims"], lay["rope_base"])
            if rotating:  # the ring's slots hold the last sliding_window positions
                check(L.sb_rope_kv_append_ring(*args, cfg.sliding_window, stream), "rope + ring cache append")
                start, n = 0, min(length, cfg.sliding_window)
            else:
                check(L.sb_rope_kv_append(*args, stream), "rope + cache append")
                # a sliding layer attends to its last sliding_window positions:
                # the same cache rows with the start moved (row stride unchanged)
                start = max(0, length - cfg.sliding_window) if lay["sliding"] else 0
                n = length - start
            check(L.sb_int8_sdpa_decode(_ptr(self.q), kc.data_ptr() + start * d, ks.data_ptr() + 2 * start,
                                        vc.data_ptr() + start * d, vs.data_ptr() + 2 * start, _ptr(self.attn), b, hq,
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

    def prefill(self, prompt):
        """Run ``prompt [batch, L]`` position by position; returns the last logits."""
        prompt = torch.as_tensor(prompt, dtype=torch.int32)
        if prompt.ndim != 2 or prompt.shape[0] != self.batch:
            raise ValueError("prompt must be [batch, L]")
        logits = None
        for i in range(prompt.shape[1]):
            logits = self.step(prompt[:, i])
        return logits

    def generate(self, prompt, steps):
        """Greedy decode: the ``steps`` tokens after ``prompt`` ([batch, steps], host)."""
        logits = self.prefill(prompt)
        out = []
        for _ in range(steps):
            tok = torch.argmax(logits.float(), dim=-1).to(torch.int32)
            out.append(tok)
            logits = self.step(tok)
        return torch.stack(out, dim=1).cpu()


def load(path, *, batch=1, capacity=None, device="cuda", rotating=True,
         model_config: Optional[dict[str, Any]] = None):
    """Load a Spark2_5 MLX-affine checkpoint directory (``loader.load``,
    ``spark_mlx_llm/loader.py:65-120``: ``config.json`` + ``model*.safetensors``)."""
    config, weights = load_checkpoint_dir(path)
    config = dict(config, **(model_config or {}))
    cfg = Spark25Config.from_dict(config)
    return Spark25Model(cfg, weights, batch=batch, capacity=capacity, device=device, rotating=rotating)
