"""The ``spark_mlx_llm.ops`` dispatch layer over the B200 kernels.

Mirrors the reference's operator entry points for the decode path:

* ``dispatch_linear(x, projection, *, config=None)``      (ops/linear.py:84-94)
* ``AffineParameters`` (``native``, ``from_module``, ``accepts``) (:97-191)
* ``dispatch_qkv(x, projection, rope, *, q_size, kv_size, n_heads,
  n_kv_heads, head_dim, offset, config=None)``               (ops/qkv.py:18-87)
* ``dispatch_sdpa(queries, keys, values, *, cache, scale, mask, config=None,
  is_sliding=False)``                                        (ops/sdpa.py:39-78)
* ``dispatch_attention_output(x, output, gate_projection, output_projection)``
                                                   (ops/attention_output.py:16-101)
* ``dispatch_ffn(x, attention_output, norm, mlp, *, mlp_type)``  (ops/ffn.py:17-118)

A ``projection`` is any object exposing the MLX ``nn.QuantizedLinear``
attributes ``weight / scales / biases / group_size / bits / mode`` (affine,
no linear bias) holding torch CUDA tensors - :class:`QuantizedLinear` is one -
or a W8 per-channel module (:class:`W8A16PerChannelLinear`,
``ext.W8A8Linear``), or any callable. ``rope`` is an object with the
``nn.RoPE`` attributes ``dims / traditional / base / scale`` (:class:`RoPE`).
KV for ``dispatch_sdpa`` is either the B200 INT8 cache pair ``(int8 codes
[B,KH,N,D], fp16 scales [B,KH,N])`` or the reference's affine tuple
``(packed, scales, biases)``.
"""

import math
from dataclasses import dataclass, fields
from typing import NamedTuple

import torch

from . import ext, ops

__all__ = [
    "AffineParameters",
    "LinearConfig",
    "QuantizedLinear",
    "RoPE",
    "SDPAConfig",
    "PreparedW8",
    "QuantizedProjections",
    "W8A16PerChannelLinear",
    "W8A8Projection",
    "W8MultirowProjection",
    "dispatch_attention_output",
    "dispatch_ffn",
    "dispatch_linear",
    "dispatch_qkv",
    "dispatch_sdpa",
    "unpack_affine_w8",
]


class _Config:
    """Field validation shared by the configs (``spark_mlx_llm/ops/base.py:14-53``,
    ``OperatorConfig``): ``from_dict`` picks this config's fields out of a flat
    model config, ``choices`` gives a field's allowed values, and
    ``validate_values`` checks supplied fields only (booleans must be bool,
    choice fields one of their choices), with the reference's messages."""

    _choices: dict = {}

    def __post_init__(self):
        self.validate()

    @classmethod
    def from_dict(cls, values):
        names = {f.name for f in fields(cls)}
        return cls(**{name: values[name] for name in names if name in values})

    @classmethod
    def choices(cls, name):
        return cls._choices[name]

    @classmethod
    def validate_values(cls, values):
        for f in fields(cls):
            if f.name not in values:
                continue
            value = values[f.name]
            allowed = cls._choices.get(f.name)
            if allowed is None and type(f.default) is bool and type(value) is not bool:
                raise ValueError(f"{f.name} must be a boolean, got {value!r}")
            if allowed is not None and value not in allowed:
                raise ValueError(f"{f.name} must be one of {allowed}, got {value!r}")

    def validate(self):
        self.validate_values({f.name: getattr(self, f.name) for f in fields(self)})


@dataclass(kw_only=True)
class LinearConfig(_Config):
    """Implementation policy for existing W8/W4 layers (ops/linear.py:56-81).

    On B200 every W4/W8 layer runs the same weight-streaming kernel family;
    the backend names are accepted and validated for compatibility."""

    w8_qmv_backend: str = "w8a16"
    w4_qmv_backend: str = "native"
    _choices = {"w8_qmv_backend": ("auto", "native", "w8a16", "w8a8", "multirow"),
                "w4_qmv_backend": ("native", "splitk", "multirow", "multirow_packed")}

    @classmethod
    def validate_values(cls, values):
        if "qmv_backend" in values:
            raise ValueError("qmv_backend was renamed to w8_qmv_backend; update the configuration")
        super().validate_values(values)


@dataclass(kw_only=True)
class SDPAConfig(_Config):
    """Kernel preferences for attention (ops/sdpa.py:13-20)."""

    fused_quantized_sdpa: bool = True
    fused_quantized_sdpa_prefill: bool = False
    tuned_bf16_sdpa: bool = False
    verification_bf16_sdpa: bool = False


class AffineParameters(NamedTuple):
    """Affine tensors and metadata passed explicitly to the projection (ops/linear.py:97-191)."""

    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int
    bits: int

    @classmethod
    def from_module(cls, layer):
        return cls(layer.weight, layer.scales, layer.biases, layer.group_size, layer.bits)

    @staticmethod
    def accepts(layer):
        return (getattr(layer, "mode", None) == "affine" and getattr(layer, "biases", None) is not None
                and getattr(layer, "bias", None) is None and hasattr(layer, "weight") and hasattr(layer, "scales"))

    @staticmethod
    def native(x, weight, scales, biases, group_size, bits):
        """``mx.quantized_matmul(x, w, scales, biases, transpose=True, mode="affine")``."""
        return ops.affine_linear(x, weight, scales, biases, group_size, bits)

    # The reference's W4 backend selection (ops/linear.py:116-257). Its routes
    # are Metal schedules of one computation; here every route is the same
    # weight-streaming kernel family, reached through the entry point the
    # route names (w4a16_qmv, w4a16_multirow), so the choice keeps the
    # reference's conditions and never changes the result's arithmetic.
    @classmethod
    def resolve(cls, layer, shape, dtype, config):
        """``(projection callable, parameters)`` for ``x`` of ``shape``/``dtype``
        under ``config``; ``multirow_packed`` needs no repacking here."""
        params = cls.from_module(layer)
        if config.w4_qmv_backend == "multirow_packed" and params.supports_multirow(shape, dtype, *params):
            return cls.multirow_packed, params
        return params.select(shape, dtype, config), params

    def select(self, shape, dtype, config):
        if config.w4_qmv_backend == "multirow" and self.supports_multirow(shape, dtype, *self):
            return self.multirow
        if config.w4_qmv_backend == "splitk" and self.supports_splitk(shape, dtype, *self):
            return self.splitk
        return self.native

    @staticmethod
    def _w4g32_bf16(shape, dtype, weight, scales, biases, group_size, bits):
        return (bits == 4 and group_size == 32 and len(shape) >= 1 and weight.ndim == 2
                and weight.shape[1] * 8 == shape[-1] and tuple(scales.shape) == (weight.shape[0], shape[-1] // 32)
                and biases is not None and biases.shape == scales.shape
                and dtype == scales.dtype == biases.dtype == torch.bfloat16
                and weight.dtype in (torch.int32, torch.uint32) and _on_gpu(weight))

    @staticmethod
    def supports_splitk(shape, dtype, weight, scales, biases, group_size, bits):
        """One BF16 row of a W4/G32 layer (``w4a16_qmv``: K % 512 == 0, N % 4 == 0)."""
        return (AffineParameters._w4g32_bf16(shape, dtype, weight, scales, biases, group_size, bits)
                and math.prod(shape[:-1]) == 1 and shape[-1] % 512 == 0 and weight.shape[0] % 4 == 0)

    @staticmethod
    def supports_multirow(shape, dtype, weight, scales, biases, group_size, bits):
        """Eight BF16 rows of a W4/G32 layer (the verification pass)."""
        return (len(shape) >= 2 and math.prod(shape[:-1]) == 8
                and AffineParameters._w4g32_bf16(shape, dtype, weight, scales, biases, group_size, bits))

    @staticmethod
    def multirow(x, weight, scales, biases, group_size, bits):
        return ext.w4a16_multirow(x, weight, scales, biases, algorithm="wide", k_lanes=8, simdgroups=8)

    @staticmethod
    def multirow_packed(x, weight, scales, biases, group_size, bits):
        # the reference's prepared nax4 tile layout is a Metal layout; the B200 kernel reads the native one
        return ext.w4a16_multirow(x, weight, scales, biases, algorithm="nax4")

    @staticmethod
    def splitk(x, weight, scales, biases, group_size, bits):
        return ext.w4a16_qmv(x, weight, scales, biases)


def _on_gpu(t):
    return t.device.type == "cuda"


class QuantizedLinear(torch.nn.Module):
    """Affine-quantized projection with the ``nn.QuantizedLinear`` attributes."""

    mode = "affine"

    def __init__(self, weight, scales, biases, group_size=64, bits=4):
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.bias = None
        self.group_size = group_size
        self.bits = bits

    def forward(self, x):
        return AffineParameters.native(x, *AffineParameters.from_module(self))


def unpack_affine_w8(layer, name, *, allow_fallback=False):
    """Per-channel INT8 parameters of an MLX affine 8-bit layer.

    Restates ``_unpack_affine_w8`` (``spark_mlx_llm/ops/linear.py:299-324``):
    the layer must hold uint32-packed affine W8 (``weight [N, K/4]`` as
    int32/uint32 words, ``scales``/``biases [N, K/G]``) written as "symmetric
    in affine clothing" - every scale of a row equal, finite and positive, and
    ``biases == -128 * scales`` (``conversion.py:585-592``). Returns
    ``(weight int8 [N, K], scales float32 [N])``: the codes are the packed
    bytes XOR 0x80 (code = int8 + 128), the scale is the row's repeated
    scale. Raises ``ValueError`` for anything else, or returns ``None`` when
    ``allow_fallback`` and only the symmetric/per-channel check fails.
    Load-time work (torch ops on the weight's device), not the hot path.
    """
    weight, scales, biases = layer.weight, layer.scales, layer.biases
    if weight.ndim != 2:
        raise ValueError(f"{name}: QMV requires UINT32-packed affine W8 parameters")
    n, packed_k = weight.shape
    group = getattr(layer, "group_size", None)
    if (getattr(layer, "mode", "affine") != "affine" or weight.dtype not in (torch.int32, torch.uint32)
            or biases is None or not group or scales.ndim != 2
            or tuple(scales.shape) != (n, packed_k * 4 // group) or tuple(biases.shape) != tuple(scales.shape)):
        raise ValueError(f"{name}: QMV requires UINT32-packed affine W8 parameters")
    s = scales.float()
    b = biases.float()
    ok = bool((torch.isfinite(s) & (s > 0)).all() & (s == s[:, :1]).all() & (b == -128 * s).all())
    if not ok:
        if allow_fallback:
            return None
        raise ValueError(f"{name}: QMV requires repeated positive per-channel scales and "
                         "affine biases=-128*scales; groupwise/asymmetric W8 is unsupported")
    words = weight.contiguous().view(torch.int32) ^ torch.tensor(-0x7F7F7F80, dtype=torch.int32,
                                                                 device=weight.device)  # 0x80808080
    return words.view(torch.int8).reshape(n, packed_k * 4).contiguous(), s[:, 0].contiguous()


class W8A16PerChannelLinear(torch.nn.Module):
    """Single-row W8 projection with its affine layer as the fallback
    (``spark_mlx_llm/ops/linear.py:413-476``).

    ``fallback`` is the bias-free affine 8-bit :class:`QuantizedLinear`;
    ``weight`` (signed INT8 ``[N, K]``) and ``scales`` (fp32 ``[N]`` or
    ``[N, 1]``) its per-channel form, derived at load time
    (:func:`unpack_affine_w8`, :meth:`from_affine`). One BF16/FP16 row on a
    GPU runs ``ext.w8a16_per_channel``; every other input runs the affine
    layer. Same checks and errors as the reference."""

    def __init__(self, fallback, weight, scales):
        super().__init__()
        if (type(fallback) is not QuantizedLinear or fallback.mode != "affine" or fallback.bits != 8
                or fallback.biases is None or fallback.bias is not None):
            raise ValueError("W8A16 fallback must be a bias-free affine W8 QuantizedLinear")
        if (weight.ndim != 2 or weight.dtype != torch.int8
                or tuple(weight.shape) != (fallback.weight.shape[0], fallback.weight.shape[1] * 4)
                or scales.dtype != torch.float32
                or tuple(scales.shape) not in ((weight.shape[0],), (weight.shape[0], 1))):
            raise ValueError("W8A16 needs matching signed INT8 [N,K] and FP32 [N] scales")
        self.fallback = fallback
        self.register_buffer("weight", weight.contiguous())
        self.register_buffer("scales", scales.reshape(-1).contiguous())

    @classmethod
    def from_affine(cls, layer, name="projection"):
        """Build from an MLX affine W8 layer (the load-time conversion of
        ``QuantizedProjections.prepare``, ``ops/linear.py:725-731``)."""
        weight, scales = unpack_affine_w8(layer, name)
        return cls(layer, weight, scales)

    @staticmethod
    def supports_rows(num_rows, dtype, device_type="cuda"):
        return num_rows == 1 and dtype in (torch.bfloat16, torch.float16) and device_type == "cuda"

    def forward(self, x):
        if x.ndim >= 1 and x.shape[-1] > 0 and self.supports_rows(x.numel() // x.shape[-1], x.dtype,
                                                                  x.device.type):
            return ext.w8a16_per_channel(x, self.weight, self.scales)
        return self.fallback(x)


class W8MultirowProjection(torch.nn.Module):
    """W8 out/head projection for the 8-row verification pass, else the affine
    layer (``spark_mlx_llm/ops/linear.py:479-528``).

    ``fallback`` is the affine 8-bit :class:`QuantizedLinear`; ``weight`` (INT8
    ``[N, K]``) and ``scales`` (fp32 ``[N]``) are its per-channel form, derived
    at load time (:func:`unpack_affine_w8`). Exactly 8 BF16 rows on a CUDA
    device run ``ext.w8a16_multirow`` (the M <= 8 weight-streaming kernel) with
    the layer's scale dtype as the output dtype; M = 1 decode and prefill keep
    the affine layer. The accepted shapes are the reference's: the measured
    out_proj (2560 x 4096) and lm_head (131072 x 2560) geometries."""

    GEOMETRY = ((131072, 2560), (2560, 4096))

    def __init__(self, fallback, weight, scales):
        super().__init__()
        if (type(fallback) is not QuantizedLinear or fallback.bits != 8 or fallback.mode != "affine"
                or fallback.bias is not None or fallback.biases is None
                or fallback.scales.dtype not in (torch.bfloat16, torch.float32)
                or fallback.biases.dtype != fallback.scales.dtype
                or weight.dtype != torch.int8 or tuple(weight.shape) not in self.GEOMETRY
                or scales.dtype != torch.float32 or tuple(scales.shape) != (weight.shape[0],)
                or tuple(fallback.weight.shape) != (weight.shape[0], weight.shape[1] // 4)):
            raise ValueError("Multirow W8 requires measured out/head per-channel geometry")
        self.fallback = fallback
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)

    def takes_multirow(self, x):
        """True when ``x`` is the 8-row BF16 verification input on a GPU."""
        return (x.ndim >= 2 and math.prod(x.shape[:-1]) == 8 and x.shape[-1] == self.weight.shape[-1]
                and x.dtype == torch.bfloat16 and x.device.type == "cuda")

    def forward(self, x):
        if self.takes_multirow(x):
            return ext.w8a16_multirow(x, self.weight, self.scales, output_dtype=self.fallback.scales.dtype,
                                      variant="nax", simdgroups=4)
        return self.fallback(x)


class W8A8Projection(torch.nn.Module):
    """W8A8 arithmetic for a W8 projection, with the affine layer as its
    fallback (``spark_mlx_llm/ops/linear.py:531-562``): on a GPU every floating
    input runs ``ext.W8A8Linear`` (per-token INT8 activations, INT32
    accumulators, the W8A8 epilogue); other inputs run ``fallback``. Raises
    ``RuntimeError`` when the W8A8 kernels are unavailable (no supported GPU),
    as the reference does without its extension."""

    def __init__(self, fallback, weight, scales):
        super().__init__()
        if not ext.is_w8a8_available():
            raise RuntimeError("w8_qmv_backend='w8a8' requires a B200 (sm_100) GPU and libsparkb200")
        self.fallback = fallback
        self.projection = ext.W8A8Linear(weight, scales, getattr(fallback, "bias", None))

    def forward(self, x):
        if x.dtype in (torch.bfloat16, torch.float16, torch.float32) and x.device.type == "cuda":
            return self.projection(x)
        return self.fallback(x)


class QuantizedProjections:
    """Load-time lifecycle of a model's W8 output projections and untied LM
    head (``spark_mlx_llm/ops/linear.py:565-731``).

    A model is any object with ``layers`` (each with ``self_attn.out_proj``),
    ``args.tie_word_embeddings`` and, when untied, ``lm_head``. ``configure``
    wraps every 8-bit affine :class:`QuantizedLinear` among them in the
    adapter of the chosen ``w8_qmv_backend`` - ``"w8a16"``
    (:class:`W8A16PerChannelLinear`), ``"multirow"``
    (:class:`W8MultirowProjection`, the measured geometries only) or
    ``"w8a8"`` (:class:`W8A8Projection`) - with the per-channel INT8 form
    derived from the checkpoint tensors (:func:`unpack_affine_w8`). Layers
    outside an adapter's format keep their affine projection (``"w8a16"`` and
    ``"multirow"`` skip group-wise/asymmetric W8; ``"w8a8"`` rejects it).
    ``"auto"`` and ``"native"`` leave the model unchanged, and so does a
    backend whose kernels are unavailable. Every adapter is built before any
    module is replaced."""

    ADAPTERS = {"w8a16": W8A16PerChannelLinear, "multirow": W8MultirowProjection, "w8a8": W8A8Projection}
    MULTIROW_PACKED = ((131072, 640), (2560, 1024))  # packed words of the measured head / out_proj

    @staticmethod
    def projections(model):
        """``(checkpoint name, parent, attribute)`` of every W8 projection slot."""
        for index, layer in enumerate(model.layers):
            yield f"model.layers.{index}.self_attn.out_proj", layer.self_attn, "out_proj"
        if not model.args.tie_word_embeddings:
            yield "lm_head", model, "lm_head"

    @staticmethod
    def configure(model, backend):
        LinearConfig(w8_qmv_backend=backend)  # the reference's choice check
        if backend in ("auto", "native"):
            return
        if backend == "w8a8" and not ext.is_w8a8_available():
            return
        replacements = []
        for name, parent, attribute in QuantizedProjections.projections(model):
            layer = getattr(parent, attribute)
            if type(layer) is not QuantizedLinear or layer.bits != 8:
                continue
            if backend == "multirow" and (
                    tuple(layer.weight.shape) not in QuantizedProjections.MULTIROW_PACKED
                    or layer.scales.dtype not in (torch.bfloat16, torch.float32) or layer.biases is None
                    or layer.biases.dtype != layer.scales.dtype or layer.mode != "affine"
                    or layer.bias is not None):
                continue
            if backend == "w8a16" and (layer.mode != "affine" or layer.bias is not None):
                continue
            pair = unpack_affine_w8(layer, name, allow_fallback=backend in ("w8a16", "multirow"))
            if pair is None:
                continue
            replacements.append((parent, attribute, QuantizedProjections.ADAPTERS[backend](layer, *pair)))
        for parent, attribute, projection in replacements:
            setattr(parent, attribute, projection)

    @staticmethod
    def unwrap(model):
        """Put every adapter's affine layer back."""
        for _, parent, attribute in QuantizedProjections.projections(model):
            projection = getattr(parent, attribute)
            if type(projection) in tuple(QuantizedProjections.ADAPTERS.values()):
                setattr(parent, attribute, projection.fallback)

    @staticmethod
    def scale_paths(model):
        """Names of the fp32 scale tensors a dtype-casting loader must keep."""
        paths = set()
        for name, parent, attribute in QuantizedProjections.projections(model):
            projection = getattr(parent, attribute)
            if type(projection) in (W8A16PerChannelLinear, W8MultirowProjection):
                paths.add(name + ".scales")
            elif type(projection) is W8A8Projection:
                paths.add(name + ".projection.scales")
        return paths

    @staticmethod
    def prepare(model):
        """``configure`` with the model's own ``args.w8_qmv_backend``."""
        QuantizedProjections.configure(model, model.args.w8_qmv_backend)


class PreparedW8:
    """Derived INT8 buffers of an affine W8 layer, cached against the identity
    of its source tensors (``W8A8QuantizedLinear.prepare_parameters``,
    ``ops/linear.py:338-369``): repeated calls with the same ``weight``,
    ``scales`` and ``biases`` objects return the cached pair; new source
    tensors are validated and unpacked again."""

    def __init__(self):
        self._cache = None

    def __call__(self, layer, name="projection"):
        sources = (layer.weight, layer.scales, layer.biases)
        cached = self._cache
        if cached is not None and all(old is new for old, new in zip(cached[0], sources)):
            return cached[1]
        pair = unpack_affine_w8(layer, name)
        self._cache = (sources, pair)
        return pair


class RoPE:
    """The ``nn.RoPE`` attributes used by ``dispatch_qkv`` (half-split rotation)."""

    def __init__(self, dims, traditional=False, base=10000.0, scale=1.0):
        self.dims, self.traditional, self.base, self.scale = dims, traditional, base, scale


def dispatch_linear(x, projection, *, config=None):
    """Run an affine projection on the weight-streaming kernels, else call it."""
    config = config if config is not None else LinearConfig()
    if not isinstance(config, LinearConfig):
        raise TypeError("config must be a LinearConfig")
    if AffineParameters.accepts(projection):
        project, params = AffineParameters.resolve(projection, tuple(x.shape), x.dtype, config)
        return project(x, *params)
    return projection(x)


def dispatch_attention_output(x, output, gate_projection, output_projection):
    """Gated attention output (``spark_mlx_llm/ops/attention_output.py:16-101``):
    ``out_proj(output * sigmoid(x @ g^T))`` with one gate per head.

    ``x [B, L, hidden]`` is the block's normed input, ``output [B, H, L, D]``
    the attention output. A bias-free BF16 ``torch.nn.Linear`` gate on the GPU
    runs ``sb_head_gate`` (bf16 gate logits with fp32 accumulation, sigmoid in
    fp32 rounded to bf16, the product rounded to bf16 - the reference's dtype
    steps) and then the output projection through :func:`dispatch_linear`
    (affine kernels, or the W8 adapters' own routes); any other gate module is
    called as a module, as the reference does for custom modules."""
    b, l = x.shape[0], x.shape[1]
    heads, d = output.shape[1], output.shape[3]
    attn = output.transpose(1, 2).contiguous()  # [B, L, H, D]
    if (isinstance(gate_projection, torch.nn.Linear) and gate_projection.bias is None
            and x.dtype == output.dtype == gate_projection.weight.dtype == torch.bfloat16
            and x.device.type == "cuda"):
        gated = ops.head_gate(x.reshape(b * l, x.shape[-1]), gate_projection.weight, attn.reshape(b * l, heads, d))
        return dispatch_linear(gated.reshape(b, l, heads * d), output_projection)
    gate = torch.sigmoid(gate_projection(x).float()).to(output.dtype)
    return output_projection((attn * gate[..., None]).reshape(b, l, heads * d))


def dispatch_ffn(x, attention_output, norm, mlp, *, mlp_type):
    """Residual, RMSNorm and the gated GELU FFN (``spark_mlx_llm/ops/ffn.py:17-118``):
    ``h = x + attention_output``; ``h + down(gelu(gate(n)) * up(n))`` with
    ``n = rms_norm(h)``.

    When ``mlp`` is exactly ``mlp_type`` with affine ``gate_proj`` /
    ``up_proj`` / ``down_proj``, ``norm`` a ``torch.nn.RMSNorm`` and the input
    on the GPU, the norm is ``sb_rms_norm``, the projections the affine
    kernels and the gate ``sb_gated_activation`` (exact GELU); the residual adds
    round once to the activation dtype. Other modules are called as modules."""
    hidden = x + attention_output
    projections = [getattr(mlp, name, None) for name in ("gate_proj", "up_proj", "down_proj")]
    if (type(mlp) is not mlp_type or type(norm) is not torch.nn.RMSNorm or norm.weight is None
            or norm.weight.dtype != hidden.dtype or hidden.device.type != "cuda" or hidden.dtype != torch.bfloat16
            or not all(AffineParameters.accepts(p) for p in projections)):
        return hidden + mlp(norm(hidden))
    eps = norm.eps if norm.eps is not None else torch.finfo(hidden.dtype).eps
    normed = ops.rms_norm(hidden, norm.weight, float(eps))
    gate, up, down = projections
    act = ops.gated_activation(dispatch_linear(normed, gate), dispatch_linear(normed, up), 1)
    return hidden + dispatch_linear(act, down)


def dispatch_qkv(x, projection, rope, *, q_size, kv_size, n_heads, n_kv_heads, head_dim, offset, config=None):
    """Project, split heads and apply RoPE; returns ``(queries, keys, values)``
    shaped ``[B, H, L, D]``. Affine W4/W8 projections with a half-split RoPE of
    scale 1 over the full head run as one fused kernel (``spark_qkv_rope``,
    ops/qkv.py:40-66); ``offset`` is a Python int or an int32 tensor of
    per-token positions ``[B, L]``."""
    config = config if config is not None else LinearConfig()
    if not isinstance(config, LinearConfig):
        raise TypeError("config must be a LinearConfig")
    bsz, length, _ = x.shape
    fused = (AffineParameters.accepts(projection) and projection.bits in (4, 8)
             and projection.group_size in (32, 64, 128) and not rope.traditional and rope.scale == 1.0
             and rope.dims == head_dim and q_size == n_heads * head_dim and kv_size == n_kv_heads * head_dim)
    if fused:
        if isinstance(offset, torch.Tensor):
            positions = offset.to(device=x.device, dtype=torch.int32).reshape(-1)
        else:
            positions = (int(offset) + torch.arange(length, device=x.device, dtype=torch.int32)).repeat(bsz)
        return ops.qkv_rope(x, projection.weight, projection.scales, projection.biases, positions, n_heads,
                            n_kv_heads, head_dim, rope.dims, float(rope.base), projection.group_size,
                            projection.bits)
    raise ValueError("dispatch_qkv on B200 needs an affine W4/W8 projection with a half-split, scale-1 RoPE "
                     "over the full head dimension")


def dispatch_sdpa(queries, keys, values, *, cache, scale, mask, config=None, is_sliding=False):
    """Decode attention over a quantized KV cache (ops/sdpa.py:39-78).

    * INT8 pair ``(codes [B,KH,N,D] int8, scales [B,KH,N] fp16)``: one query
      token (``L == 1``, the last position attends to all N keys) runs the
      B200 INT8-KV decode kernel; ``L > 1`` queries (the last L of the N
      positions) run the INT8-KV prefill kernel, with the bottom-right causal
      mask for ``mask="causal"``.
    * Affine tuple ``(packed, scales, biases)`` with ``cache.bits`` /
      ``cache.group_size``: ``int8_quantized_sdpa`` (decode or causal prefill).
    * BF16 ``K/V [B,KH,N,D]`` tensors (the reference's bf16 caches, its
      ``tuned_bf16_sdpa`` and ``verification_bf16_sdpa`` routes,
      ``ops/sdpa.py:62-78``): the BF16 multi-query kernel for any query count,
      with no mask, ``"causal"`` or a boolean ``[L, N]`` array (a sliding
      layer's window arrives in that array), head_dim 128 / 256 and 1, 2, 4 or
      8 query heads per KV head.
    Other inputs raise ``ValueError``.
    """
    config = config if config is not None else SDPAConfig()
    if not isinstance(config, SDPAConfig):
        raise TypeError("config must be an SDPAConfig")
    if isinstance(keys, (tuple, list)) and len(keys) == 2 and len(values) == 2:
        if mask not in (None, "causal"):
            raise ValueError("the INT8 KV pair path takes no mask or 'causal'")
        n = keys[0].shape[2]
        if queries.shape[2] == 1:
            return ops.int8_sdpa_decode(queries, keys[0], keys[1], values[0], values[1], n, float(scale))
        return ops.int8_sdpa_prefill(queries, keys[0], keys[1], values[0], values[1], n, float(scale),
                                     mask == "causal")
    if isinstance(keys, (tuple, list)) and len(keys) == 3 and len(values) == 3:
        return ext.int8_quantized_sdpa(queries, keys, values, scale=scale,
                                       group_size=getattr(cache, "group_size", 32), bits=getattr(cache, "bits", 8),
                                       mask=mask)
    if isinstance(keys, torch.Tensor) and isinstance(values, torch.Tensor):
        causal = isinstance(mask, str) and mask == "causal"
        if mask is not None and not causal and not isinstance(mask, torch.Tensor):
            raise ValueError("mask must be None, 'causal' or a boolean [L, N] array")
        g = queries.shape[1] // keys.shape[1] if keys.ndim == 4 and keys.shape[1] > 0 else 0
        if (queries.dtype == keys.dtype == values.dtype == torch.bfloat16 and queries.ndim == 4
                and queries.shape[-1] in (128, 256) and g in (1, 2, 4, 8) and queries.shape[1] == g * keys.shape[1]):
            return ops.bf16_sdpa_multiquery(queries, keys, values, float(scale), causal, 0,
                                            mask if isinstance(mask, torch.Tensor) else None)
        raise ValueError("BF16 K/V attention needs bfloat16 Q/K/V, head_dim 128 or 256 and 1, 2, 4 or 8 "
                         "query heads per KV head")
    raise ValueError("dispatch_sdpa on B200 serves an (int8, fp16 scale) pair, an affine (packed, scales, "
                     "biases) tuple or BF16 K/V tensors")
