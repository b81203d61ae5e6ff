"""Device-side quantizers that produce the hot path's weight formats.

They run on whatever device their input lives on (the synthetic model builds
its 3.2 GB of weights on the GPU with them) and produce bytes identical to the
CPU restatement used as the test oracle (checked on CPU in
``tests/test_quantize.py``):

* MLX affine codes with per-group min/max (``scale = (max - min) / (2**b - 1)``,
  ``bias = min``, both rounded to bf16; ``q = clip(rint((w - bias) / scale))``),
  packed little-endian into uint32 words (``spark_mlx_llm/conversion.py:429-433``).
* symmetric per-channel int8 (``scale = absmax / 127``, optionally rounded to bf16).
"""

import torch

__all__ = ["quantize_affine_minmax", "quantize_w8_per_channel", "pack_codes"]


def pack_codes(codes, bits):
    """Pack unsigned codes ``[..., K]`` into int32 words ``[..., K*bits/32]``
    (element j of a word at bits ``[j*bits, (j+1)*bits)``)."""
    per_word = 32 // bits
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], -1, per_word)
    shifts = torch.arange(per_word, device=codes.device, dtype=torch.int64) * bits
    words = (c << shifts).sum(dim=-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


def quantize_affine_minmax(w, group_size, bits):
    """Returns ``(packed int32 [N, K*bits/32], scales bf16 [N, K/G], biases bf16 [N, K/G])``."""
    w = w.float()
    n, k = w.shape
    levels = float((1 << bits) - 1)
    g = w.reshape(n, k // group_size, group_size)
    lo = g.amin(dim=-1)
    hi = g.amax(dim=-1)
    scale = ((hi - lo) / levels).to(torch.bfloat16).float()
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    bias = lo.to(torch.bfloat16).float()
    q = torch.round((g - bias[..., None]) / scale[..., None]).clamp_(0, levels)
    packed = pack_codes(q.reshape(n, k).to(torch.int32), bits)
    return packed, scale.to(torch.bfloat16), bias.to(torch.bfloat16)


def quantize_w8_per_channel(w, scale_to_bf16=True):
    """Returns ``(int8 [N, K], float32 scales [N])`` with ``scale = absmax / 127``."""
    w = w.float()
    scale = w.abs().amax(dim=1) / 127.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    if scale_to_bf16:
        scale = scale.to(torch.bfloat16).float()
    q = torch.round(w / scale[:, None]).clamp_(-127, 127).to(torch.int8)
    return q, scale
