"""Weight streams and descriptor of the persistent decode-step kernel.

``sb_step_run`` (include/spark_b200_step.h) reads each weight matrix as a
stream of tiles - one 16-row block x one K chunk - laid out in the order one
warp consumes them, so every shared-memory read of a tile is a conflict-free
16-byte load that is already an MMA fragment. This module builds those
streams once, on the GPU, from the checkpoint tensors the per-operator path
uses (MLX affine 4-bit words with bf16 scales/biases, per-channel int8 with
fp32 scales, bf16 rows) - the "offline repack behind the same API" the
reference also does for its multi-row kernels (``prepare_w4a16_nax4``,
``spark_mlx_ext/w4a16_multirow.py:132-222``). The streams hold the same codes
and metadata; only the byte order changes.

Lane ``L = 4g + c`` of a warp holds rows ``g`` and ``g + 8`` of a block.
"""

import ctypes

import torch

from ._lib import check, lib, sb_step_desc, sb_step_layer

__all__ = ["pack_w8", "pack_w4", "pack_bf16", "qkv_row_order", "sb_step_layer", "sb_step_desc", "CHUNKS"]

CHUNKS = 8  # K chunks of o_proj / down_proj / lm_head (the tensor-parallel unit)


def qkv_row_order(num_heads, num_kv_heads, head_dim=128, device=None):
    """Stream row order of the fused QKV matrix: block ``8*hd + i`` of head
    ``hd`` holds dims ``8i..8i+7`` in rows 0-7 and their RoPE partners
    ``64+8i..`` in rows 8-15 (heads: query, then key, then value)."""
    heads = num_heads + 2 * num_kv_heads
    hd = torch.arange(heads, device=device).view(heads, 1, 1, 1)
    i = torch.arange(head_dim // 16, device=device).view(1, -1, 1, 1)
    hh = torch.arange(2, device=device).view(1, 1, 2, 1)
    g = torch.arange(8, device=device).view(1, 1, 1, 8)
    return (hd * head_dim + hh * (head_dim // 2) + 8 * i + g).reshape(-1)


def pack_w8(w_int8, chunk_k, row_order=None, chunk_major=False):
    """Per-channel int8 ``[N, K]`` -> W8 tile stream (uint8).

    Tile (block b, chunk c) is ``chunk_k/32`` runs of 512 bytes; in run j
    lane (g, c4) holds row g bytes [32j+8c4, +4), row g+8 same, row g bytes
    [32j+8c4+4, +4), row g+8 same; each byte is the code XOR 0x80."""
    if row_order is not None:
        w_int8 = w_int8[row_order]
    n, k = w_int8.shape
    if n % 16 or k % chunk_k or chunk_k % 32:
        raise ValueError("W8 stream: N % 16, K % chunk and chunk % 32 must be 0")
    u = w_int8.contiguous().view(torch.uint8) ^ 0x80
    t = u.view(n // 16, 2, 8, k // chunk_k, chunk_k // 32, 4, 2, 4)  # [rb, hh, g, ch, kb, c, word, byte]
    t = t.permute(0, 3, 4, 2, 5, 6, 1, 7)  # [rb, ch, kb, g, c, word, hh, byte]
    if chunk_major:  # tiles ordered by K chunk first (o_proj: a CTA's tiles read few chunks)
        t = t.transpose(0, 1)
    return t.contiguous().view(-1)


def pack_w4(mats, groups_per_chunk, chunk_major=False):
    """MLX affine 4-bit, group 64 -> W4 tile stream (uint8).

    ``mats`` is a list of 1 or 2 ``(packed int32 [N, K/8], scales bf16
    [N, K/64], biases bf16 [N, K/64])`` with equal shapes (gate and up share
    tiles). A tile is, per group, per matrix, 512 bytes where lane (g, c)
    holds words [row g word c, row g+8 word c, row g word c+4, row g+8 word
    c+4] of the group; then scales as [round of 8 groups][matrix][16 rows][8]
    bf16 and biases likewise (zero padded). Tiles are ordered row-block-major,
    or K-chunk-major with ``chunk_major`` (down_proj: a CTA's run of tiles then
    reads one or two K chunks of the activations)."""
    packed0 = mats[0][0]
    n, kw = packed0.shape
    k = kw * 8
    gc = groups_per_chunk
    if n % 16 or (k // 64) % gc:
        raise ValueError("W4 stream: N % 16 == 0 and whole chunks of groups required")
    nm = len(mats)
    rb, ch = n // 16, (k // 64) // gc
    rounds = (gc + 7) // 8
    codes = torch.stack([m[0].contiguous().view(torch.int32) for m in mats], 0)  # [mat, N, K/8]
    codes = codes.view(nm, rb, 2, 8, ch, gc, 2, 4)  # [mat, rb, hh, g, ch, gc, wq, c]
    codes = codes.permute(1, 4, 5, 0, 3, 7, 6, 2).contiguous()  # [rb, ch, gc, mat, g, c, wq, hh]
    codes = codes.view(rb, ch, -1).view(torch.uint8)

    def meta(idx):
        t = torch.stack([m[idx].contiguous().view(torch.int16) for m in mats], 0)  # [mat, N, K/64]
        t = t.view(nm, rb, 16, ch, gc)
        if rounds * 8 != gc:
            pad = torch.zeros(nm, rb, 16, ch, rounds * 8 - gc, dtype=t.dtype, device=t.device)
            t = torch.cat([t, pad], -1)
        t = t.view(nm, rb, 16, ch, rounds, 8).permute(1, 3, 4, 0, 2, 5).contiguous()  # [rb, ch, round, mat, row, 8]
        return t.view(rb, ch, -1).view(torch.uint8)

    tiles = torch.cat([codes, meta(1), meta(2)], -1)  # [rb, ch, bytes]
    if chunk_major:
        tiles = tiles.transpose(0, 1)
    return tiles.contiguous().view(-1)


def pack_bf16(w_bf16, chunk_k):
    """bf16 ``[V, K]`` -> BF16 tile stream (rows padded to a multiple of 16 with zeros).

    Tile (block b, chunk c) is ``chunk_k/16`` runs of 512 bytes; in run j lane
    (g, c4) holds row g cols 16j+4c4+{0,1}, row g+8 same, row g cols
    16j+4c4+{2,3}, row g+8 same."""
    v, k = w_bf16.shape
    vp = (v + 15) // 16 * 16
    if vp != v:
        w_bf16 = torch.cat([w_bf16, torch.zeros(vp - v, k, dtype=w_bf16.dtype, device=w_bf16.device)])
    if k % chunk_k or chunk_k % 16:
        raise ValueError("BF16 stream: K % chunk and chunk % 16 must be 0")
    t = w_bf16.contiguous().view(torch.int16).view(vp // 16, 2, 8, k // chunk_k, chunk_k // 16, 4, 2, 2)
    # [rb, hh, g, ch, j, c, p, e] -> [rb, ch, j, g, c, p, hh, e]
    return t.permute(0, 3, 4, 2, 5, 6, 1, 7).contiguous().view(-1).view(torch.uint8)


class StepStreams:
    """The decoder's weights as tile streams plus the kernel descriptor and
    its scratch buffers (one rank, batch 1)."""

    def __init__(self, dec):
        cfg = dec.cfg
        dev = dec.device
        self.dec = dec
        d = cfg.head_dim
        if dec.batch != 1 or dec.world != 1:
            raise ValueError("the decode-step kernel serves batch 1 on one rank")
        if d != 128:
            raise ValueError("the decode-step kernel supports head_dim 128")
        order = qkv_row_order(dec.hq, dec.hkv, d, device=dev)
        down_groups = cfg.intermediate // 64 // CHUNKS
        self.keep = []
        layers = (sb_step_layer * cfg.num_layers)()
        for li, layer in enumerate(dec.layers):
            qkv = pack_w8(layer["qkv_w"], 512, order)
            qkv_s = layer["qkv_s"][order].contiguous()
            o = pack_w8(layer["o_w"], (dec.hq * d) // CHUNKS, chunk_major=True)
            gu = pack_w4([layer["gate"], layer["up"]], 8)
            dn = pack_w4([layer["down"]], down_groups, chunk_major=True)
            self.keep += [qkv, qkv_s, o, gu, dn]
            L = layers[li]
            L.qkv, L.qkv_scale, L.o, L.o_scale = qkv.data_ptr(), qkv_s.data_ptr(), o.data_ptr(), layer["o_s"].data_ptr()
            L.gateup, L.down = gu.data_ptr(), dn.data_ptr()
            L.in_norm, L.post_norm = layer["in_norm"].data_ptr(), layer["post_norm"].data_ptr()
            L.k_cache, L.k_scale = dec.k_cache[li].data_ptr(), dec.k_scale[li].data_ptr()
            L.v_cache, L.v_scale = dec.v_cache[li].data_ptr(), dec.v_scale[li].data_ptr()
        self.layer_table = torch.frombuffer(bytearray(bytes(layers)), dtype=torch.uint8).to(dev)
        self.head = pack_bf16(dec.head, cfg.hidden // CHUNKS)
        self.q = torch.zeros(dec.hq * d, dtype=torch.bfloat16, device=dev)
        self.kv_new = torch.zeros(2 * dec.hkv * d, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros(dec.hq * d, dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros(dec.inter, dtype=torch.bfloat16, device=dev)
        self.x = torch.zeros(cfg.hidden, dtype=torch.bfloat16, device=dev)
        desc = sb_step_desc()
        desc.layers = self.layer_table.data_ptr()
        desc.num_layers = cfg.num_layers
        desc.hidden = cfg.hidden
        desc.num_heads, desc.num_kv_heads, desc.head_dim = dec.hq, dec.hkv, d
        desc.inter, desc.inter_total = dec.inter, cfg.intermediate
        desc.vocab, desc.vocab_offset, desc.vocab_total = dec.vocab_shard, dec.plan.vocab_rows[0], cfg.vocab
        desc.capacity = dec.capacity
        desc.rms_eps, desc.rope_theta = cfg.rms_eps, cfg.rope_theta
        desc.embed, desc.head, desc.final_norm = dec.embed.data_ptr(), self.head.data_ptr(), dec.final_norm.data_ptr()
        desc.tokens, desc.positions = dec.tokens.data_ptr(), dec.positions.data_ptr()
        desc.x, desc.q, desc.kv_new = self.x.data_ptr(), self.q.data_ptr(), self.kv_new.data_ptr()
        desc.attn, desc.act, desc.argmax_key = self.attn.data_ptr(), self.act.data_ptr(), dec.keys.data_ptr()
        desc.world, desc.rank = dec.world, dec.rank
        nbytes = lib().sb_step_workspace_size(ctypes.byref(desc))
        if nbytes == 0:
            raise ValueError("shape not supported by the decode-step kernel: "
                             + lib().sb_last_error_message().decode(errors="replace"))
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        desc.workspace, desc.workspace_bytes = self.workspace.data_ptr(), nbytes
        self.desc = desc
        torch.cuda.synchronize(dev)

    def run(self, stream):
        check(lib().sb_step_run(ctypes.byref(self.desc), stream), "decode step")

    def run_layers(self, layers, stream):
        """Inspection aid: run the step with only the first ``layers`` layers
        (plus the lm_head); the residual stream after them lands in ``x``.
        Writes the same K/V rows at the current position as a full step."""
        full = self.desc.num_layers
        self.desc.num_layers = layers
        try:
            self.run(stream)
        finally:
            self.desc.num_layers = full

    def status(self):
        """Device status word of the step kernel (nonzero: a bounded wait gave up,
        or a position outside the cache); sticky across launches until cleared."""
        at = lib().sb_step_status_offset()
        return int(self.workspace[at:at + 4].view(torch.int32).item())

    def clear_status(self):
        at = lib().sb_step_status_offset()
        self.workspace[at:at + 4].zero_()
