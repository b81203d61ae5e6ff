"""Tensor-parallel shard plan of the decoder (Megatron layout, one exchange per sub-block).

Per rank r of `world`:
* QKV: column split by heads - rows [r*Hq/t*D, ...) of Wq and [r*KH/t*D, ...)
  of Wk and Wv (every rank keeps whole KV heads; its KV cache holds them);
* o_proj and down_proj: row split over K (their inputs are the rank's heads /
  intermediate slice), followed by an all-reduce (sum) of the partial outputs;
* gate/up: column split of the intermediate dimension;
* lm_head: vocabulary split; each rank's argmax key (orderable float bits in
  the high 32 bits, inverted row index in the low 32 bits, compared unsigned)
  meets the others in an all-reduce MAX - the global argmax with the
  lowest-index tie-break. The collective compares signed 64-bit integers, so
  the keys cross it with their top bit flipped (``signed_key``), which maps
  unsigned order onto signed order.

The ranges here are what ``SyntheticDecoder`` slices from the full matrices.
"""

import struct
from dataclasses import dataclass

SIGN_FLIP = -(1 << 63)  # int64 with only the top bit set: x ^ SIGN_FLIP flips bit 63


@dataclass(frozen=True)
class ShardPlan:
    q_rows: tuple  # (start, count) rows of Wq [Hq*D, hidden]
    kv_rows: tuple  # rows of Wk and of Wv [KH*D, hidden]
    o_cols: tuple  # columns of Wo [hidden, Hq*D]
    inter_rows: tuple  # rows of Wgate / Wup [I, hidden]
    down_cols: tuple  # columns of Wdown [hidden, I]
    vocab_rows: tuple  # rows of lm_head [V, hidden]
    heads: int
    kv_heads: int
    inter: int
    vocab: int


def check(cfg, world):
    """Raise ValueError when the configuration cannot be split over `world` ranks."""
    if world < 1:
        raise ValueError("world size must be positive")
    if cfg.num_kv_heads % world or cfg.num_heads % world or cfg.intermediate % (world * cfg.mlp_group):
        raise ValueError("heads and intermediate size must divide across the tensor-parallel ranks")
    if cfg.vocab % world:
        raise ValueError("vocabulary must divide across the tensor-parallel ranks")


def plan(cfg, rank, world):
    """Shard ranges of rank `rank` (0 <= rank < world)."""
    check(cfg, world)
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    d = cfg.head_dim
    hq, hkv = cfg.num_heads // world, cfg.num_kv_heads // world
    inter, vocab = cfg.intermediate // world, cfg.vocab // world
    return ShardPlan(q_rows=(rank * hq * d, hq * d), kv_rows=(rank * hkv * d, hkv * d),
                     o_cols=(rank * hq * d, hq * d), inter_rows=(rank * inter, inter),
                     down_cols=(rank * inter, inter), vocab_rows=(rank * vocab, vocab), heads=hq, kv_heads=hkv,
                     inter=inter, vocab=vocab)


def argmax_key(value, index):
    """Host form of the device's greedy key (unsigned 64-bit): orderable float
    bits << 32 | (2^32 - 1 - index), NaN below every number."""
    bits = struct.unpack("<I", struct.pack("<f", value))[0]
    if value != value:
        u = 0x007FFFFF
    elif bits & 0x80000000:
        u = (~bits) & 0xFFFFFFFF
    else:
        u = bits | 0x80000000
    return (u << 32) | (0xFFFFFFFF - index)


def key_index(key):
    """Row index encoded in an (unsigned) argmax key."""
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


def signed_key(key):
    """Unsigned key -> int64 whose signed order is the unsigned order (top bit flipped)."""
    return (key ^ (1 << 63)) - (1 << 64) if key & (1 << 63) == 0 else key ^ (1 << 63)


def unsigned_key(value):
    """Inverse of ``signed_key``."""
    return (value & ((1 << 64) - 1)) ^ (1 << 63)
