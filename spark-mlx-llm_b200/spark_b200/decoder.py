"""Synthetic 4B-class decoder on the spark_b200 kernels (1 GPU or tensor parallel).

Architecture: 36 layers, hidden 2560, 32 query / 8 KV
heads, head_dim 128, SwiGLU MLP with intermediate 9728, RMSNorm eps 1e-6,
vocab 151936, RoPE theta 1e6. Attention projections are per-channel INT8
(the reference's default W8A16 backend, ``spark_mlx_llm/ops/linear.py:413-476``),
the MLP is MLX affine INT4 with group 64, embedding and lm_head are bf16, and
the KV cache is INT8 with one fp16 scale per token per head.

One decode step is, per layer (``spark_mlx_llm/model.py:172-207,249-262``):
  1. RMSNorm + QKV projection + RoPE        -> q, k_new, v_new   (one kernel)
  2. INT8 KV append of the new token                             (one kernel)
  3. INT8-KV attention over the cache                            (one kernel)
  4. o_proj + residual add                                       (one kernel)
  5. RMSNorm + gate/up + SwiGLU                                  (one kernel)
  6. down projection + residual add                              (one kernel)
then RMSNorm + lm_head + greedy argmax and the token/position update. Tensor
parallel (Megatron layout): QKV/gate/up split by output rows (heads), o/down by
input columns followed by an NCCL all-reduce, lm_head by vocabulary rows with
an all-reduce(max) of packed (logit, index) keys. Every per-step value lives in
device memory, so a whole step is captured once as a CUDA graph and replayed.

Weights are random (seeded) and built on the GPU: the workload has the real
shapes, formats and byte counts, not trained values.
"""

import ctypes
import math
from dataclasses import dataclass

import torch

from . import quantize
from . import tp as tensor_parallel
from ._lib import SBError, check, lib, sb_linear_ex_desc

__all__ = ["DecoderConfig", "SyntheticDecoder"]

SB_WEIGHT_AFFINE4, SB_WEIGHT_AFFINE8, SB_WEIGHT_INT8_PC, SB_WEIGHT_BF16 = 0, 1, 2, 3
SB_EPI_STORE, SB_EPI_RESID, SB_EPI_SWIGLU, SB_EPI_ROPE, SB_EPI_ARGMAX = 0, 1, 2, 3, 4
BF16 = 0
# device status word: the last 32-bit word of a workspace's 128 KiB counter
# region (nonzero when a bounded device-side wait gave up)
STATUS_WORD = 128 * 1024 // 4 - 1
# prompt tokens per batched prefill chunk (the reference's prompt chunk, generation.py:78)
PREFILL_CHUNK = 512
# fixed K chunks of the row-split projections: the largest tensor-parallel degree
TP_CHUNKS = 8


@dataclass(frozen=True)
class DecoderConfig:
    num_layers: int = 36
    hidden: int = 2560
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 9728
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    mlp_group: int = 64
    # init scales of the synthetic weights
    weight_std: float = 0.02
    embed_std: float = 1.0
    head_std: float = 0.02

    @staticmethod
    def small(**overrides):
        """A reduced shape with the same kernels (tests)."""
        base = dict(num_layers=2, hidden=512, num_heads=4, num_kv_heads=2, head_dim=128, intermediate=1024,
                    vocab=1000)
        base.update(overrides)
        return DecoderConfig(**base)

    def weight_bytes(self):
        """HBM bytes of weights read per decode step (all shards together)."""
        q = self.num_heads * self.head_dim
        kv = self.num_kv_heads * self.head_dim
        qkv = (q + 2 * kv) * self.hidden + (q + 2 * kv) * 4
        o = self.hidden * q + self.hidden * 4
        g = self.mlp_group
        mlp_in = 2 * (self.intermediate * self.hidden // 2 + self.intermediate * (self.hidden // g) * 4)
        mlp_out = self.hidden * self.intermediate // 2 + self.hidden * (self.intermediate // g) * 4
        norms = 2 * self.hidden * 2
        per_layer = qkv + o + mlp_in + mlp_out + norms
        return self.num_layers * per_layer + self.vocab * self.hidden * 2 + self.hidden * 2


def _ptr(t):
    return 0 if t is None else t.data_ptr()


class SyntheticDecoder:
    """The decoder's weights, INT8 KV cache, device state and launch sequence.

    ``rank``/``world`` select the tensor-parallel shard; ``group`` is the
    ``torch.distributed`` process group used for the all-reduces (None for 1 GPU).

    ``invariant`` (launch engine) fixes every floating-point summation order
    independently of ``world``, so greedy tokens are bit-identical at TP
    1/2/4/8: the column-split GEMVs (QKV, gate/up, lm_head) split K as for the
    unsharded matrix, the row-split o/down projections sum K in 8 fixed chunks
    added in a balanced tree (a rank holds 8/world of them; the fused exchange
    adds the ranks' partials in the same tree), and attention splits its tokens
    as for all KV heads.
    """

    def __init__(self, config, *, batch, capacity, device="cuda", seed=0, rank=0, world=1, group=None,
                 engine="auto", invariant=True):
        cfg = config
        self.cfg = cfg
        self.batch = batch
        self.capacity = ((capacity + 15) // 16) * 16
        self.device = torch.device(device)
        self.rank, self.world, self.group = rank, world, group
        if batch < 1 or batch > 8:
            raise ValueError("batch must be in [1, 8]")
        self.plan = tensor_parallel.plan(cfg, rank, world)
        self.hq = self.plan.heads
        self.hkv = self.plan.kv_heads
        self.inter = self.plan.inter
        self.vocab_shard = self.plan.vocab
        # K/V quantized into the cache by the QKV kernel's epilogue (head_dim 64/128)
        self.fused_append = cfg.head_dim in (64, 128)
        # TP: o/down partial sums meet inside the GEMV epilogue (NVLink peer
        # stores) instead of an NCCL all-reduce and a residual-add launch
        self.fused_allreduce = world > 1 and world <= 8
        # K chunks of the unsharded o/down projections (1: no fixed chunking)
        self.k_chunks = 1
        if invariant and TP_CHUNKS % world == 0:
            o_k, down_k = cfg.num_heads * cfg.head_dim, cfg.intermediate
            if (o_k % (TP_CHUNKS * 64) == 0 and (o_k // TP_CHUNKS) % 16 == 0
                    and down_k % (TP_CHUNKS * cfg.mlp_group) == 0 and (down_k // TP_CHUNKS) % 32 == 0):
                self.k_chunks = TP_CHUNKS
        self.invariant = invariant
        if engine not in ("auto", "step", "launches"):
            raise ValueError("engine must be 'auto', 'step' or 'launches'")
        self._build_weights(seed)
        self._alloc_state()
        self.graph = None
        # "step": the whole decode step is one persistent kernel (batch 1, one
        # rank, head_dim 128; spark_b200_step.h); "launches": one fused kernel
        # per operator with programmatic dependent launch. "auto" takes the
        # launch sequence, measured the faster of the two at the 4B shape
        # (1.80 vs 1.86 ms per batch-1 step on B200)
        if engine == "auto":
            engine = "launches"
        if engine == "step" and not (batch == 1 and world == 1 and cfg.head_dim == 128):
            raise ValueError("the decode-step kernel serves batch 1 on one GPU with head_dim 128")
        self.engine = engine
        self.stepper = None
        if engine == "step":
            from .step import StepStreams

            self.stepper = StepStreams(self)

    # ------------------------------------------------------------------ weights
    def _build_weights(self, seed):
        cfg, dev = self.cfg, self.device
        gen = torch.Generator(device=dev)
        d = cfg.head_dim
        sp = self.plan

        def randn(*shape, std, key):
            gen.manual_seed(seed * 1_000_003 + key)
            return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std

        def rows(t, start, count):
            return t[start:start + count]

        self.layers = []
        for li in range(cfg.num_layers):
            base = 1000 * (li + 1)
            layer = {}
            # full matrices are generated identically on every rank, then sharded
            wq = randn(cfg.num_heads * d, cfg.hidden, std=cfg.weight_std, key=base + 1)
            wk = randn(cfg.num_kv_heads * d, cfg.hidden, std=cfg.weight_std, key=base + 2)
            wv = randn(cfg.num_kv_heads * d, cfg.hidden, std=cfg.weight_std, key=base + 3)
            qkv = torch.cat([rows(wq, *sp.q_rows), rows(wk, *sp.kv_rows), rows(wv, *sp.kv_rows)])
            del wq, wk, wv
            layer["qkv_w"], layer["qkv_s"] = quantize.quantize_w8_per_channel(qkv)
            del qkv
            # the checkpoint is quantized once (per-row scales over the full K);
            # a tensor-parallel rank keeps its columns of the same codes
            wo = randn(cfg.hidden, cfg.num_heads * d, std=cfg.weight_std, key=base + 4)
            o_w, layer["o_s"] = quantize.quantize_w8_per_channel(wo)
            layer["o_w"] = o_w[:, sp.o_cols[0]:sp.o_cols[0] + sp.o_cols[1]].contiguous()
            del wo, o_w
            for name, key in (("gate", 5), ("up", 6)):
                w = randn(cfg.intermediate, cfg.hidden, std=cfg.weight_std, key=base + key)
                w = rows(w, *sp.inter_rows)
                layer[name] = quantize.quantize_affine_minmax(w, cfg.mlp_group, 4)
                del w
            wd = randn(cfg.hidden, cfg.intermediate, std=cfg.weight_std, key=base + 7)
            wd = wd[:, sp.down_cols[0]:sp.down_cols[0] + sp.down_cols[1]].contiguous()
            layer["down"] = quantize.quantize_affine_minmax(wd, cfg.mlp_group, 4)
            # the decode GEMV's copy of the scale/bias tables, rows padded to a
            # multiple of 8 groups (16 bytes) so a shard's tables stream by TMA
            groups = layer["down"][1].shape[1]
            ld = -(-groups // 8) * 8
            pads = []
            for t in layer["down"][1:]:
                pad = torch.zeros(t.shape[0], ld, dtype=t.dtype, device=dev)
                pad[:, :groups] = t
                pads.append(pad)
            layer["down_tables"], layer["down_ld"] = pads, ld
            del wd
            layer["in_norm"] = (1.0 + 0.1 * randn(cfg.hidden, std=1.0, key=base + 8)).to(torch.bfloat16)
            layer["post_norm"] = (1.0 + 0.1 * randn(cfg.hidden, std=1.0, key=base + 9)).to(torch.bfloat16)
            self.layers.append(layer)
        self.embed = randn(cfg.vocab, cfg.hidden, std=cfg.embed_std, key=11).to(torch.bfloat16)
        head = randn(cfg.vocab, cfg.hidden, std=cfg.head_std, key=12)
        self.head = rows(head, *sp.vocab_rows).to(torch.bfloat16).contiguous()
        del head
        self.final_norm = (1.0 + 0.1 * randn(cfg.hidden, std=1.0, key=13)).to(torch.bfloat16)
        torch.cuda.synchronize(dev)

    # -------------------------------------------------------------------- state
    def _alloc_state(self):
        cfg, dev, b = self.cfg, self.device, self.batch
        d = cfg.head_dim
        self.k_cache = [torch.zeros((b, self.hkv, self.capacity, d), dtype=torch.int8, device=dev)
                        for _ in range(cfg.num_layers)]
        self.v_cache = [torch.zeros_like(self.k_cache[0]) for _ in range(cfg.num_layers)]
        self.k_scale = [torch.ones((b, self.hkv, self.capacity), dtype=torch.float16, device=dev)
                        for _ in range(cfg.num_layers)]
        self.v_scale = [torch.ones_like(self.k_scale[0]) for _ in range(cfg.num_layers)]
        self.x = torch.zeros((b, cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.q = torch.zeros((b, self.hq, 1, d), dtype=torch.bfloat16, device=dev)
        self.k_new = torch.zeros((b, self.hkv, 1, d), dtype=torch.bfloat16, device=dev)
        self.v_new = torch.zeros_like(self.k_new)
        self.attn = torch.zeros((b, self.hq * d), dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros((b, self.inter), dtype=torch.bfloat16, device=dev)
        self.part = torch.zeros((b, cfg.hidden), dtype=torch.bfloat16, device=dev)
        self.tokens = torch.zeros((b,), dtype=torch.int32, device=dev)
        self.positions = torch.zeros((b,), dtype=torch.int32, device=dev)
        self.keys = torch.zeros((b,), dtype=torch.int64, device=dev)
        self._setup_exchange()
        self._build_descs()
        sizes = [lib().sb_linear_ex_workspace_size(ctypes.byref(desc)) for desc in self._descs_all()]
        # attention plans its token splits as for the unsharded heads (invariant)
        sizes.append(lib().sb_int8_sdpa_workspace_size(b, cfg.num_heads, cfg.num_kv_heads, self.capacity, d))
        self.workspace = torch.zeros(max(sizes) + 256, dtype=torch.uint8, device=dev)
        for desc in self._descs_all():
            desc.workspace = self.workspace.data_ptr()
            desc.workspace_bytes = self.workspace.numel()

    def _setup_exchange(self):
        """Tensor parallel: every rank allocates a zeroed exchange buffer, exports
        it as a CUDA IPC handle and maps the other ranks' buffers (NVLink peer
        access), for the all-reduce fused into the o/down GEMV epilogues."""
        self.ar_buffers = []
        self._own_buffer = None
        self._mapped = []
        if not self.fused_allreduce:
            return
        import torch.distributed as dist

        L = lib()
        nbytes = L.sb_tp_exchange_bytes(self.world, self.cfg.hidden)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        check(L.sb_peer_buffer_alloc(nbytes, ctypes.byref(ptr), handle), "exchange buffer")
        self._own_buffer = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        for r in range(self.world):
            if r == self.rank:
                self.ar_buffers.append(self._own_buffer)
                continue
            peer = ctypes.c_void_p()
            h = (ctypes.c_ubyte * 64).from_buffer_copy(handles[r])
            check(L.sb_peer_buffer_open(h, ctypes.byref(peer)), "map peer exchange buffer")
            self._mapped.append(peer.value)
            self.ar_buffers.append(peer.value)
        dist.barrier(group=self.group)

    def close(self):
        """Unmap the peers' exchange buffers and free this rank's (tensor parallel)."""
        L = lib()
        for ptr in self._mapped:
            L.sb_peer_buffer_close(ptr)
        self._mapped = []
        if self._own_buffer:
            L.sb_peer_buffer_free(self._own_buffer)
            self._own_buffer = None

    def _allreduce_desc(self, desc, channel):
        """o/down epilogue: residual add with the ranks' partial sums reduced in-kernel."""
        desc.epilogue = SB_EPI_RESID
        desc.y = _ptr(self.x)
        desc.residual = _ptr(self.x)
        desc.ar_world = self.world
        desc.ar_rank = self.rank
        desc.ar_channel = channel
        for r, ptr in enumerate(self.ar_buffers):
            desc.ar_buffers[r] = ptr

    def _desc(self, **kw):
        desc = sb_linear_ex_desc()
        desc.x_dtype = BF16
        desc.norm_eps = self.cfg.rms_eps
        desc.weights_constant = 1
        for key, value in kw.items():
            setattr(desc, key, value)
        return desc

    def _build_descs(self):
        cfg, b = self.cfg, self.batch
        d = cfg.head_dim
        tp = self.world > 1
        chunks = self.k_chunks // self.world
        plan_chunks = self.k_chunks if self.k_chunks > 1 else 0

        def plan(rows):  # column-split shards plan their K split as the whole matrix
            return rows if self.invariant else 0

        self.descs = []
        for layer in self.layers:
            qkv = self._desc(x=_ptr(self.x), M=b, N=(self.hq + 2 * self.hkv) * d, K=cfg.hidden,
                             weight_format=SB_WEIGHT_INT8_PC, weight=_ptr(layer["qkv_w"]), scales=_ptr(layer["qkv_s"]),
                             norm_weight=_ptr(layer["in_norm"]), epilogue=SB_EPI_ROPE,
                             positions=_ptr(self.positions), num_heads=self.hq, num_kv_heads=self.hkv, head_dim=d,
                             seq_len=1, rope_base=cfg.rope_theta, q_out=_ptr(self.q), k_out=_ptr(self.k_new),
                             v_out=_ptr(self.v_new), plan_rows=plan((cfg.num_heads + 2 * cfg.num_kv_heads) * d))
            if self.fused_append:
                # the QKV kernel quantizes K/V straight into this layer's INT8 cache
                li = len(self.descs)
                qkv.kv_k_cache = _ptr(self.k_cache[li])
                qkv.kv_k_scale = _ptr(self.k_scale[li])
                qkv.kv_v_cache = _ptr(self.v_cache[li])
                qkv.kv_v_scale = _ptr(self.v_scale[li])
                qkv.kv_capacity = self.capacity
            o = self._desc(x=_ptr(self.attn), M=b, N=cfg.hidden, K=self.hq * d, weight_format=SB_WEIGHT_INT8_PC,
                           weight=_ptr(layer["o_w"]), scales=_ptr(layer["o_s"]),
                           epilogue=SB_EPI_STORE if tp else SB_EPI_RESID,
                           y=_ptr(self.part if tp else self.x), residual=_ptr(self.x), k_chunks=chunks,
                           plan_k_chunks=plan_chunks)
            gw, gs, gb = layer["gate"]
            uw, us, ub = layer["up"]
            gateup = self._desc(x=_ptr(self.x), M=b, N=self.inter, K=cfg.hidden, weight_format=SB_WEIGHT_AFFINE4,
                                weight=_ptr(gw), scales=_ptr(gs), biases=_ptr(gb), weight2=_ptr(uw),
                                scales2=_ptr(us), biases2=_ptr(ub), group_size=cfg.mlp_group,
                                norm_weight=_ptr(layer["post_norm"]), epilogue=SB_EPI_SWIGLU, y=_ptr(self.act),
                                plan_rows=plan(cfg.intermediate))
            dw = layer["down"][0]
            ds, db = layer["down_tables"]
            down = self._desc(x=_ptr(self.act), M=b, N=cfg.hidden, K=self.inter, weight_format=SB_WEIGHT_AFFINE4,
                              weight=_ptr(dw), scales=_ptr(ds), biases=_ptr(db), group_size=cfg.mlp_group,
                              epilogue=SB_EPI_STORE if tp else SB_EPI_RESID,
                              y=_ptr(self.part if tp else self.x), residual=_ptr(self.x), k_chunks=chunks,
                              plan_k_chunks=plan_chunks, scales_ld=layer["down_ld"])
            if self.fused_allreduce:
                self._allreduce_desc(o, 0)
                self._allreduce_desc(down, 1)
            self.descs.append((qkv, o, gateup, down))
        self.head_desc = self._desc(x=_ptr(self.x), M=b, N=self.vocab_shard, K=cfg.hidden,
                                    weight_format=SB_WEIGHT_BF16, weight=_ptr(self.head),
                                    norm_weight=_ptr(self.final_norm), epilogue=SB_EPI_ARGMAX,
                                    argmax_keys=_ptr(self.keys), argmax_offset=self.plan.vocab_rows[0],
                                    plan_rows=plan(cfg.vocab))

    def _descs_all(self):
        out = [self.head_desc]
        for group in self.descs:
            out.extend(group)
        return out

    # ------------------------------------------------------------------- launch
    def _allreduce(self, t, op=None):
        import torch.distributed as dist

        dist.all_reduce(t, op=op or dist.ReduceOp.SUM, group=self.group)

    def residual(self):
        """The residual stream after the last step's layers, [batch, hidden] bf16 (device)."""
        return self.stepper.x.view(1, -1) if self.engine == "step" else self.x

    def run_layers(self, n):
        """Enqueue the embedding and the first ``n`` layers of a step on the current
        stream (no lm_head, no cache-position advance); ``residual()`` then holds
        layer n's output. Used to compare layer outputs with the oracle."""
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.engine == "step":
            self.stepper.run_layers(n, stream)
            return
        self.step(lm_head=False, advance=False, layers=n)

    def step(self, *, lm_head=True, advance=True, layers=None):
        """Enqueue one decode step on the current stream (token in ``tokens``);
        ``layers`` (launch engine) stops after that many layers."""
        cfg, b = self.cfg, self.batch
        L = lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self.engine == "step":
            # one persistent kernel: every layer, the lm_head and the argmax key
            self.stepper.run(stream)
            if advance:
                check(L.sb_decode_advance(_ptr(self.keys), _ptr(self.tokens), _ptr(self.positions), b, 1, stream),
                      "advance")
            return
        d = cfg.head_dim
        tp = self.world > 1
        check(L.sb_embed_rows(_ptr(self.embed), _ptr(self.tokens), _ptr(self.x), b, cfg.hidden, cfg.vocab, stream),
              "embed")
        scale = 1.0 / math.sqrt(d)
        for li, (qkv, o, gateup, down) in enumerate(self.descs[:layers]):
            check(L.sb_linear_ex(ctypes.byref(qkv), stream), "qkv_rope")
            if not self.fused_append:
                check(L.sb_kv_append_int8(_ptr(self.k_new), _ptr(self.v_new), _ptr(self.k_cache[li]),
                                          _ptr(self.k_scale[li]), _ptr(self.v_cache[li]), _ptr(self.v_scale[li]), b,
                                          self.hkv, 1, d, self.capacity, _ptr(self.positions), stream), "kv_append")
            check(L.sb_int8_sdpa_decode_dev(_ptr(self.q), _ptr(self.k_cache[li]), _ptr(self.k_scale[li]),
                                            _ptr(self.v_cache[li]), _ptr(self.v_scale[li]), _ptr(self.attn), b,
                                            self.hq, self.hkv, _ptr(self.positions), 1, self.capacity,
                                            self.capacity, d, scale, 1,
                                            cfg.num_kv_heads if self.invariant else 0, self.workspace.data_ptr(),
                                            self.workspace.numel(), stream), "int8_sdpa")
            check(L.sb_linear_ex(ctypes.byref(o), stream), "o_proj")
            if tp and not self.fused_allreduce:
                self._allreduce(self.part)
                check(L.sb_residual_add(_ptr(self.x), _ptr(self.part), b * cfg.hidden, stream), "residual")
            check(L.sb_linear_ex(ctypes.byref(gateup), stream), "gate_up")
            check(L.sb_linear_ex(ctypes.byref(down), stream), "down")
            if tp and not self.fused_allreduce:
                self._allreduce(self.part)
                check(L.sb_residual_add(_ptr(self.x), _ptr(self.part), b * cfg.hidden, stream), "residual")
        if lm_head:
            check(L.sb_linear_ex(ctypes.byref(self.head_desc), stream), "lm_head")
            if tp:
                import torch.distributed as dist

                # the keys compare unsigned; the collective compares int64: flip the top bit around it
                self.keys.bitwise_xor_(tensor_parallel.SIGN_FLIP)
                self._allreduce(self.keys, dist.ReduceOp.MAX)
                self.keys.bitwise_xor_(tensor_parallel.SIGN_FLIP)
        if advance:
            check(L.sb_decode_advance(_ptr(self.keys), _ptr(self.tokens), _ptr(self.positions), b, 1, stream),
                  "advance")

    def kernels_per_step(self):
        """Number of this library's kernel launches in one ``step()``."""
        if self.engine == "step":
            return 2  # the decode-step kernel + the token/position advance
        per_layer = (5 if self.fused_append else 6) + (2 if self.world > 1 and not self.fused_allreduce else 0)
        return 1 + self.cfg.num_layers * per_layer + 2

    # ------------------------------------------------------------------ drivers
    def reset(self, first_tokens):
        """Start a sequence: empty cache, position 0, first input tokens [batch]."""
        self.positions.zero_()
        self.keys.zero_()
        self.tokens.copy_(torch.as_tensor(first_tokens, dtype=torch.int32, device=self.device).reshape(-1))

    def prefill(self, prompt, *, chunk=PREFILL_CHUNK):
        """Feed prompt[:, 0..P-1]; leaves the greedy next token in ``tokens``.

        ``prompt`` is an int32 device tensor [batch, P]; positions end at P.
        One GPU: the prompt runs in chunks of ``chunk`` tokens (the reference's
        prompt chunk, ``generation.py:78``) through the batched path - tensor-core
        linears at M = batch x chunk, RoPE and the INT8 cache append per chunk,
        and the INT8-KV prefill attention (bottom-right causal over the cache).
        Tensor-parallel ranks, or ``chunk=0``, feed it token by token
        (``prefill_stepwise``).
        """
        prompt = prompt.to(device=self.device, dtype=torch.int32)
        if self.world > 1 or not chunk:
            self.prefill_stepwise(prompt)
            return
        self._prefill_chunked(prompt, int(chunk))

    def prefill_stepwise(self, prompt):
        """Feed the prompt through single-token decode steps (the lm_head only on
        the last one); positions end at P."""
        prompt = prompt.to(device=self.device, dtype=torch.int32)
        self.reset(prompt[:, 0])
        for t in range(prompt.shape[1]):
            last = t == prompt.shape[1] - 1
            self.step(lm_head=last, advance=True)
            if not last:
                self.tokens.copy_(prompt[:, t + 1])
        # positions[b] == P now; tokens holds the first generated token

    def _prefill_buffers(self, rows):
        """Activation buffers for `rows` prompt tokens (grown on demand, kept)."""
        cfg, dev = self.cfg, self.device
        have = getattr(self, "_pf", None)
        if have is not None and have["rows"] >= rows:
            return have
        d, hq, hkv = cfg.head_dim, self.hq, self.hkv
        nqkv = (hq + 2 * hkv) * d

        def buf(*shape):
            return torch.empty(shape, dtype=torch.bfloat16, device=dev)

        L = lib()
        ws = max(L.sb_w8a16_per_channel_workspace_size(rows, nqkv, cfg.hidden),
                 L.sb_w8a16_per_channel_workspace_size(rows, cfg.hidden, hq * d),
                 L.sb_affine_linear_workspace_size(rows, self.inter, cfg.hidden, cfg.mlp_group, 4),
                 L.sb_affine_linear_workspace_size(rows, cfg.hidden, self.inter, cfg.mlp_group, 4))
        self._pf = dict(rows=rows, x=buf(rows, cfg.hidden), xn=buf(rows, cfg.hidden), qkv=buf(rows, nqkv),
                        q=buf(rows, hq * d), attn=buf(rows, hq * d), o=buf(rows, cfg.hidden),
                        g=buf(rows, self.inter), u=buf(rows, self.inter), act=buf(rows, self.inter),
                        ws=torch.zeros(max(ws, 256), dtype=torch.uint8, device=dev))
        return self._pf

    def _prefill_chunked(self, prompt, chunk):
        b, cap, hidden = self.batch, self.capacity, self.cfg.hidden
        total = prompt.shape[1]
        if total < 1 or total > cap:
            raise ValueError(f"prompt length {total} must be in [1, capacity {cap}]")
        if chunk < 1:
            raise ValueError("chunk must be positive")
        L = lib()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        t = self._prefill_buffers(b * min(chunk, total))
        self.reset(prompt[:, 0])
        for c0 in range(0, total, chunk):
            lc = min(chunk, total - c0)
            x = self._forward_rows(prompt[:, c0:c0 + lc], c0, t, stream)
            if c0 + lc == total:
                self.x.copy_(x.view(b, lc, hidden)[:, lc - 1])
        self.positions.fill_(total)
        check(L.sb_linear_ex(ctypes.byref(self.head_desc), stream), "lm_head")
        check(L.sb_decode_advance(_ptr(self.keys), _ptr(self.tokens), _ptr(self.positions), b, 0, stream), "advance")

    def _forward_rows(self, ids2d, c0, t, stream):
        """Every layer for tokens ``ids2d [batch, lc]`` at positions c0..c0+lc-1
        (their K/V appended to the cache, attention causal over positions <=
        each row's); returns the output rows [batch * lc, hidden] (a view of
        the buffers ``t``)."""
        cfg, b = self.cfg, self.batch
        d, hq, hkv, cap = cfg.head_dim, self.hq, self.hkv, self.capacity
        L = lib()
        nqkv = (hq + 2 * hkv) * d
        hidden, inter, group = cfg.hidden, self.inter, cfg.mlp_group
        scale = 1.0 / math.sqrt(d)
        ws, wsb = t["ws"].data_ptr(), t["ws"].numel()
        lc = ids2d.shape[1]
        m = b * lc
        ids = ids2d.reshape(-1).to(self.device, torch.int32).contiguous()
        pos = torch.arange(c0, c0 + lc, device=self.device, dtype=torch.int32).repeat(b)
        x, xn, qkv, q, attn, o = (t[k][:m] for k in ("x", "xn", "qkv", "q", "attn", "o"))
        g, u, act = (t[k][:m] for k in ("g", "u", "act"))
        check(L.sb_embed_rows(_ptr(self.embed), _ptr(ids), _ptr(x), m, hidden, cfg.vocab, stream), "embed")
        for li, layer in enumerate(self.layers):
            kc, ks, vc, vs = self.k_cache[li], self.k_scale[li], self.v_cache[li], self.v_scale[li]
            check(L.sb_rms_norm(_ptr(x), _ptr(layer["in_norm"]), _ptr(xn), BF16, m, hidden, cfg.rms_eps, stream),
                  "rms_norm")
            check(L.sb_w8a16_per_channel(_ptr(xn), BF16, _ptr(layer["qkv_w"]), _ptr(layer["qkv_s"]), _ptr(qkv),
                                         m, nqkv, hidden, ws, wsb, stream), "qkv")
            check(L.sb_rope_kv_append(_ptr(qkv), nqkv, _ptr(pos), _ptr(q), _ptr(kc), _ptr(ks), _ptr(vc),
                                      _ptr(vs), b, lc, hq, hkv, d, cap, d, cfg.rope_theta, stream), "rope")
            check(L.sb_int8_sdpa_prefill(_ptr(q), _ptr(kc), _ptr(ks), _ptr(vc), _ptr(vs), _ptr(attn), b, hq, hkv,
                                         lc, c0 + lc, cap, d, scale, 1, 1, stream), "prefill attention")
            check(L.sb_w8a16_per_channel(_ptr(attn), BF16, _ptr(layer["o_w"]), _ptr(layer["o_s"]), _ptr(o), m,
                                         hidden, hq * d, ws, wsb, stream), "o_proj")
            check(L.sb_residual_add(_ptr(x), _ptr(o), m * hidden, stream), "residual")
            check(L.sb_rms_norm(_ptr(x), _ptr(layer["post_norm"]), _ptr(xn), BF16, m, hidden, cfg.rms_eps,
                                stream), "rms_norm")
            for (w, sc, bi), out in ((layer["gate"], g), (layer["up"], u)):
                check(L.sb_affine_linear(_ptr(xn), BF16, _ptr(w), _ptr(sc), _ptr(bi), _ptr(out), m, inter, hidden,
                                         group, 4, ws, wsb, stream), "gate/up")
            check(L.sb_swiglu(_ptr(g), _ptr(u), _ptr(act), m * inter, stream), "swiglu")
            dw, ds, db = layer["down"]
            check(L.sb_affine_linear(_ptr(act), BF16, _ptr(dw), _ptr(ds), _ptr(db), _ptr(o), m, hidden, inter,
                                     group, 4, ws, wsb, stream), "down")
            check(L.sb_residual_add(_ptr(x), _ptr(o), m * hidden, stream), "residual")
        return x

    def verify(self, tokens):
        """Speculative verification (the target pass of a draft-and-verify loop,
        ``dspark/generation.py:30-60``; batch 1, one GPU): run ``tokens`` = [anchor,
        *draft] (1 to 8 ids) at positions ``positions[0]`` onward in one
        multi-position pass - the M <= 8 weight-streaming kernels and the causal
        multi-query attention over the INT8 cache - and return the greedy token
        after each of them (host list, lowest index on ties). Their K/V rows are
        written to the cache; rows past the accepted prefix are overwritten by
        the next pass. Positions and tokens are not advanced (``commit``)."""
        if self.batch != 1 or self.world != 1:
            raise ValueError("verification runs at batch 1 on one GPU")
        ids = torch.as_tensor(tokens, dtype=torch.int32).reshape(1, -1)
        k1 = ids.shape[1]
        if not 1 <= k1 <= 8:
            raise ValueError("verify takes 1 to 8 tokens (the anchor and up to 7 drafts)")
        pos0 = int(self.positions[0])
        if pos0 + k1 > self.capacity:
            raise ValueError("KV cache is full")
        cfg = self.cfg
        stream = torch.cuda.current_stream(self.device).cuda_stream
        t = self._prefill_buffers(8)
        x = self._forward_rows(ids, pos0, t, stream)
        keys = torch.zeros(k1, dtype=torch.int64, device=self.device)
        head = self._desc(x=_ptr(x), M=k1, N=self.vocab_shard, K=cfg.hidden, weight_format=SB_WEIGHT_BF16,
                          weight=_ptr(self.head), norm_weight=_ptr(self.final_norm), epilogue=SB_EPI_ARGMAX,
                          argmax_keys=_ptr(keys), argmax_offset=self.plan.vocab_rows[0],
                          workspace=self.workspace.data_ptr(), workspace_bytes=self.workspace.numel())
        check(lib().sb_linear_ex(ctypes.byref(head), stream), "lm_head (verify)")
        return [tensor_parallel.key_index(int(k) & 0xFFFFFFFFFFFFFFFF) for k in keys.cpu().tolist()]

    def commit(self, next_token, advance):
        """After a verification pass: move the position by ``advance`` (the anchor
        plus the accepted drafts) and make ``next_token`` the next input."""
        self.positions.add_(int(advance))
        self.tokens.fill_(int(next_token))

    def capture(self):
        """Capture one decode step (lm_head, argmax and position advance included)."""
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        saved_pos = self.positions.clone()
        saved_tok = self.tokens.clone()
        with torch.cuda.stream(stream):
            # warm up once outside the graph on the side stream (NCCL needs it), then restore state
            self.step()
            self.positions.copy_(saved_pos)
            self.tokens.copy_(saved_tok)
            self.keys.zero_()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(graph, stream=stream):
            self.step()
        torch.cuda.synchronize(self.device)
        self.graph = graph
        return graph

    def decode(self, steps):
        """Replay the captured step ``steps`` times; returns generated tokens [batch, steps] (device).

        Raises ``SBError`` when a bounded device-side wait gave up during these
        steps (``check_status``); the tokens are then not returned."""
        if self.graph is None:
            self.capture()
        out = torch.empty((self.batch, steps), dtype=torch.int32, device=self.device)
        for i in range(steps):
            out[:, i] = self.tokens
            self.graph.replay()
        self.check_status()
        return out

    def check_status(self):
        """Read (synchronizing) and clear the workspace status word.

        A kernel whose bounded wait ran out (a tensor-parallel peer that stopped
        posting its partial sums, or a copy that never landed) records the
        timeout there and returns with incomplete outputs; the fused exchange
        then skips every later wait. The tokens of such steps are invalid, so
        this raises ``SBError`` (status SB_ETIMEOUT) after clearing the word.
        ``decode`` calls it; callers driving ``step()`` themselves call it
        after synchronizing."""
        words = self.workspace[: 128 * 1024].view(torch.int32)
        status = int(words[STATUS_WORD].item())
        if self.stepper is not None:
            status |= self.stepper.status()
            self.stepper.clear_status()
        if status:
            words[STATUS_WORD] = 0
            if status & 2:
                raise SBError(f"decode step: position outside the KV cache capacity {self.capacity} "
                              f"(status {status:#x}); the steps beyond it did nothing")
            raise SBError(f"decode step: a bounded device-side wait gave up (status {status:#x}); a "
                          "tensor-parallel peer stopped responding - the tokens of these steps are invalid")
