"""Tensor-parallel host logic on CPU: two gloo ranks run the decoder's shard
plan (spark_b200.tp) with plain float arithmetic and exchange exactly what the
GPU decoder exchanges - a sum all-reduce of the o/down partial outputs and a
MAX all-reduce of the lm_head argmax keys (top bit flipped so that the int64
comparison of the collective orders them like the kernel's unsigned keys). The
results must equal the unsharded computation. No GPU involved.
"""

import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
dist = pytest.importorskip("torch.distributed")
mp = pytest.importorskip("torch.multiprocessing")

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [os.path.join(HERE, ".."), os.path.join(HERE, "..", "spark-mlx-llm_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spark_b200 import tp
        from spark_b200.decoder import DecoderConfig

        cfg = DecoderConfig.small()
        sp = tp.plan(cfg, rank, world)
        rng = np.random.default_rng(7)  # every rank draws the same full tensors
        d = cfg.head_dim
        hq_d, kv_d = cfg.num_heads * d, cfg.num_kv_heads * d
        x_attn = rng.standard_normal((2, hq_d)).astype(np.float32)
        wo = rng.standard_normal((cfg.hidden, hq_d)).astype(np.float32) * 0.02
        x_act = rng.standard_normal((2, cfg.intermediate)).astype(np.float32)
        wd = rng.standard_normal((cfg.hidden, cfg.intermediate)).astype(np.float32) * 0.02
        head = rng.standard_normal((cfg.vocab, cfg.hidden)).astype(np.float32)
        h = rng.standard_normal((3, cfg.hidden)).astype(np.float32)
        wq = rng.standard_normal((hq_d, cfg.hidden)).astype(np.float32)
        wk = rng.standard_normal((kv_d, cfg.hidden)).astype(np.float32)

        # o_proj / down_proj: row split over K, then a sum all-reduce
        c0, cn = sp.o_cols
        part_o = torch.from_numpy(np.ascontiguousarray(x_attn[:, c0:c0 + cn] @ wo[:, c0:c0 + cn].T))
        dist.all_reduce(part_o)
        c0, cn = sp.down_cols
        part_d = torch.from_numpy(np.ascontiguousarray(x_act[:, c0:c0 + cn] @ wd[:, c0:c0 + cn].T))
        dist.all_reduce(part_d)

        # QKV column split by heads: each rank's q/k rows are whole heads
        q_local = np.ascontiguousarray(h @ wq[sp.q_rows[0]:sp.q_rows[0] + sp.q_rows[1]].T, dtype=np.float32)
        k_local = np.ascontiguousarray(h @ wk[sp.kv_rows[0]:sp.kv_rows[0] + sp.kv_rows[1]].T, dtype=np.float32)
        q_all = [torch.zeros((3, sp.q_rows[1]), dtype=torch.float32) for _ in range(world)]
        k_all = [torch.zeros((3, sp.kv_rows[1]), dtype=torch.float32) for _ in range(world)]
        dist.all_gather(q_all, torch.from_numpy(q_local))
        dist.all_gather(k_all, torch.from_numpy(k_local))

        # lm_head: vocabulary split, local argmax key, MAX all-reduce of the signed form
        logits = h @ head[sp.vocab_rows[0]:sp.vocab_rows[0] + sp.vocab_rows[1]].T
        logits[1, :] = 3.0  # a tie across ranks: the lowest global index wins
        # rank 0 all negative, rank 1 one positive value: without the top-bit flip
        # the int64 MAX would prefer rank 0's (negative-float) key
        logits[2, :] = -7.0 - np.arange(logits.shape[1])
        if rank == 1:
            logits[2, 5] = 1.0
        keys = []
        for m in range(3):
            j = int(np.argmax(logits[m]))
            keys.append(tp.signed_key(tp.argmax_key(float(logits[m, j]), sp.vocab_rows[0] + j)))
        kt = torch.tensor(keys, dtype=torch.int64)
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
        tokens = [tp.key_index(tp.unsigned_key(int(k))) for k in kt.tolist()]

        if rank == 0:
            full = h @ head.T
            full[1, :] = 3.0
            full[2, :] = np.concatenate([-7.0 - np.arange(sp.vocab_rows[1])] * world)
            full[2, sp.vocab_rows[1] + 5] = 1.0
            np.savez(os.path.join(out_dir, "tp.npz"), o=part_o.numpy(), o_ref=x_attn @ wo.T, d=part_d.numpy(),
                     d_ref=x_act @ wd.T, q=torch.cat(q_all, 1).numpy(), q_ref=h @ wq.T,
                     k=torch.cat(k_all, 1).numpy(), k_ref=h @ wk.T, tokens=np.array(tokens),
                     tokens_ref=np.argmax(full, axis=1))
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_plan_and_reductions(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    r = np.load(tmp_path / "tp.npz")
    np.testing.assert_allclose(r["o"], r["o_ref"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r["d"], r["d_ref"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(r["q"], r["q_ref"], rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(r["k"], r["k_ref"], rtol=1e-5, atol=1e-4)
    np.testing.assert_array_equal(r["tokens"], r["tokens_ref"])
    assert r["tokens"][1] == 0  # tie across ranks -> lowest index
    assert r["tokens"][2] == r["tokens_ref"][2] > 0  # the positive logit on rank 1 wins


def test_plan_partitions_and_rejects_indivisible_configs():
    from spark_b200 import tp
    from spark_b200.decoder import DecoderConfig

    cfg = DecoderConfig()
    for world in (1, 2, 4, 8):
        plans = [tp.plan(cfg, r, world) for r in range(world)]
        assert sum(p.vocab for p in plans) == cfg.vocab
        assert [p.inter_rows[0] for p in plans] == [r * cfg.intermediate // world for r in range(world)]
        assert all(p.inter % cfg.mlp_group == 0 for p in plans)  # whole quantization groups
        assert sum(p.kv_heads for p in plans) == cfg.num_kv_heads
    with pytest.raises(ValueError):
        tp.plan(cfg, 0, 3)
    with pytest.raises(ValueError):
        tp.plan(cfg, 2, 2)


def test_argmax_keys_order_and_sign_flip():
    from spark_b200 import tp

    vals = [(-1.0, 5), (2.0, 9), (2.0, 3), (float("nan"), 0), (-np.inf, 1), (-0.5, 7)]
    keys = [tp.argmax_key(v, i) for v, i in vals]
    assert vals[keys.index(max(keys))] == (2.0, 3)
    signed = [tp.signed_key(k) for k in keys]
    assert all(-(1 << 63) <= s < (1 << 63) for s in signed)
    assert sorted(range(len(keys)), key=lambda i: keys[i]) == sorted(range(len(keys)), key=lambda i: signed[i])
    assert [tp.unsigned_key(s) for s in signed] == keys
    assert tp.key_index(tp.argmax_key(0.5, 12345)) == 12345
