"""Tensor-parallel decoder on 2 GPUs (o/down partials added inside the GEMV
epilogue over NVLink peer memory, vocabulary-split lm_head with the
sign-flipped MAX all-reduce of argmax keys) against the same model on one GPU:
with the summation order fixed across degrees (K chunks in a balanced tree,
shards planned as the unsharded matrices) the teacher-forced greedy
predictions are identical. Skipped on boxes with fewer than two GPUs."""

import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_tp2_matches_tp1(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    sys.path.insert(0, HERE)
    import tp_child

    tp1 = tp_child.predictions(1, 0, None, torch.device("cuda", 0))
    out = tmp_path / "tp2.npy"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29517", os.path.join(HERE, "tp_child.py"),
           str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    tp2 = np.load(out)
    assert np.array_equal(tp1, tp2), (float(np.mean(tp1 == tp2)), tp1.T, tp2.T)
