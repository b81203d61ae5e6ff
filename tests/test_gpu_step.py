"""The persistent decode-step kernel (``sb_step_run``) on the GPU.

* against the NumPy decoder oracle, teacher forced (small shape, batch 1):
  the residual stream after every step within tolerance, and the greedy token
  on every step whose oracle top-1/top-2 gap is decisive;
* against the per-operator launch path of the same weights: greedy tokens
  equal and residual streams close;
* determinism: replaying the same steps gives bit-identical state;
* the launch that follows a prompt: the decode-step engine's tokens after a
  CUDA-graph capture equal eager steps.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.model import OracleDecoder  # noqa: E402

from test_gpu_decoder import oracle_weights  # noqa: E402

pytestmark = pytest.mark.gpu


def _f32(t):
    return t.detach().float().cpu().numpy()


def _decoder(engine, layers=2, capacity=432, seed=3):
    from spark_b200.decoder import DecoderConfig, SyntheticDecoder

    cfg = DecoderConfig.small(num_layers=layers)
    return SyntheticDecoder(cfg, batch=1, capacity=capacity, seed=seed, engine=engine)


@pytest.fixture(scope="module")
def pair():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return _decoder("step"), _decoder("launches")


def test_step_kernel_matches_oracle_teacher_forced(pair):
    dec = pair[0]
    assert dec.engine == "step"
    cfg = dec.cfg
    orc = OracleDecoder(oracle_weights(dec), num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads,
                        head_dim=cfg.head_dim, rope_theta=cfg.rope_theta, eps=cfg.rms_eps, group=cfg.mlp_group,
                        capacity=dec.capacity, batch=1)
    rng = np.random.default_rng(0)
    # 400 positions: several 32-token warp slices and two 352-token attention spans (cross-CTA merge)
    inputs = rng.integers(0, cfg.vocab, 400).astype(np.int32)
    dec.reset(torch.from_numpy(inputs[:1]))
    agree = 0
    for t in range(inputs.shape[0]):
        dec.tokens.copy_(torch.from_numpy(inputs[t:t + 1]).cuda())
        dec.step()
        torch.cuda.synchronize()
        logits = orc.step(inputs[t:t + 1], t)
        np.testing.assert_allclose(_f32(dec.stepper.x)[None], orc.last_x, rtol=2e-2, atol=5e-2)
        top2 = np.sort(logits, axis=-1)[0, -2:]
        if top2[1] - top2[0] > 1e-2 * abs(top2[1]) + 1e-3:
            assert int(dec.tokens[0]) == int(orc.greedy(logits)[0]), t
            agree += 1
        assert int(dec.positions[0]) == t + 1
    assert agree >= 300
    dec.check_status()


def test_step_kernel_matches_launch_path(pair):
    step_dec, ref_dec = pair
    rng = np.random.default_rng(1)
    inputs = rng.integers(0, step_dec.cfg.vocab, 40).astype(np.int32)
    for dec in pair:
        dec.reset(torch.from_numpy(inputs[:1]))
    mism = 0
    for t in range(inputs.shape[0]):
        for dec in pair:
            dec.tokens.copy_(torch.from_numpy(inputs[t:t + 1]).cuda())
            dec.step()
        torch.cuda.synchronize()
        np.testing.assert_allclose(_f32(step_dec.stepper.x), _f32(ref_dec.x)[0], rtol=2e-2, atol=5e-2)
        mism += int(step_dec.tokens[0]) != int(ref_dec.tokens[0])
    assert mism <= 2, mism  # both are fp32 accumulations in different orders; near ties may differ


def test_step_kernel_is_deterministic(pair):
    dec = pair[0]
    rng = np.random.default_rng(2)
    prompt = torch.from_numpy(rng.integers(0, dec.cfg.vocab, (1, 12)).astype(np.int32)).cuda()
    runs = []
    for _ in range(2):
        dec.prefill(prompt)
        toks = [int(dec.tokens[0])]
        for _ in range(10):
            dec.step()
            toks.append(int(dec.tokens[0]))
        torch.cuda.synchronize()
        runs.append((toks, dec.stepper.x.clone(), dec.k_cache[0].clone()))
    assert runs[0][0] == runs[1][0]
    assert torch.equal(runs[0][1], runs[1][1])
    assert torch.equal(runs[0][2], runs[1][2])


def test_step_kernel_graph_replay_matches_eager(pair):
    dec = pair[0]
    rng = np.random.default_rng(3)
    prompt = torch.from_numpy(rng.integers(0, dec.cfg.vocab, (1, 9)).astype(np.int32)).cuda()
    dec.prefill(prompt)
    eager = []
    for _ in range(12):
        eager.append(int(dec.tokens[0]))
        dec.step()
    torch.cuda.synchronize()
    dec.prefill(prompt)
    dec.graph = None
    replayed = dec.decode(12).cpu().numpy()[0].tolist()
    assert replayed == eager


def test_step_kernel_rejects_positions_beyond_the_cache():
    """A step whose position is outside the KV cache writes nothing and reports it."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import SBError

    dec = _decoder("step", layers=1, capacity=16)
    dec.reset(torch.tensor([5], dtype=torch.int32))
    dec.positions.fill_(dec.capacity)
    before = [t.clone() for t in (dec.k_cache[0], dec.v_cache[0], dec.k_scale[0])]
    dec.step()
    torch.cuda.synchronize()
    with pytest.raises(SBError, match="outside the KV cache"):
        dec.check_status()
    for a, b in zip(before, (dec.k_cache[0], dec.v_cache[0], dec.k_scale[0])):
        assert torch.equal(a, b)
    dec.check_status()  # cleared


def test_step_kernel_status_is_sticky_across_launches():
    """A status raised by one launch survives the launches after it until it is read."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import SBError

    dec = _decoder("step", layers=1, capacity=16)
    dec.reset(torch.tensor([5], dtype=torch.int32))
    dec.positions.fill_(dec.capacity)
    dec.step()  # outside the cache: reports and does nothing
    dec.positions.fill_(1)
    for _ in range(3):
        dec.step()  # good steps after it
    torch.cuda.synchronize()
    with pytest.raises(SBError, match="outside the KV cache"):
        dec.check_status()
    dec.check_status()  # cleared
