"""Greedy draft-and-verify decoding on the GPU (``spark_b200.speculative``;
the reference's DSpark loop, ``dspark/generation.py``, with its greedy
acceptance rule) against the NumPy decoder oracle.

* Every verification prediction inside an accepted prefix (its inputs are the
  committed sequence) equals the oracle's greedy token whenever the oracle's
  top-1/top-2 margin is decisive (the decoder test's criterion).
* Drafting the plain greedy continuation (computed by the single-token decode
  path) is accepted at least 75 % of the time, and the speculative output
  equals that continuation up to the first position where the oracle margin is
  not decisive: the verification pass runs the multi-row kernels, whose fp32
  summation order differs from the single-token kernels', so a near tie may
  resolve the other way (then the two runs continue from different tokens).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.model import OracleDecoder  # noqa: E402

from test_gpu_decoder import oracle_weights  # noqa: E402

pytestmark = pytest.mark.gpu

PROMPT, STEPS, CAP = 16, 40, 96


def _decisive(logits):
    top2 = np.sort(logits)[-2:]
    return top2[1] - top2[0] > 1e-2 * abs(top2[1]) + 1e-3


def test_speculative_greedy_matches_oracle_and_plain_greedy():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200.decoder import DecoderConfig, SyntheticDecoder
    from spark_b200.speculative import speculative_generate

    cfg = DecoderConfig.small(num_layers=3)
    dec = SyntheticDecoder(cfg, batch=1, capacity=CAP, seed=5)
    prompt = torch.from_numpy(np.random.default_rng(2).integers(0, cfg.vocab, (1, PROMPT)).astype(np.int32))
    # plain greedy through the single-token path
    dec.prefill(prompt.cuda())
    plain = [int(dec.tokens[0])]
    for _ in range(STEPS - 1):
        dec.step()
        plain.append(int(dec.tokens[0]))
    # speculative: draft the plain continuation; record every verification pass
    passes = []
    verify = dec.verify

    def recording_verify(tokens):
        pos0 = int(dec.positions[0])
        targets = verify(tokens)
        passes.append((pos0, list(tokens), targets))
        return targets

    dec.verify = recording_verify

    def drafter(history, k):
        n = len(history) - PROMPT  # tokens generated so far
        return plain[n:n + k]

    out, stats = speculative_generate(dec, prompt, STEPS, drafter, num_draft=7)
    assert len(out) == STEPS
    # the oracle over the committed sequence: greedy after every position
    orc = OracleDecoder(oracle_weights(dec), num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads,
                        head_dim=cfg.head_dim, rope_theta=cfg.rope_theta, eps=cfg.rms_eps, group=cfg.mlp_group,
                        capacity=CAP, batch=1)
    seq = prompt.reshape(-1).tolist() + out
    logits_at = {}
    for p in range(PROMPT + STEPS - 1):
        logits_at[p] = orc.step(np.array([seq[p]], np.int32), p)[0]
    checked = 0
    for pos0, tokens, targets in passes:
        for i, tgt in enumerate(targets):
            p = pos0 + i
            if p not in logits_at or seq[p] != tokens[i]:
                break  # past the committed prefix
            if _decisive(logits_at[p]):
                assert tgt == int(np.argmax(logits_at[p])), (p, tgt)
                checked += 1
            if i < len(tokens) - 1 and tgt != tokens[i + 1]:
                break
    assert checked >= STEPS // 2, checked
    assert stats["accepted"] >= 0.75 * stats["drafted"], stats
    first = next((i for i in range(STEPS) if out[i] != plain[i]), STEPS)
    if first < STEPS:
        assert not _decisive(logits_at[PROMPT + first - 1]), first
    print({"stats": stats, "first_divergence": first, "checked": checked})
