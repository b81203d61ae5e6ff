"""Host logic of greedy draft-and-verify decoding (CPU): the acceptance rule of
``dspark/acceptance.py:23-39`` and the prompt-lookup drafter."""

import pytest

from spark_b200.speculative import greedy_accept, prompt_lookup_drafter


def test_greedy_accept_correction_and_bonus():
    r = greedy_accept([5, 6, 7], [5, 6, 9, 1])
    assert r.tokens == (5, 6, 9) and r.num_accepted == 2 and r.num_rejected == 1
    r = greedy_accept([5, 6], [5, 6, 8])  # every draft matched: the bonus token follows
    assert r.tokens == (5, 6, 8) and r.num_accepted == 2
    r = greedy_accept([], [3])
    assert r.tokens == (3,) and r.num_drafted == 0


@pytest.mark.parametrize("draft,target", [([1], [1]), ([1, 2], [1, 2, 3, 4]), ([-1], [0, 0]), ([1.0], [1, 2])])
def test_greedy_accept_rejects_bad_inputs(draft, target):
    with pytest.raises(ValueError):
        greedy_accept(draft, target)


def test_prompt_lookup_drafter():
    d = prompt_lookup_drafter(ngram=3)
    assert d([1, 2, 3, 4, 9, 1, 2, 3], 3) == [4, 9, 1]   # continuation of the earlier "1 2 3"
    assert d([7, 1, 2, 5, 1, 2], 2) == [5, 1]            # shorter n-grams when the long one is new
    assert d([1, 2, 3], 2) == []                          # nothing to copy


def test_greedy_accept_matches_the_reference_cases():
    """The cases of ``tests/golden/greedy_accept_cases.json``, produced by the
    reference's own ``dspark/acceptance.py`` greedy_accept
    (``tests/golden/make_acceptance_golden.py``): same accepted tokens and counts,
    and the same error class on invalid inputs."""
    import json
    import os

    path = os.path.join(os.path.dirname(__file__), "golden", "greedy_accept_cases.json")
    with open(path) as f:
        cases = json.load(f)["cases"]
    assert len(cases) >= 200
    for case in cases:
        if "error" in case:
            with pytest.raises(ValueError):
                greedy_accept(case["draft"], case["target"])
            assert case["error"] == "ValueError"
            continue
        r = greedy_accept(case["draft"], case["target"])
        assert list(r.tokens) == case["tokens"]
        assert (r.num_drafted, r.num_accepted, r.num_rejected) == (
            case["num_drafted"], case["num_accepted"], case["num_rejected"])
