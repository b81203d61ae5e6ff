"""Generate golden cases of the reference's greedy acceptance rule.

The reference's ``spark_mlx_llm/dspark/acceptance.py`` keeps ``greedy_accept``
(:23-39) on the standard library alone (its MLX imports sit inside the sampled
rule), so the module can be loaded here by file path. Seeded random draft and
target token lists - long and short, all / none / some drafts matching, empty
drafts - plus the rule's invalid inputs are run through it, and the accepted
tokens and counts (or the error class) are written to
``greedy_accept_cases.json`` next to this script; ``tests/test_speculative.py``
checks ``spark_b200.speculative.greedy_accept`` against them.

Run (where the reference tree is present):
    python tests/golden/make_acceptance_golden.py --reference PATH
The GPU box does not have the reference; it uses the committed ``.json``.
"""

import argparse
import importlib.util
import json
import random
from pathlib import Path

HERE = Path(__file__).resolve().parent


def load_acceptance(reference):
    path = Path(reference) / "spark_mlx_llm" / "dspark" / "acceptance.py"
    spec = importlib.util.spec_from_file_location("_ref_acceptance", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def cases(seed=0):
    rng = random.Random(seed)
    out = []
    for _ in range(200):
        k = rng.choice([0, 1, 2, 3, 7, 7, 15])
        vocab = rng.choice([2, 3, 50, 151936])
        target = [rng.randrange(vocab) for _ in range(k + 1)]
        mode = rng.choice(["all", "none", "prefix", "random"])
        if mode == "all":
            draft = target[:k]
        elif mode == "none":
            draft = [(t + 1) % vocab for t in target[:k]]
        elif mode == "prefix":
            cut = rng.randrange(k + 1)
            draft = target[:cut] + [(t + 1) % vocab for t in target[cut:k]]
        else:
            draft = [rng.randrange(vocab) for _ in range(k)]
        out.append((draft, target))
    # invalid inputs: wrong target count, negative ids, non-int ids
    out += [([1, 2], [1, 2]), ([1, 2], [1, 2, 3, 4]), ([], []), ([-1], [0, 1]), ([1], [1, -2]),
            ([1.0], [1, 2]), ([True], [1, 2])]
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference project tree")
    args = parser.parse_args()
    acc = load_acceptance(args.reference)
    records = []
    for draft, target in cases():
        rec = {"draft": draft, "target": target}
        try:
            r = acc.greedy_accept(draft, target)
            rec.update(tokens=list(r.tokens), num_drafted=r.num_drafted, num_accepted=r.num_accepted,
                       num_rejected=r.num_rejected)
        except Exception as e:  # the rule's own validation
            rec["error"] = type(e).__name__
        records.append(rec)
    with open(HERE / "greedy_accept_cases.json", "w") as f:
        json.dump({"source": "spark_mlx_llm/dspark/acceptance.py:23-39 greedy_accept", "cases": records}, f,
                  separators=(",", ":"))
    print(len(records), "cases")


if __name__ == "__main__":
    main()
