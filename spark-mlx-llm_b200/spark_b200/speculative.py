"""Greedy draft-and-verify decoding on the synthetic decoder.

The reference's DSpark loop (``spark_mlx_llm/dspark/generation.py``) drafts a
few tokens with a small model, verifies them with one target forward over
``[anchor, *draft]`` and keeps the longest prefix the target agrees with plus
the target's own next token (``dspark/acceptance.py:23-39``, greedy rule). Here
the target pass is ``SyntheticDecoder.verify`` (the M <= 8 weight-streaming
kernels and the causal multi-query INT8 attention) and the drafter is any
callable; ``prompt_lookup_drafter`` (copy the continuation of the latest
earlier occurrence of the last n tokens) is a model-free default. The
reference's learned drafter and its cached Markov bias are not part of this
library.
"""

from dataclasses import dataclass
from typing import Callable, Sequence

import torch

__all__ = ["AcceptanceResult", "greedy_accept", "prompt_lookup_drafter", "speculative_generate"]


@dataclass(frozen=True)
class AcceptanceResult:
    tokens: tuple
    num_drafted: int
    num_accepted: int

    @property
    def num_rejected(self):
        return self.num_drafted - self.num_accepted


def greedy_accept(draft_tokens: Sequence[int], target_tokens: Sequence[int]) -> AcceptanceResult:
    """Keep the drafts the target predicted, then the target's token after them
    (the correction, or a bonus token when every draft matched).

    ``target_tokens`` holds one prediction per verified position: after the
    anchor and after each draft (``len(draft) + 1`` of them)."""
    draft, target = tuple(draft_tokens), tuple(target_tokens)
    if len(target) != len(draft) + 1:
        raise ValueError("Need one target prediction per draft token plus a bonus row")
    if any(type(t) is not int or t < 0 for t in (*draft, *target)):
        raise ValueError("Token IDs must be nonnegative integers")
    n = 0
    while n < len(draft) and draft[n] == target[n]:
        n += 1
    return AcceptanceResult(target[:n + 1], len(draft), n)


def prompt_lookup_drafter(ngram: int = 3) -> Callable[[Sequence[int], int], list]:
    """A model-free drafter: find the latest earlier occurrence of the history's
    last ``ngram`` (down to 1) tokens and propose what followed it."""
    def draft(history, k):
        hist = list(history)
        for n in range(min(ngram, len(hist) - 1), 0, -1):
            tail = hist[-n:]
            for start in range(len(hist) - n - 1, -1, -1):
                if hist[start:start + n] == tail:
                    cont = hist[start + n:start + n + k]
                    if cont:
                        return cont
        return []
    return draft


def speculative_generate(decoder, prompt, steps: int, drafter=None, *, num_draft: int = 7):
    """Greedy decode ``steps`` tokens after ``prompt`` ([1, L] ids) with draft and
    verify passes. Returns ``(tokens, stats)``: the generated ids (the first is
    the prompt's greedy continuation) and ``{"passes", "drafted", "accepted"}``."""
    if not 0 <= num_draft <= 7:
        raise ValueError("num_draft must be in [0, 7] (a pass verifies at most 8 positions)")
    drafter = drafter or prompt_lookup_drafter()
    prompt = torch.as_tensor(prompt, dtype=torch.int32)
    decoder.prefill(prompt.to(decoder.device))
    history = prompt.reshape(-1).tolist()
    out = [int(decoder.tokens[0])]
    stats = {"passes": 0, "drafted": 0, "accepted": 0}
    while len(out) < steps:
        room = decoder.capacity - int(decoder.positions[0]) - 1
        k = max(0, min(num_draft, steps - len(out), room))
        draft = [int(t) for t in drafter(history + out, k)][:k]
        targets = decoder.verify([out[-1], *draft])
        res = greedy_accept(draft, targets)
        stats["passes"] += 1
        stats["drafted"] += res.num_drafted
        stats["accepted"] += res.num_accepted
        decoder.commit(res.tokens[-1], res.num_accepted + 1)
        out.extend(res.tokens)
    return out[:steps], stats
