"""Greedy and speculative-greedy decoding over any model with the
``CirrusModel`` call signature, plus the prompt-lookup drafter.

Same names, arguments and results as the reference
(``cirrus/model/generate.py:28-89``, ``cirrus/decoding/prompt_lookup.py:19-86``):
speculative output is token-identical to greedy output.  The drafter keeps,
for n = min_ngram..max_ngram, a map from each n-gram to the position right
after its latest occurrence, so a draft costs O(max_ngram) per step.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class GenStats:
    steps: int = 0
    tokens: int = 0

    @property
    def tokens_per_step(self) -> float:
        return self.tokens / max(1, self.steps)


class PromptLookupDrafter:
    """Copy drafts: continue the longest recent n-gram match (prompt_lookup.py:19-58)."""

    def __init__(self, max_ngram: int = 4, min_ngram: int = 2, max_draft: int = 12):
        if not 1 <= min_ngram <= max_ngram:
            raise ValueError("need 1 <= min_ngram <= max_ngram")
        self.max_ngram, self.min_ngram, self.max_draft = max_ngram, min_ngram, max_draft
        self.tokens: list = []
        self._after: dict = {n: {} for n in range(min_ngram, max_ngram + 1)}

    def __len__(self) -> int:
        return len(self.tokens)

    def extend(self, tokens) -> None:
        for tok in tokens:
            self.tokens.append(int(tok))
            end = len(self.tokens)
            # index the n-grams that end just before the newest token; their
            # continuation (the newest token) is then known
            for n in range(self.min_ngram, self.max_ngram + 1):
                if end - 1 < n:
                    break
                self._after[n][tuple(self.tokens[end - 1 - n:end - 1])] = end - 1

    def draft(self, k: int | None = None) -> list:
        k = self.max_draft if k is None else min(k, self.max_draft)
        toks = self.tokens
        for n in range(self.max_ngram, self.min_ngram - 1, -1):
            if len(toks) <= n:
                continue
            at = self._after[n].get(tuple(toks[-n:]))
            if at is not None:
                return toks[at:at + k]
        return []


def accept_greedy(draft, target) -> tuple:
    """Longest prefix of ``draft`` that the model's argmax ``target`` agrees with,
    plus the model's own next token (prompt_lookup.py:61-74)."""
    if len(target) != len(draft) + 1:
        raise ValueError("target must have exactly one more position than draft")
    n = 0
    while n < len(draft) and draft[n] == target[n]:
        n += 1
    return n, list(draft[:n]) + [target[n]]


def choose_draft(lookup, mtp, min_lookup: int = 2) -> list:
    """Copy draft when it is long enough, else the MTP draft (prompt_lookup.py:77-86)."""
    if len(lookup) >= min_lookup and len(lookup) >= len(mtp):
        return list(lookup)
    return list(mtp) if mtp else list(lookup)


@torch.no_grad()
def greedy(model, prompt: list, max_new: int, stop=frozenset()):
    """generate.py:28-40."""
    out = model(torch.tensor([prompt]), use_cache=True, n_logits=1)
    gen, stats = [], GenStats()
    while True:
        tok = int(out.logits[0, -1].argmax())
        gen.append(tok)
        stats.steps += 1
        stats.tokens += 1
        if tok in stop or len(gen) >= max_new:
            return gen, stats
        out = model(torch.tensor([[tok]]), cache=out.cache, n_logits=1)


@torch.no_grad()
def speculative_greedy(model, prompt: list, max_new: int, stop=frozenset(), max_draft: int = 8, use_mtp: bool = True,
                       drafter: PromptLookupDrafter | None = None):
    """generate.py:43-89: draft, verify all drafted positions in one forward,
    keep the agreeing prefix; on a partial accept restore the snapshot and
    re-run the accepted prefix (recurrent state cannot be rewound)."""
    drafter = drafter or PromptLookupDrafter(max_draft=max_draft)
    out = model(torch.tensor([prompt]), use_cache=True, n_logits=1)
    cache, h_last = out.cache, out.hidden[:, -1]
    pending = int(out.logits[0, -1].argmax())
    drafter.extend(prompt + [pending])
    gen, stats = [pending], GenStats(steps=1, tokens=1)
    while pending not in stop and len(gen) < max_new:
        mtp = model.mtp_draft(h_last, torch.tensor([pending])) if use_mtp and hasattr(model, "mtp_draft") else []
        draft = choose_draft(drafter.draft(max_draft), mtp)[:max(0, max_new - len(gen) - 1)]
        snapshot = cache.clone() if draft else None
        inp = [pending] + draft
        o = model(torch.tensor([inp]), cache=cache, n_logits=len(inp))
        target = o.logits[0].argmax(-1).tolist()
        n_acc, emit = accept_greedy(draft, target)
        if n_acc < len(draft):
            o = model(torch.tensor([[pending] + draft[:n_acc]]), cache=snapshot, n_logits=1)
        cache, h_last = o.cache, o.hidden[:, -1]
        for i, t in enumerate(emit):
            if t in stop:
                emit = emit[:i + 1]
                break
        gen.extend(emit)
        drafter.extend(emit)
        pending = emit[-1]
        stats.steps += 1
        stats.tokens += len(emit)
    return gen[:max_new], stats
