"""Prompt-lookup drafting, greedy acceptance and draft choice, in plain Python.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``cirrus/decoding/prompt_lookup.py`` without its incremental index:

* ``lookup_draft`` is ``PromptLookupDrafter(max_ngram, min_ngram,
  max_draft).extend(tokens)`` followed by ``.draft(k)`` (``:19-58``).  The
  index maps each n-gram to the position just after its most recent
  occurrence that ends before the newest token (``:35-44``), so the draft for
  the longest n (from ``max_ngram`` down to ``min_ngram``) whose last-n suffix
  occurred before is the tokens that followed the latest earlier occurrence,
  up to ``min(k, max_draft)`` of them (``:46-58``).  Here that occurrence is
  found by scanning the positions from the end.
* ``accept_greedy`` is ``:61-74``; ``choose_draft`` is ``:77-86``.

The B200 drafter (``cb_prompt_lookup_draft``) scans the same positions in
parallel; ``tests/test_gpu_speculative.py`` compares it with this function,
and ``tests/test_oracle.py`` pins this function to the reference's own
drafter through ``tests/golden/decoding_ref.pt``.
"""

from __future__ import annotations


def lookup_draft(tokens, k: int, min_ngram: int = 2, max_ngram: int = 4, max_draft: int | None = None) -> list:
    toks = list(tokens)
    kk = k if max_draft is None else min(k, max_draft)
    n_tok = len(toks)
    for n in range(max_ngram, min_ngram - 1, -1):
        if n_tok < n + 1:
            continue
        key = toks[n_tok - n:]
        for p in range(n_tok - 1, n - 1, -1):  # the n-gram ending just before position p
            if toks[p - n:p] == key:
                return toks[p:p + kk]
    return []


def accept_greedy(draft, target) -> tuple:
    if len(target) != len(draft) + 1:
        raise ValueError("target must have exactly one more position than draft")
    n = 0
    while n < len(draft) and draft[n] == target[n]:
        n += 1
    return n, list(draft[:n]) + [target[n]]


def choose_draft(lookup, mtp, min_lookup: int = 2) -> list:
    if len(lookup) >= min_lookup and len(lookup) >= len(mtp):
        return list(lookup)
    return list(mtp) if mtp else list(lookup)
