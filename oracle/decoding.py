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


# ------------------------------------------------------------ verifier loops
# The reference's decoding loops (cirrus/model/generate.py:28-40 greedy,
# :43-89 speculative_greedy), restated over any model object with the
# reference's inference surface: model(ids, cache=..., use_cache=..., n_logits=...)
# returning .logits [1, n, V], .hidden [1, n, d] and .cache (with .clone()), and
# model.mtp_draft(h_last, token) -> list of draft tokens.  The tests run them
# over the oracle model (pinned to the reference's own token sequences by
# tests/golden/debug_ref.pt) and over the B200 engine (the drop-in check).

def _argmax_last(out) -> int:
    return int(out.logits[0, -1].argmax())


def greedy_loop(model, prompt, max_new: int, stop=frozenset()) -> list:
    """generate.py:28-40: one forward of the prompt, then one token per forward."""
    import torch

    out = model(torch.tensor([list(prompt)]), use_cache=True, n_logits=1)
    tokens = []
    while True:
        tok = _argmax_last(out)
        tokens.append(tok)
        if tok in stop or len(tokens) >= max_new:
            return tokens
        out = model(torch.tensor([[tok]]), cache=out.cache, n_logits=1)


def speculative_loop(model, prompt, max_new: int, stop=frozenset(), max_draft: int = 8, use_mtp: bool = True,
                     min_ngram: int = 2, max_ngram: int = 4) -> tuple:
    """generate.py:43-89.  Returns (tokens, steps).

    State per step: the pending token (already emitted, not yet in the cache),
    the cache and the hidden state that predicted the pending token.  A step
    drafts (prompt lookup over everything emitted so far, or the MTP head when
    it proposes more), verifies pending + draft in one forward with logits at
    every position, keeps the agreeing prefix plus the model's next token, and
    on a partial acceptance recomputes the cache from a snapshot taken before
    the verify with only pending + the accepted prefix."""
    import torch

    history = list(prompt)
    out = model(torch.tensor([history]), use_cache=True, n_logits=1)
    cache, h_last = out.cache, out.hidden[:, -1]
    pending = _argmax_last(out)
    history.append(pending)
    tokens, steps = [pending], 1
    while pending not in stop and len(tokens) < max_new:
        mtp = model.mtp_draft(h_last, torch.tensor([pending])) if use_mtp else []
        lookup = lookup_draft(history, max_draft, min_ngram, max_ngram, max_draft)
        draft = choose_draft(lookup, mtp)[:max(0, max_new - len(tokens) - 1)]
        before = cache.clone() if draft else None
        row = [pending] + list(draft)
        o = model(torch.tensor([row]), cache=cache, n_logits=len(row))
        verified = o.logits[0].argmax(-1).tolist()
        n_ok, emitted = accept_greedy(draft, verified)
        if n_ok < len(draft):
            o = model(torch.tensor([row[:1 + n_ok]]), cache=before, n_logits=1)
        cache, h_last = o.cache, o.hidden[:, -1]
        for i, t in enumerate(emitted):
            if t in stop:
                emitted = emitted[:i + 1]
                break
        tokens.extend(emitted)
        history.extend(emitted)
        pending = emitted[-1]
        steps += 1
    return tokens[:max_new], steps
