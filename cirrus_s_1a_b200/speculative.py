"""Batched greedy and speculative decoding, kept on the device.

``SpecDecoder`` runs the draft -> verify -> accept loop of the reference's
``speculative_greedy`` (``cirrus/model/generate.py:43-89``) with its
prompt-lookup drafter and greedy acceptance (``cirrus/decoding/prompt_lookup.py
:19-74``; ``use_mtp=False``) for a whole batch of independent sequences, as
three launches per step that are captured once in a CUDA graph:

1. ``cb_prompt_lookup_draft``: each sequence's draft from its own token history
   (prompt + generated tokens), written straight into the verify input;
2. ``cb_forward``: one verify forward of 1 + ``max_draft`` tokens per sequence,
   recording the GDN state after every token (``DeviceCache.enable_snapshots``);
3. ``cb_spec_accept``: the accepted prefix plus the model's next token are
   appended on the device, and the cache is rewound to the accepted prefix
   (position, and the GDN state from its snapshot) instead of the reference's
   re-run of the prefix (``generate.py:76-77``).

The host reads the sequences' remaining budgets every few steps to stop, and
the tokens once at the end.  Every step emits at least one token per unfinished
sequence, and the emitted tokens are the model's greedy tokens: ``max_draft=0``
is the reference's ``greedy`` (``generate.py:28-40``) on the same loop.
Sequences that finish early keep running in the fixed-shape step, with their
results discarded and their position held.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from cirrus_s_1a_b200 import _lib


@dataclass
class DecodeStats:
    """Steps and tokens of one ``SpecDecoder.run`` (``generate.py:17-25`` counts
    the same two numbers per sequence)."""
    steps: int = 0
    tokens: int = 0

    @property
    def tokens_per_step(self) -> float:
        return self.tokens / max(1, self.steps)


class SpecDecoder:
    def __init__(self, engine, cache, max_draft: int = 4, min_ngram: int = 2, max_ngram: int = 4):
        if max_draft < 0 or 1 + max_draft > _lib.CB_MAX_T:
            raise ValueError(f"max_draft must be in [0, {_lib.CB_MAX_T - 1}]")
        self.engine, self.cache = engine, cache
        self.max_draft, self.min_ngram, self.max_ngram = max_draft, min_ngram, max_ngram
        self.T = 1 + max_draft
        dev = engine.device
        B = cache.batch
        if self.T > 1:
            cache.enable_snapshots(self.T)
        self.ld = cache.max_ctx
        self.tokens = torch.zeros(B, self.ld, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.budget = torch.zeros(B, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(B, self.T, dtype=torch.int64, device=dev)
        self.draft_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.argmax = torch.zeros(B, self.T, dtype=torch.int32, device=dev)
        self.emitted = torch.zeros(1, dtype=torch.int64, device=dev)
        self.prompt_lens: list = []
        self.steps = 0
        self.graph = None

    # ------------------------------------------------------------ set-up
    def start(self, prompts, max_new: int, first_tokens=None) -> None:
        """Prefill ``prompts`` (a list of equal-length token lists, or a [B, P]
        tensor) into the cache in one forward and take each sequence's greedy
        token as its first generated token; or, with ``first_tokens``, only
        record ``prompts`` as the token histories of a cache that already holds
        them (for instance a synthetic cache) with those first tokens pending."""
        ids = torch.as_tensor(prompts, dtype=torch.int64)
        if ids.dim() != 2 or ids.shape[0] != self.cache.batch:
            raise ValueError("prompts must be [batch, P] with the cache's batch")
        B, P = ids.shape
        if P + max_new + self.T > self.ld:
            raise ValueError(f"{P} prompt + {max_new} new + {self.T} verify tokens exceed max_ctx {self.ld}")
        if max_new < 1:
            raise ValueError("max_new must be >= 1")
        if first_tokens is None:
            out = self.engine(ids, cache=self.cache, n_logits=1)
            first = out.logits[:, -1].argmax(-1).to(torch.int32)
        else:
            first = torch.as_tensor(first_tokens, dtype=torch.int32, device=self.engine.device).view(B)
        self.tokens.zero_()
        self.tokens[:, :P] = ids.to(self.engine.device, torch.int32)
        self.tokens[:, P] = first
        self.lens.fill_(P + 1)
        self.budget.fill_(max_new - 1)
        self.emitted.fill_(B)
        self.prompt_lens = [P] * B
        self.steps = 1
        self.cache.pos_host = [int(p) for p in self.cache.pos_dev.tolist()]

    def _launch(self, stream: int) -> None:
        L = _lib.lib()
        B = self.cache.batch
        _lib.check(L.cb_prompt_lookup_draft(self.tokens.data_ptr(), self.ld, self.lens.data_ptr(),
                                            self.budget.data_ptr(), B, self.min_ngram, self.max_ngram,
                                            self.max_draft, self.ids.data_ptr(), self.T, self.draft_len.data_ptr(),
                                            stream), "cb_prompt_lookup_draft")
        self.engine.launch(self.cache, self.ids, self.T, self.T, None, None, self.argmax, stream)
        _lib.check(L.cb_spec_accept(C.byref(self.engine.model.desc), C.byref(self.cache.struct()),
                                    self.argmax.data_ptr(), self.ids.data_ptr(), self.draft_len.data_ptr(), self.T,
                                    self.tokens.data_ptr(), self.ld, self.lens.data_ptr(), self.budget.data_ptr(),
                                    self.emitted.data_ptr(), stream), "cb_spec_accept")

    def capture(self) -> None:
        """Capture one step in a CUDA graph (an eager step first sets the kernels'
        attributes; its effects are undone)."""
        dev = self.engine.device
        c = self.cache
        keep = [t.clone() for t in (self.tokens, self.lens, self.budget, self.emitted, c.pos_dev, c.gdn_state,
                                    c.gdn_conv)]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._launch(side.cuda_stream)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self._launch(side.cuda_stream)
        torch.cuda.current_stream(dev).wait_stream(side)
        for dst, src in zip((self.tokens, self.lens, self.budget, self.emitted, c.pos_dev, c.gdn_state, c.gdn_conv),
                            keep):
            dst.copy_(src)
        torch.cuda.synchronize(dev)

    # ------------------------------------------------------------ decoding
    def step(self, n: int = 1) -> None:
        """Run n steps (graph replays once captured, eager launches otherwise)."""
        for _ in range(n):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._launch(torch.cuda.current_stream(self.engine.device).cuda_stream)
            self.steps += 1

    def active(self) -> int:
        """Sequences still generating (reads the budgets: synchronises)."""
        return int((self.budget > 0).sum())

    def run(self, check_every: int = 8, max_steps: int = 1 << 30) -> tuple:
        """Decode until every sequence has its tokens; returns (the generated
        tokens of each sequence, DecodeStats)."""
        done = 1
        while self.active() > 0 and done < max_steps:
            k = min(check_every, max_steps - done)
            self.step(k)
            done += k
        return self.results(), DecodeStats(self.steps, int(self.emitted.item()))

    def results(self) -> list:
        lens = self.lens.tolist()
        toks = self.tokens.cpu()
        self.cache.pos_host = [int(p) for p in self.cache.pos_dev.tolist()]
        return [toks[b, p:lens[b]].tolist() for b, p in enumerate(self.prompt_lens)]
