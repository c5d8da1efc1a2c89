"""Two-level conditional semantic-ID (SID) GRBeam on the native engine.

In generative retrieval an item is a short sequence of semantic-ID tokens: a
level-1 token from one codebook, then a level-2 token that must belong to the
level-1 token's group.  Built on ``grbeam_search`` (``src/kadllm/grbeam.py``:
the constraint hook at ``:98-102`` and ``:110-111``):

* :class:`SidCodebook` -- the two codebooks (token ids) and their group maps,
  with a seeded synthetic builder (application codebooks are not part of the
  reference);
* :func:`sid_constraint` -- the tensorised constraint: a device mask that
  allows the level-1 tokens at step 0 and, at step 1, the level-2 tokens of the
  first token's group (no host loop, no per-request Python);
* :class:`SidHeadAdapter` -- an adapter with a SID-only LM head: logits over
  the codebook tokens only (the head rows gathered once, so the last GEMM is
  (n1 + n2) / vocabulary of the full one), history entries are codebook
  positions; scores are then log-probabilities over the SID tokens;
* :func:`grbeam_search_varlen` -- requests with different prompt lengths.  The
  reference adapter takes unpadded ``[B, L]`` prompts only
  (``src/kadllm/adapters/qwen3_5.py:106-110``); here all requests go through
  one packed prefill (per-request offsets in every kernel) and one search, or,
  for adapters without it, are grouped by length; results come back in
  request order.
* :func:`sid_search` -- the two together, returning token ids.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from .grbeam import GRBeamResult, PrefillResult, grbeam_search, search_from_prefill


@dataclass(frozen=True)
class SidCodebook:
    level1: torch.Tensor  # [n1] int64 token ids
    level2: torch.Tensor  # [n2] int64 token ids (disjoint from level1)
    group1: torch.Tensor  # [n1] int64 group of each level-1 token
    group2: torch.Tensor  # [n2] int64 group of each level-2 token

    @staticmethod
    def synthetic(vocab: int, n1: int = 4096, n2: int = 4096, groups: int = 256, seed: int = 0) -> SidCodebook:
        """Seeded stand-in: n1 + n2 distinct token ids drawn from the vocabulary;
        level-1 token i and level-2 token j belong to groups i % groups, j % groups."""
        if n1 < 1 or n2 < 1 or groups < 1 or n1 + n2 > vocab:
            raise ValueError("codebook sizes must be positive and fit the vocabulary")
        gen = torch.Generator().manual_seed(seed)
        ids = torch.randperm(vocab, generator=gen)[: n1 + n2]
        return SidCodebook(ids[:n1].clone(), ids[n1:].clone(), torch.arange(n1) % groups, torch.arange(n2) % groups)

    @property
    def n1(self) -> int:
        return int(self.level1.numel())

    @property
    def tokens(self) -> torch.Tensor:
        """Token id of each codebook position: level-1 positions first, then level-2."""
        return torch.cat([self.level1, self.level2])

    @property
    def position_groups(self) -> torch.Tensor:
        return torch.cat([self.group1, self.group2])

    def to(self, device) -> SidCodebook:
        return SidCodebook(*(t.to(device) for t in (self.level1, self.level2, self.group1, self.group2)))


def sid_constraint(codebook: SidCodebook, *, vocab: int | None = None):
    """Constraint for ``grbeam_search(..., allowed=...)``.

    ``vocab=None``: logits are over codebook positions (:class:`SidHeadAdapter`);
    otherwise over the full vocabulary of that size (tokens outside the
    codebooks are never allowed).  Step 0 allows level 1; step 1 allows the
    level-2 tokens whose group equals the group of the beam's first token.
    """
    cache: dict = {}

    def tables(device):
        if device not in cache:
            cb = codebook.to(device)
            if vocab is None:
                n = cb.tokens.numel()
                level = torch.cat([torch.ones(cb.n1, dtype=torch.int8, device=device),
                                   torch.full((n - cb.n1,), 2, dtype=torch.int8, device=device)])
                group = cb.position_groups
                first_group = cb.group1  # indexed by level-1 position
            else:
                level = torch.zeros(vocab, dtype=torch.int8, device=device)
                level[cb.level1] = 1
                level[cb.level2] = 2
                group = torch.full((vocab,), -1, dtype=torch.int64, device=device)
                group[cb.level1] = cb.group1
                group[cb.level2] = cb.group2
                first_group = group  # indexed by token id
            cache[device] = (level, group, first_group)
        return cache[device]

    def allowed(history: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        level, group, first_group = tables(logits.device)
        B, W, V = logits.shape
        if level.numel() != V:
            raise ValueError("constraint vocabulary does not match the logits")
        step = history.shape[2]
        if step == 0:
            return (level == 1).expand(B, W, V)
        if step == 1:
            g = first_group[history[..., 0].to(logits.device)]  # [B, W]
            return (level == 2) & (group == g[..., None])
        raise ValueError("two-level SID search has two steps")

    return allowed


class SidHeadAdapter:
    """Wrap a native-engine adapter with a SID-only LM head.

    Logits cover the codebook positions only; the decode history holds codebook
    positions, mapped to token ids before the engine embeds them.
    """

    def __init__(self, adapter, codebook: SidCodebook):
        if not hasattr(adapter, "engine"):
            raise TypeError("SidHeadAdapter wraps a kadllm_b200 adapter")
        self.base = adapter
        engine = adapter.engine
        self.codebook = codebook
        self.tokens = codebook.tokens.to(engine.device)
        if int(self.tokens.max()) >= engine.lm_head.shape[0] or int(self.tokens.min()) < 0:
            raise ValueError("codebook token outside the vocabulary")
        self.head = engine.lm_head.index_select(0, self.tokens).contiguous()

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor) -> PrefillResult:
        self.base._check(input_ids)
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must be nonempty unpadded [B,L]")
        logits, state = self.base.engine.prefill(input_ids, head=self.head)
        return PrefillResult(logits, state)

    @torch.no_grad()
    def prefill_varlen(self, prompts) -> PrefillResult:
        for p in prompts:
            self.base._check(p)
            if p.ndim != 1 or p.numel() < 1:
                raise ValueError("each prompt must be a nonempty 1-D tensor")
        logits, state = self.base.engine.prefill_varlen(list(prompts), head=self.head)
        return PrefillResult(logits, state)

    def check(self) -> None:
        """Raise if a tensor-core kernel of the engine reported a timed-out wait (synchronises)."""
        self.base.engine.check()

    @torch.no_grad()
    def decode(self, history: torch.Tensor, state) -> torch.Tensor:
        self.base._check_state(history, state)  # entries are codebook positions (from the selection)
        return self.base.engine.decode(self.tokens[history], state, head=self.head)


def grbeam_search_varlen(adapter, prompts: Sequence[torch.Tensor], widths: Sequence[int], *,
                         allowed=None, streams: int = 1, packed: bool = True) -> GRBeamResult:
    """``grbeam_search`` over requests with their own prompt lengths.

    ``prompts`` are 1-D integer tensors; the result rows follow their order.
    With ``packed`` (and an adapter that has ``prefill_varlen``: this package's
    adapters on head dim 256 / 128-dim GDN heads) all requests share one
    packed prefill and one search.  Otherwise requests of equal length share
    one search (one prefill of ``[group, L]``); with ``streams > 1`` the length
    groups are spread over that many CUDA streams, each driven by its own host
    thread.
    """
    if len(prompts) == 0:
        raise ValueError("prompts must be nonempty")
    groups: dict[int, list[int]] = {}
    for i, p in enumerate(prompts):
        if p.ndim != 1 or p.numel() < 1:
            raise ValueError("each prompt must be a nonempty 1-D tensor")
        groups.setdefault(int(p.numel()), []).append(i)
    if packed and len(groups) > 1 and hasattr(adapter, "prefill_varlen"):
        try:
            pre = adapter.prefill_varlen(list(prompts))
        except NotImplementedError:
            pre = None
        if pre is not None:
            return search_from_prefill(adapter, pre, len(prompts), widths, allowed=allowed)
    order = sorted(groups, reverse=True)  # longest first: the slowest groups start earliest

    def run(length):
        idx = groups[length]
        return idx, grbeam_search(adapter, torch.stack([prompts[i] for i in idx]), widths, allowed=allowed)

    if streams <= 1 or len(order) == 1:
        results = [run(n) for n in order]
    else:
        results = _run_on_streams(run, order, streams, prompts[0].device)
    tokens = scores = valid = None
    for idx, res in results:
        if tokens is None:
            n = len(prompts)
            tokens = res.tokens.new_empty((n, *res.tokens.shape[1:]))
            scores = res.scores.new_empty((n, *res.scores.shape[1:]))
            valid = res.valid.new_empty((n, *res.valid.shape[1:]))
        where = torch.tensor(idx, device=tokens.device)
        tokens[where], scores[where], valid[where] = res.tokens, res.scores, res.valid
    return GRBeamResult(tokens, scores, valid)


def _run_on_streams(run, items, streams: int, device):
    """run(item) for every item, spread round-robin over `streams` CUDA streams, one
    host thread per stream; the caller's stream waits for all of them."""
    from concurrent.futures import ThreadPoolExecutor

    main = torch.cuda.current_stream(device)
    side = [torch.cuda.Stream(device) for _ in range(min(streams, len(items)))]
    for st in side:
        st.wait_stream(main)  # inputs written on the caller's stream

    def worker(k):
        out = []
        with torch.cuda.device(device), torch.cuda.stream(side[k]), torch.inference_mode():
            for item in items[k::len(side)]:
                out.append(run(item))
        return out

    with ThreadPoolExecutor(len(side)) as ex:
        parts = list(ex.map(worker, range(len(side))))
    results = []
    for st, part in zip(side, parts):
        main.wait_stream(st)
        for _, res in part:
            for t in (res.tokens, res.scores, res.valid):
                t.record_stream(main)
        results.extend(part)
    return results


def sid_search(adapter, prompts: Sequence[torch.Tensor], codebook: SidCodebook,
               widths: Sequence[int] = (256, 256), *, sid_head: bool = True, streams: int = 1,
               head: SidHeadAdapter | None = None, packed: bool = True) -> GRBeamResult:
    """Two-level conditional SID search; ``tokens`` holds token ids.

    ``sid_head=True`` scores over the codebook tokens (SID-only head; pass a
    prepared ``head`` to reuse its gathered weights); ``False`` keeps the
    full-vocabulary head and masks it.  ``streams`` as in
    :func:`grbeam_search_varlen`.
    """
    if len(widths) != 2:
        raise ValueError("two-level SID search takes two widths")
    if sid_head:
        head = head or SidHeadAdapter(adapter, codebook)
        res = grbeam_search_varlen(head, prompts, widths, allowed=sid_constraint(codebook), streams=streams,
                                   packed=packed)
        return GRBeamResult(head.tokens[res.tokens], res.scores, res.valid)
    vocab = int(adapter.engine.lm_head.shape[0])
    return grbeam_search_varlen(adapter, prompts, widths, allowed=sid_constraint(codebook, vocab=vocab),
                                streams=streams, packed=packed)
