"""GRBeam: fixed-depth beam decoding with an immutable, request-sized prefix.

Drop-in for Kadllm's ``src/kadllm/grbeam.py``: the same protocol
(``PrefillResult``, ``GRBeamAdapter``, ``GRBeamResult``, ``Constraint``) and
``grbeam_search`` signature, validation and error messages.  The per-request
host loop of log-softmax + top-k (``src/kadllm/grbeam.py:87-104``) is replaced
by one batched CUDA selection (``csrc/beam_select.cu``) that also gathers the
history; nothing of logits size is allocated.

Adapters that expose ``decode_select(history, state, scores, width, mask)``
(this package's ``Qwen35GRBeamAdapter``) are driven through it so decode and
selection can share buffers; any other adapter goes through the protocol's
``decode`` and the same selection kernels.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any, Protocol

import torch

from . import _lib


@dataclass(frozen=True)
class PrefillResult:
    logits: torch.Tensor  # [B, vocabulary], predicts the first new token
    state: Any


class GRBeamAdapter(Protocol):
    def prefill(self, input_ids: torch.Tensor) -> PrefillResult:
        """Process [B, prompt_length] and save a request-sized prefix."""
        ...

    def decode(self, history: torch.Tensor, state: Any) -> torch.Tensor:
        """Replay [B, W, T] suffix tokens; return [B, W, vocabulary] logits.

        The prefix is read-only. No state from one beam may affect another.
        """
        ...


@dataclass(frozen=True)
class GRBeamResult:
    tokens: torch.Tensor  # [B, final_width, depth]
    scores: torch.Tensor  # unnormalized cumulative full-vocabulary log-prob
    valid: torch.Tensor  # False for unfilled slots under constraints


# Returns a bool mask shaped like the logits; True means allowed (no renormalisation).
Constraint = Callable[[torch.Tensor, torch.Tensor], torch.Tensor]


class BeamSelector:
    """Owns the selection workspace for a batch and runs one step at a time."""

    def __init__(self, batch: int, max_prev_width: int, device: torch.device):
        self.batch = batch
        self.max_prev = max_prev_width
        # sized for the fused selection too: an LM head run through kadllm_gemm_logits writes
        # its chunk statistics here and step_fused selects from them
        nbytes = int(_lib.lib().kadllm_beam_select_workspace_fused(batch, max_prev_width))
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=device)

    def step_fused(self, logits: torch.Tensor, scores: torch.Tensor | None, history: torch.Tensor,
                   width: int, parents: bool = False):
        """Like :meth:`step` for BF16 logits [B, Wp, V] (contiguous) whose chunk statistics
        the LM-head GEMM (``kadllm_gemm_logits``) wrote into this selector's workspace."""
        B, Wp, V = logits.shape
        if Wp > self.max_prev:
            raise ValueError("selection workspace too small for this width")
        depth = history.shape[2]
        old = history.to(torch.int64).contiguous() if depth else None
        parent = None if scores is None else scores.to(torch.float32).contiguous()
        out_scores = torch.empty(B, width, dtype=torch.float32, device=logits.device)
        out_hist = torch.empty(B, width, depth + 1, dtype=torch.int64, device=logits.device)
        out_parent = torch.empty(B, width, dtype=torch.int32, device=logits.device) if parents else None
        _lib.call("kadllm_beam_select_fused", logits.data_ptr(), V, _lib.ptr(parent), _lib.ptr(old),
                  out_scores.data_ptr(), out_hist.data_ptr(), _lib.ptr(out_parent), self.workspace.data_ptr(),
                  self.workspace.numel(), B, Wp, V, width, depth, _lib.stream(logits.device))
        return (out_scores, out_hist, out_parent) if parents else (out_scores, out_hist)

    def step(self, logits: torch.Tensor, scores: torch.Tensor | None, history: torch.Tensor,
             width: int, mask: torch.Tensor | None = None, parents: bool = False):
        """logits [B, Wp, V] -> (scores [B, width] f32, history [B, width, depth+1] int64),
        plus each selected beam's previous-beam index [B, width] int32 with ``parents``."""
        B, Wp, V = logits.shape
        if Wp > self.max_prev:
            raise ValueError("selection workspace too small for this width")
        # row r = b * Wp + w must sit at r * ld elements from the base
        if Wp == 1:
            ld = logits.stride(0) if B > 1 else V
            ok = logits.stride(-1) == 1 and ld >= V
        else:
            ld = logits.stride(1)
            ok = logits.stride(-1) == 1 and ld >= V and (B == 1 or logits.stride(0) == Wp * ld)
        if not ok:
            logits = logits.contiguous()
            ld = V
        depth = history.shape[2]
        old = history.to(torch.int64).contiguous() if depth else None
        parent = None if scores is None else scores.to(torch.float32).contiguous()
        m = None if mask is None else mask.contiguous().view(torch.uint8)
        out_scores = torch.empty(B, width, dtype=torch.float32, device=logits.device)
        out_hist = torch.empty(B, width, depth + 1, dtype=torch.int64, device=logits.device)
        out_parent = torch.empty(B, width, dtype=torch.int32, device=logits.device) if parents else None
        _lib.call(
            "kadllm_beam_select",
            logits.data_ptr(), _lib.dtype_code(logits), ld, _lib.ptr(parent), _lib.ptr(m), _lib.ptr(old),
            out_scores.data_ptr(), out_hist.data_ptr(), _lib.ptr(out_parent), self.workspace.data_ptr(),
            self.workspace.numel(), B, Wp, V, width, depth, _lib.stream(logits.device),
        )
        return (out_scores, out_hist, out_parent) if parents else (out_scores, out_hist)

    def check(self) -> None:
        """Raise if any step overflowed its candidate buffer (synchronises)."""
        import ctypes

        flags = ctypes.c_uint32(0)
        _lib.call("kadllm_beam_select_status", self.workspace.data_ptr(), self.batch, self.max_prev,
                  ctypes.addressof(flags), _lib.stream(self.workspace.device))
        if flags.value & 1:
            raise RuntimeError("beam selection: more than 16384 candidates tied above the threshold")


@torch.no_grad()
def grbeam_search(
    adapter: GRBeamAdapter,
    input_ids: torch.Tensor,
    widths: Sequence[int],
    *,
    allowed: Constraint | None = None,
) -> GRBeamResult:
    """Run GRBeam with a fixed token count and an explicit width per level.

    Same contract as ``src/kadllm/grbeam.py:45-105``.  Call model.eval() first.
    Invalid constrained slots remain marked (score -inf, valid False; their
    tokens are unspecified) rather than invented.
    """
    if input_ids.ndim != 2 or min(input_ids.shape) < 1:
        raise ValueError("input_ids must be nonempty [B, prompt_length]")
    if not widths or any(not isinstance(w, int) or isinstance(w, bool) or w < 1 for w in widths):
        raise ValueError("widths must contain positive integers")
    prefill = adapter.prefill(input_ids)
    return search_from_prefill(adapter, prefill, input_ids.shape[0], widths, allowed=allowed)


@torch.no_grad()
def search_from_prefill(adapter: GRBeamAdapter, prefill: PrefillResult, B: int, widths: Sequence[int], *,
                        allowed: Constraint | None = None, selector: BeamSelector | None = None) -> GRBeamResult:
    """The decode / selection loop of ``grbeam_search`` after the prefill (shared by the
    packed variable-length search and the graphed search).  With a caller-owned
    ``selector`` nothing synchronises the host: the caller checks it (CUDA-graph capture)."""
    if not widths or any(not isinstance(w, int) or isinstance(w, bool) or w < 1 for w in widths):
        raise ValueError("widths must contain positive integers")
    if prefill.logits.ndim != 2 or prefill.logits.shape[0] != B:
        raise ValueError("prefill logits must have shape [B, vocabulary]")
    V = prefill.logits.shape[-1]
    if V < 1:
        raise ValueError("vocabulary must be nonempty")
    _lib.require_cuda(prefill.logits)
    device = prefill.logits.device
    own = selector is None
    if own:
        selector = BeamSelector(B, max([1, *widths[:-1]]), device)
    history = torch.empty(B, 1, 0, dtype=torch.int64, device=device)
    scores = None
    logits = prefill.logits[:, None, :]
    fused = hasattr(adapter, "decode_select") and allowed is None
    for step, width in enumerate(widths):
        current = history.shape[1]
        if width > current * V:
            raise ValueError("beam width exceeds the number of candidate slots")
        if step and fused:
            scores, history = adapter.decode_select(history, prefill.state, scores, width, selector)
            continue
        if step:
            logits = adapter.decode(history, prefill.state)
        if logits.shape != (*history.shape[:2], V):
            raise ValueError("decode logits must be [B, current_width, vocabulary]")
        mask = None
        if allowed is not None:
            mask = allowed(history, logits)
            if mask.shape != logits.shape or mask.dtype != torch.bool:
                raise ValueError("constraint must return a bool mask matching logits")
        scores, history = selector.step(logits, scores, history, width, mask)
        del logits, mask
    end = getattr(adapter, "end_search", None)
    if callable(end):  # release per-search caches the adapter kept between steps
        end()
    if own:
        selector.check()
        check_adapter(adapter)
    return GRBeamResult(history, scores, torch.isfinite(scores))


def check_adapter(adapter) -> None:
    """Raise if the adapter's device kernels reported an error (a tensor-core
    pipeline wait that timed out).  Adapters without a ``check`` have nothing to report."""
    check = getattr(adapter, "check", None)
    if callable(check):
        check()


class GraphedSearch:
    """A whole ``grbeam_search`` over a fixed batch shape captured once as a CUDA graph.

    Every replay runs all of the search's kernels (prefill, decodes, selections)
    from the static input buffer ``ids`` into static outputs; the launches are
    issued by the device, not by the host.  ``__call__(ids)`` copies new prompts in
    first; ``check()`` reads the selection's overflow flag and the adapter's device
    status word (synchronises).  The
    adapter must be this package's (its kernels go to the current stream).
    """

    def __init__(self, adapter, batch: int, prompt_len: int, widths: Sequence[int], device):
        self.adapter, self.widths = adapter, list(widths)
        self.ids = torch.zeros(batch, prompt_len, dtype=torch.int64, device=device)
        self.selector = BeamSelector(batch, max([1, *self.widths[:-1]]), device)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):  # allocations, tables and library workspaces before capture
            for _ in range(2):
                self._search()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.result = self._search()

    def _search(self) -> GRBeamResult:
        prefill = self.adapter.prefill(self.ids)
        return search_from_prefill(self.adapter, prefill, self.ids.shape[0], self.widths, selector=self.selector)

    def __call__(self, ids: torch.Tensor | None = None) -> GRBeamResult:
        if ids is not None:
            self.ids.copy_(ids, non_blocking=True)
        self.graph.replay()
        return self.result

    def check(self) -> None:
        """Raise on a selection overflow or a device error of the adapter's kernels (synchronises)."""
        self.selector.check()
        check_adapter(self.adapter)
