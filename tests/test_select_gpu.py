"""GPU parity of the batched beam-selection kernels and the drop-in search loop."""

import numpy as np
import pytest
import torch

from oracle import grbeam_oracle as O
from tests.parity import beam_mismatches, load

pytestmark = pytest.mark.gpu


class FixedAdapter:
    """Protocol adapter replaying stored logits (depends only on history shape)."""

    def __init__(self, steps, dtype=torch.float32):
        self.steps = torch.from_numpy(steps).cuda().to(dtype)

    def prefill(self, ids):
        from kadllm_b200.grbeam import PrefillResult

        return PrefillResult(self.steps[0, :, 0], None)

    def decode(self, history, state):
        return self.steps[history.shape[2], :, : history.shape[1]]


def _allowed(history, logits):
    m = torch.ones_like(logits, dtype=torch.bool)
    m[..., 1::3] = False
    if history.shape[2] >= 1:
        m[:, 0, :] = False
    return m


def test_search_matches_reference_golden():
    from kadllm_b200.grbeam import grbeam_search

    g = load("select.npz")
    ids = torch.zeros(3, 5, dtype=torch.long, device="cuda")
    r = grbeam_search(FixedAdapter(g["smooth"]), ids, [4, 4, 3])
    np.testing.assert_array_equal(r.tokens.cpu().numpy(), g["smooth_tokens"])
    np.testing.assert_allclose(r.scores.cpu().numpy(), g["smooth_scores"], atol=1e-5)
    r = grbeam_search(FixedAdapter(g["smooth"]), ids, [4, 4, 4], allowed=_allowed)
    fin = np.isfinite(g["smooth_masked_scores"])
    np.testing.assert_array_equal(r.valid.cpu().numpy(), g["smooth_masked_valid"])
    np.testing.assert_array_equal(r.tokens.cpu().numpy()[fin], g["smooth_masked_tokens"][fin])
    np.testing.assert_allclose(r.scores.cpu().numpy(), g["smooth_masked_scores"], atol=1e-5)
    # exact ties everywhere: the selected score multiset must match
    r = grbeam_search(FixedAdapter(g["coarse"]), ids, [4, 4, 3])
    np.testing.assert_allclose(r.scores.cpu().numpy(), g["coarse_scores"], atol=1e-5)


@pytest.mark.parametrize("dtype,B,Wp,V,W", [
    (torch.float32, 3, 16, 5000, 64), (torch.bfloat16, 3, 16, 5000, 64), (torch.float16, 3, 16, 5000, 64),
    (torch.bfloat16, 3, 16, 65536, 256), (torch.bfloat16, 3, 16, 65536, 500), (torch.bfloat16, 3, 16, 65536, 1100),
    (torch.bfloat16, 4, 96, 32768, 256), (torch.bfloat16, 3, 16, 8200, 64), (torch.bfloat16, 2, 16, 10001, 64)])
def test_select_step_matches_oracle_with_tie_rule(dtype, B, Wp, V, W):
    """One step over bf16-quantised logits (many exact ties): scores and the
    lowest-index tie rule must match the oracle's stable top-k exactly.  The
    V = 65536 BF16 cases give every thread of the row-statistics kernel a
    64-element slice, so its per-row top-W pruning bound is finite (W = 256
    and 500, ranks 8 and 16 of each warp's thread maxima) or disabled
    (W = 1100 > 32 x 32 warps); 4 x 96 rows exceed one row per SM, so a row's
    vector maxima are binned from shared memory while the next row streams in.  V = 8200 (1025 vectors) leaves
    one vector in a second table slot, so collect's chunk summary holds a
    partial chunk past the first slot; V = 10001 (not a multiple of 8) takes the
    element-wise statistics path without the summary."""
    from kadllm_b200.grbeam import BeamSelector

    rng = np.random.default_rng(0)
    logits = O.bf16((2 * rng.standard_normal((B, Wp, V))).astype(np.float32))
    if dtype == torch.float16:
        logits = np.float16(logits).astype(np.float32)
    parent = np.sort(-rng.uniform(0, 3, (B, Wp)).astype(np.float32), -1)[:, ::-1].copy()
    parent[1, 5] = -np.inf
    hist = rng.integers(0, V, (B, Wp, 2))
    sel = BeamSelector(B, Wp, torch.device("cuda"))
    t = torch.from_numpy(logits).cuda().to(dtype)
    sc, h = sel.step(t, torch.from_numpy(parent).cuda(), torch.from_numpy(hist).cuda(), W)
    ref_s, ref_p, ref_t = O.beam_select(logits, parent, W)
    np.testing.assert_allclose(sc.cpu().numpy(), ref_s, atol=1e-5, rtol=0)
    hh = h.cpu().numpy()
    np.testing.assert_array_equal(hh[..., -1], ref_t)
    np.testing.assert_array_equal(hh[..., :2], np.take_along_axis(hist, ref_p[..., None].repeat(2, -1), 1))
    sel.check()


def test_select_full_vocab_shape_and_properties():
    """Step shape: 32 requests x 256 beams x 248320 tokens (bf16)."""
    from kadllm_b200.grbeam import BeamSelector

    B, Wp, V, W = 32, 256, 248320, 256
    gen = torch.Generator(device="cuda").manual_seed(0)
    logits = (torch.randn(B, Wp, V, device="cuda", generator=gen) * 0.5).bfloat16()
    parent = -torch.rand(B, Wp, device="cuda", generator=gen).sort(-1, descending=True).values * 4
    # history column = parent index, so the gathered history reveals each parent
    hist = torch.arange(Wp, device="cuda")[None, :, None].expand(B, Wp, 1).contiguous()
    sel = BeamSelector(B, Wp, torch.device("cuda"))
    sc, h = sel.step(logits, parent, hist, W)
    sel.check()
    # reference semantics (src/kadllm/grbeam.py:90-95) on the GPU in fp32
    for b in (0, 7, 19, 31):
        logp = logits[b].float().log_softmax(-1) + parent[b, :, None]
        rs, ri = logp.reshape(-1).topk(W)
        torch.testing.assert_close(sc[b], rs, atol=2e-5, rtol=0)
        mine = h[b].cpu().numpy()  # [W, 2] = (parent, token)
        ref = torch.stack([ri // V, ri % V], -1).cpu().numpy()
        assert beam_mismatches(mine[None], sc[b:b + 1].cpu().numpy(), ref[None], rs[None].cpu().numpy(), 2e-5) == []
    assert bool((sc[:, :-1] >= sc[:, 1:]).all())


def test_oracle_search_on_gpu_selection_with_constraints():
    """grbeam_search with a constraint against the oracle (no ties: smooth logits)."""
    from kadllm_b200.grbeam import grbeam_search

    rng = np.random.default_rng(3)
    steps = (3 * rng.standard_normal((4, 2, 8, 300))).astype(np.float32)
    ids = torch.zeros(2, 3, dtype=torch.long, device="cuda")
    r = grbeam_search(FixedAdapter(steps), ids, [8, 8, 5, 6], allowed=_allowed)
    B = 2
    history = np.zeros((B, 1, 0), np.int64)
    scores = np.zeros((B, 1), np.float32)
    logits = steps[0, :, 0][:, None, :]
    for step, width in enumerate([8, 8, 5, 6]):
        if step:
            logits = steps[step, :, : history.shape[1]]
        mask = np.ones(logits.shape, bool)
        mask[..., 1::3] = False
        if step:
            mask[:, 0, :] = False
        scores, parents, tokens = O.beam_select(logits, scores, width, mask)
        old = np.take_along_axis(history, np.repeat(parents[..., None], step, -1), 1) if step else np.zeros((B, width, 0), np.int64)
        history = np.concatenate([old, tokens[..., None]], -1)
    np.testing.assert_allclose(r.scores.cpu().numpy(), scores, atol=1e-5)
    fin = np.isfinite(scores)
    np.testing.assert_array_equal(r.tokens.cpu().numpy()[fin], history[fin])


@pytest.mark.parametrize("max_prev", [16, 64])
def test_overflow_reported_at_every_width_and_cleared_by_a_new_search(max_prev):
    """More than 16384 candidates tied above the threshold set the overflow flag,
    whether the overflowing step's previous width is below the selector's maximum
    (the first step, Wp = 1) or equal to it; the first step of the next search
    clears it."""
    from kadllm_b200.grbeam import BeamSelector

    B, V, W = 2, 20000, 16
    dev = torch.device("cuda")
    sel = BeamSelector(B, max_prev, dev)
    empty = torch.empty(B, 1, 0, dtype=torch.long, device=dev)
    flat = torch.zeros(B, 1, V, dtype=torch.bfloat16, device=dev)  # 20000 exact ties per request
    sel.step(flat, None, empty, W)
    with pytest.raises(RuntimeError, match="16384"):
        sel.check()
    gen = torch.Generator(device="cuda").manual_seed(0)
    smooth = torch.randn(B, 1, V, device=dev, generator=gen).bfloat16()
    sc, h = sel.step(smooth, None, empty, max_prev)  # a new search: flag cleared
    sel.check()
    flat_wide = torch.zeros(B, max_prev, V, dtype=torch.bfloat16, device=dev)
    sel.step(flat_wide, sc, h, W)  # Wp == max_prev, ties overflow again
    with pytest.raises(RuntimeError, match="16384"):
        sel.check()
