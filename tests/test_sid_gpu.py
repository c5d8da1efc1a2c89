"""Two-level conditional SID search with per-request prompt lengths against the
oracle (SID-only head = the oracle's logits at the codebook columns; the
constraint restated in numpy), and the full-vocabulary masked variant."""

import numpy as np
import pytest
import torch

from kadllm_b200.sid import SidCodebook, sid_search
from kadllm_b200.synthetic import numpy_weights, random_prompts
from oracle import grbeam_oracle as O
from tests.parity import beam_mismatches, bf16_tol
from tests.test_model_gpu import MID

pytestmark = pytest.mark.gpu

LENGTHS = (70, 40, 70, 100)  # two requests share a length (one grouped search)


@pytest.fixture(scope="module")
def mid_sid():
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.model import HybridModel

    w = {k: O.bf16(v) for k, v in numpy_weights(MID, seed=1, init="test").items()}
    engine = HybridModel(MID, {k: torch.from_numpy(v) for k, v in w.items()}, device="cuda")
    cb = SidCodebook.synthetic(MID.vocab_size, n1=128, n2=128, groups=8, seed=2)
    return NativeGRBeamAdapter(engine), O.HybridOracle(MID, w, "bf16"), cb


class _SidOracle:
    """The oracle model seen through a SID-only head (codebook columns)."""

    def __init__(self, orc, tokens):
        self.orc, self.tokens = orc, tokens

    def prefill(self, ids):
        logits, layers = self.orc.prefill(ids)
        return logits[:, self.tokens], layers

    def decode(self, history, length, layers):
        return self.orc.decode(self.tokens[history], length, layers)[..., self.tokens]


def _np_constraint(level, group, first_group):
    def allowed(history, logits):
        B, W, V = logits.shape
        if history.shape[2] == 0:
            return np.broadcast_to(level == 1, (B, W, V))
        g = first_group[history[..., 0]]
        return (level == 2)[None, None, :] & (group[None, None, :] == g[..., None])
    return allowed


def _prompts():
    return [random_prompts(1, n, MID.vocab_size, seed=20 + i)[0] for i, n in enumerate(LENGTHS)]


@pytest.mark.parametrize("sid_head,streams,packed", [(True, 1, True), (True, 2, False), (False, 1, True)])
def test_sid_search_matches_oracle(mid_sid, sid_head, streams, packed):
    """SID-only head through one packed prefill of all prompts, the same through length
    groups on two CUDA streams, and the full-vocabulary head with the masked selection."""
    adapter, orc, cb = mid_sid
    widths = (16, 16)
    prompts = _prompts()
    res = sid_search(adapter, [torch.from_numpy(p).cuda() for p in prompts], cb, widths, sid_head=sid_head,
                     streams=streams, packed=packed)
    tokens = cb.tokens.numpy()
    n1 = cb.n1
    if sid_head:
        model = _SidOracle(orc, tokens)
        level = np.array([1] * n1 + [2] * (tokens.size - n1), np.int8)
        group = cb.position_groups.numpy()
        allowed = _np_constraint(level, group, cb.group1.numpy())
    else:
        model = orc
        V = MID.vocab_size
        level = np.zeros(V, np.int8)
        level[cb.level1.numpy()] = 1
        level[cb.level2.numpy()] = 2
        group = np.full(V, -1, np.int64)
        group[cb.level1.numpy()] = cb.group1.numpy()
        group[cb.level2.numpy()] = cb.group2.numpy()
        allowed = _np_constraint(level, group, group)
    assert res.tokens.shape == (len(prompts), widths[-1], 2) and bool(res.valid.all())
    got_t, got_s = res.tokens.cpu().numpy(), res.scores.cpu().numpy()
    for i, p in enumerate(prompts):
        tok, sc, valid = O.grbeam_search(model, p[None], widths, allowed=allowed)
        if sid_head:
            tok = tokens[tok]  # positions -> token ids
        assert valid.all()
        # every returned item is a valid two-level SID
        l1 = {int(t): int(g) for t, g in zip(cb.level1, cb.group1)}
        l2 = {int(t): int(g) for t, g in zip(cb.level2, cb.group2)}
        for a, b in got_t[i]:
            assert int(a) in l1 and int(b) in l2 and l1[int(a)] == l2[int(b)]
        # scores within a few BF16 ulps of the logits' scale (this test model's logits
        # reach ~100); other beams only at near-ties
        tol = 4 * bf16_tol(model.prefill(p[None])[0])
        assert beam_mismatches(got_t[i:i + 1], got_s[i:i + 1], tok, sc, tol) == []
