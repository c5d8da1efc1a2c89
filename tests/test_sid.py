"""Two-level SID constraint tables and codebook (host logic; no kernels)."""

import torch

from kadllm_b200.sid import SidCodebook, sid_constraint


def _cb():
    return SidCodebook.synthetic(vocab=500, n1=12, n2=24, groups=4, seed=3)


def test_codebook_is_disjoint_and_grouped():
    cb = _cb()
    toks = cb.tokens
    assert toks.numel() == 36 and len(set(toks.tolist())) == 36
    assert int(toks.min()) >= 0 and int(toks.max()) < 500
    assert cb.group1.tolist() == [i % 4 for i in range(12)]
    assert cb.group2.tolist() == [i % 4 for i in range(24)]


def test_sid_head_positions_mask():
    cb = _cb()
    allowed = sid_constraint(cb)
    B, W, V = 2, 3, 36
    m0 = allowed(torch.zeros(B, 1, 0, dtype=torch.int64), torch.zeros(B, 1, V))
    assert m0.shape == (B, 1, V) and m0[..., :12].all() and not m0[..., 12:].any()
    hist = torch.tensor([[[0], [5], [11]], [[2], [3], [7]]])  # level-1 positions
    m1 = allowed(hist, torch.zeros(B, W, V))
    for b in range(B):
        for w in range(W):
            g = int(hist[b, w, 0]) % 4
            want = [(v >= 12) and ((v - 12) % 4 == g) for v in range(V)]
            assert m1[b, w].tolist() == want


def test_full_vocabulary_mask():
    cb = _cb()
    allowed = sid_constraint(cb, vocab=500)
    m0 = allowed(torch.zeros(1, 1, 0, dtype=torch.int64), torch.zeros(1, 1, 500))
    assert sorted(torch.nonzero(m0[0, 0]).flatten().tolist()) == sorted(cb.level1.tolist())
    first = cb.level1[6]  # group 6 % 4 = 2
    m1 = allowed(first.view(1, 1, 1), torch.zeros(1, 1, 500))
    want = sorted(cb.level2[[j for j in range(24) if j % 4 == 2]].tolist())
    assert sorted(torch.nonzero(m1[0, 0]).flatten().tolist()) == want
