"""The fused LM head + selection: kadllm_gemm_logits writes the logits and every
row's per-chunk statistics, kadllm_beam_select_fused selects from them without a
pass over the logits.  Checked against the unfused path (the same logits through
kadllm_beam_select) and against torch's own log_softmax + topk of the reference
(src/kadllm/grbeam.py:90-95)."""

import numpy as np
import pytest
import torch

from kadllm_b200 import _lib
from tests.parity import beam_mismatches

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,Wp,V,K,W", [(4, 64, 248320, 1024, 256), (3, 16, 10000, 256, 64), (2, 256, 4096, 512, 256)])
def test_fused_selection_matches_unfused_and_torch(B, Wp, V, K, W):
    from kadllm_b200.grbeam import BeamSelector

    dev = torch.device("cuda")
    g = torch.Generator(device="cuda").manual_seed(V + Wp)
    hidden = torch.randn(B * Wp, K, device=dev, generator=g).bfloat16()
    head = (torch.randn(V, K, device=dev, generator=g) * 0.05).bfloat16()
    parent = -torch.rand(B, Wp, device=dev, generator=g).sort(-1, descending=True).values * 3
    parent[0, 3] = -float("inf")  # a dead parent beam contributes no candidates
    hist = torch.randint(0, V, (B, Wp, 2), device=dev, generator=g)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    sel = BeamSelector(B, Wp, dev)
    logits = torch.empty(B * Wp, V, dtype=torch.bfloat16, device=dev)
    _lib.call("kadllm_gemm_logits", hidden.data_ptr(), K, head.data_ptr(), K, logits.data_ptr(), V, B * Wp, V, K,
              sel.workspace.data_ptr(), sel.workspace.numel(), B, Wp, status.data_ptr(), _lib.stream(dev))
    fs, fh, fp = sel.step_fused(logits.view(B, Wp, V), parent, hist, W, parents=True)
    sel.check()

    ref_sel = BeamSelector(B, Wp, dev)
    us, uh, up = ref_sel.step(logits.view(B, Wp, V), parent, hist, W, parents=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # the same logits (the GEMM's main loop is shared), the same candidates: identical up
    # to the order-of-summation difference in each row's log-sum-exp
    torch.testing.assert_close(fs, us, rtol=0, atol=2e-5)
    assert beam_mismatches(fh.cpu().numpy(), fs.cpu().numpy(), uh.cpu().numpy(), us.cpu().numpy(), 2e-5) == []
    # the parents index the previous beams: the gathered history's first entries are theirs
    gathered = torch.gather(hist, 1, fp.long()[..., None].expand(B, W, 2))
    assert torch.equal(gathered, fh[..., :2])
    # the reference's own selection on the same logits (fp32 log_softmax + parent, topk)
    for b in range(B):
        logp = logits.view(B, Wp, V)[b].float().log_softmax(-1) + parent[b, :, None]
        rs, ri = logp.reshape(-1).topk(W)
        torch.testing.assert_close(fs[b], rs, atol=2e-5, rtol=0)
        ref = torch.stack([ri // V, ri % V], -1).cpu().numpy()
        mine = torch.stack([fp[b].long(), fh[b, :, 2]], -1).cpu().numpy()
        assert beam_mismatches(mine[None], fs[b:b + 1].cpu().numpy(), ref[None], rs[None].cpu().numpy(), 2e-5) == []


def test_engine_fused_head_matches_plain_head():
    """The engine's decode with the fused LM head returns the plain head's logits."""
    from kadllm_b200.grbeam import BeamSelector
    from kadllm_b200.model import HybridModel
    from kadllm_b200.synthetic import numpy_weights, random_prompts
    from oracle import grbeam_oracle as O
    from tests.test_model_gpu import MID

    w = {k: O.bf16(v) for k, v in numpy_weights(MID, seed=1, init="spec").items()}
    engine = HybridModel(MID, {k: torch.from_numpy(v) for k, v in w.items()}, device="cuda")
    ids = torch.from_numpy(random_prompts(2, 50, MID.vocab_size, seed=2)).cuda()
    _, state = engine.prefill(ids)
    hist = torch.from_numpy(np.random.default_rng(0).integers(0, MID.vocab_size, (2, 8, 1))).cuda()
    sel = BeamSelector(2, 8, torch.device("cuda"))
    fused = engine.decode(hist, state, select_workspace=sel.workspace)
    plain = engine.decode(hist, state)
    engine.check()
    assert torch.equal(fused, plain)
