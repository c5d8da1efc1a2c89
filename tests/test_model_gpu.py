"""End-to-end GPU parity of the native hybrid pipeline (prefill, decode, search)."""

import numpy as np
import pytest
import torch

from kadllm_b200.config import TINY, HybridConfig
from kadllm_b200.synthetic import numpy_weights, random_prompts
from oracle import grbeam_oracle as O
from tests.parity import assert_bf16_as_accurate, assert_close_rel, beam_mismatches, bf16_tol, load

pytestmark = pytest.mark.gpu


def _hf_tiny():
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    w = numpy_weights(TINY, seed=0, init="test")
    model = Qwen3_5TextModel._from_config(Qwen3_5TextConfig(**TINY.to_hf_kwargs()), dtype=torch.bfloat16)
    model.load_state_dict({k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()})
    model = model.eval().cuda()
    head = torch.nn.Linear(TINY.hidden_size, TINY.vocab_size, bias=False).eval()
    head.weight = model.embed_tokens.weight
    return model, head


def test_tiny_model_matches_reference_golden():
    """The tiny CPU-plumbing architecture, BF16, through the drop-in adapter + search."""
    from kadllm_b200 import grbeam_search
    from kadllm_b200.adapters import Qwen35GRBeamAdapter

    g = load("model_bf16.npz")
    g32 = load("model_fp32.npz")  # same weights and prompts, fp32 reference (the exact answer)
    model, head = _hf_tiny()
    adapter = Qwen35GRBeamAdapter(model, head)
    ids = torch.from_numpy(g["ids"]).cuda()
    pre = adapter.prefill(ids)
    assert_bf16_as_accurate(pre.logits.float().cpu().numpy(), g["prefill_logits"], g32["prefill_logits"],
                            what="prefill logits")
    for i, (a, b) in enumerate(pre.state.layers):
        assert_bf16_as_accurate(a.float().cpu().numpy(), g[f"layer{i}_a"], g32[f"layer{i}_a"], what=f"layer {i} a")
        assert_bf16_as_accurate(b.float().cpu().numpy(), g[f"layer{i}_b"], g32[f"layer{i}_b"], what=f"layer {i} b")
    for T in (1, 2, 3):
        hist = torch.from_numpy(g[f"fixed{T}_history"]).cuda()
        got = adapter.decode(hist, pre.state).float().cpu().numpy()
        assert_bf16_as_accurate(got, g[f"fixed{T}_logits"], g32[f"fixed{T}_logits"], what=f"decode T={T}")
    res = grbeam_search(adapter, ids, [8, 8, 8])
    tol = 2 * bf16_tol(g["decode2_logits"])
    assert beam_mismatches(res.tokens.cpu().numpy(), res.scores.cpu().numpy(), g["tokens"], g["scores"], tol) == []
    assert bool(res.valid.all())


MID = HybridConfig(
    vocab_size=2048, hidden_size=1024, intermediate_size=1024,
    layer_types=("linear_attention", "linear_attention", "linear_attention", "full_attention"),
    num_attention_heads=8, num_key_value_heads=2, head_dim=256,
    linear_num_key_heads=16, linear_num_value_heads=16, linear_key_head_dim=128, linear_value_head_dim=128,
    rope_theta=10_000_000.0,
)


@pytest.fixture(scope="module")
def mid():
    from kadllm_b200.model import HybridModel

    w = {k: O.bf16(v) for k, v in numpy_weights(MID, seed=1, init="test").items()}
    engine = HybridModel(MID, {k: torch.from_numpy(v) for k, v in w.items()}, device="cuda")
    return engine, O.HybridOracle(MID, w, "bf16")


def test_qwen35_head_dims_prefill_matches_oracle(mid):
    """0.8B head dims (GDN 16x128, attention 8q/2kv x 256, rotary 64), ragged last chunk."""
    engine, orc = mid
    ids = random_prompts(2, 100, MID.vocab_size, seed=4)
    logits, state = engine.prefill(torch.from_numpy(ids).cuda())
    ref_logits, ref_layers = orc.prefill(ids)
    exact = O.HybridOracle(MID, orc.w, "fp32")
    ex_logits, ex_layers = exact.prefill(ids)
    assert_bf16_as_accurate(logits.float().cpu().numpy(), ref_logits, ex_logits, what="prefill logits")
    for i, ((a, b), (ra, rb), (ea, eb)) in enumerate(zip(state.layers, ref_layers, ex_layers)):
        assert_bf16_as_accurate(a.float().cpu().numpy(), ra, ea, what=f"layer {i} a")
        assert_bf16_as_accurate(b.float().cpu().numpy(), rb, eb, what=f"layer {i} b")


def test_qwen35_head_dims_decode_and_search_match_oracle(mid):
    from kadllm_b200 import grbeam_search
    from kadllm_b200.adapters import NativeGRBeamAdapter

    engine, orc = mid
    ids = random_prompts(2, 70, MID.vocab_size, seed=5)
    _, ref_layers = orc.prefill(ids)
    tids = torch.from_numpy(ids).cuda()
    _, state = engine.prefill(tids)
    hist = np.random.default_rng(0).integers(0, MID.vocab_size, (2, 8, 3))
    got = engine.decode(torch.from_numpy(hist).cuda(), state).float().cpu().numpy()
    ref = orc.decode(hist, 70, ref_layers)
    exact = O.HybridOracle(MID, orc.w, "fp32")
    _, ex_layers = exact.prefill(ids)
    assert_bf16_as_accurate(got, ref, exact.decode(hist, 70, ex_layers), what="decode logits T=3")
    res = grbeam_search(NativeGRBeamAdapter(engine), tids, [8, 8, 8])
    tok, sc, _ = O.grbeam_search(orc, ids, [8, 8, 8])
    tol = 4 * bf16_tol(ref)
    assert beam_mismatches(res.tokens.cpu().numpy(), res.scores.cpu().numpy(), tok, sc, tol) == []


def test_prefix_is_immutable_and_owner_checked(mid):
    from kadllm_b200.adapters import NativeGRBeamAdapter

    engine, _ = mid
    adapter = NativeGRBeamAdapter(engine)
    ids = torch.from_numpy(random_prompts(1, 40, MID.vocab_size, seed=6)).cuda()
    pre = adapter.prefill(ids)
    snap = [tuple(t.clone() for t in layer) for layer in pre.state.layers]
    adapter.decode(torch.zeros(1, 4, 2, dtype=torch.long, device="cuda"), pre.state)
    for layer, old in zip(pre.state.layers, snap):
        for t, o in zip(layer, old):
            assert torch.equal(t, o)
    with pytest.raises(ValueError):
        adapter.decode(torch.zeros(2, 4, 2, dtype=torch.long, device="cuda"), pre.state)
    other = NativeGRBeamAdapter(engine)
    other._owner = object()  # an adapter that did not create this prefix
    with pytest.raises(ValueError):
        other.decode(torch.zeros(1, 4, 2, dtype=torch.long, device="cuda"), pre.state)


def test_packed_prefill_and_decode_match_per_request(mid):
    """Prompts of lengths 70, 40, 100, 65 in one packed prefill (per-request offsets in the
    GDN prefill, the tiled causal attention, RoPE and the K/V tiles) and one decode against
    each request run alone through the same engine."""
    engine, _ = mid
    lens = (70, 40, 100, 65)
    prompts = [torch.from_numpy(random_prompts(1, n, MID.vocab_size, seed=30 + i)[0]).cuda() for i, n in enumerate(lens)]
    logits, state = engine.prefill_varlen(prompts)
    assert state.lengths == lens and state.length == max(lens)
    hist = torch.from_numpy(np.random.default_rng(1).integers(0, MID.vocab_size, (len(lens), 3, 2))).cuda()
    dec = engine.decode(hist, state)
    engine.check()
    for i, p in enumerate(prompts):
        one_logits, one_state = engine.prefill(p[None])
        assert_close_rel(logits[i:i + 1].float().cpu().numpy(), one_logits.float().cpu().numpy(), rel=2e-2,
                         what=f"packed prefill logits, request {i}")
        for j, ((a, b), (oa, ob)) in enumerate(zip(state.layers, one_state.layers)):
            if a.shape[0] == len(lens):  # GDN layer: per-request conv and recurrent state
                assert_close_rel(a[i].float().cpu().numpy(), oa[0].float().cpu().numpy(), rel=2e-2,
                                 what=f"conv state, layer {j}, request {i}")
                assert_close_rel(b[i].float().cpu().numpy(), ob[0].float().cpu().numpy(), rel=2e-2,
                                 what=f"recurrent state, layer {j}, request {i}")
        one_dec = engine.decode(hist[i:i + 1], one_state)
        assert_close_rel(dec[i:i + 1].float().cpu().numpy(), one_dec.float().cpu().numpy(), rel=2e-2,
                         what=f"packed decode logits, request {i}")


def test_graphed_search_matches_eager(mid):
    """A whole search captured as one CUDA graph and replayed (static prompt buffer)
    gives the eager search's beams, for the captured prompts and for new ones."""
    from kadllm_b200 import grbeam_search
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.grbeam import GraphedSearch

    engine, _ = mid
    adapter = NativeGRBeamAdapter(engine)
    widths = [8, 8, 8]
    graphed = GraphedSearch(adapter, 2, 64, widths, torch.device("cuda"))
    for seed in (6, 7):
        ids = torch.from_numpy(random_prompts(2, 64, MID.vocab_size, seed=seed)).cuda()
        got = graphed(ids)
        graphed.check()
        want = grbeam_search(adapter, ids, widths)
        assert torch.equal(got.tokens, want.tokens)
        torch.testing.assert_close(got.scores, want.scores, rtol=0, atol=0)
