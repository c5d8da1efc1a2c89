"""Pin the numpy oracle against fixtures produced by the reference itself."""

import numpy as np
import pytest

from kadllm_b200.config import TINY
from kadllm_b200.synthetic import numpy_weights
from oracle import grbeam_oracle as O
from tests.parity import assert_close_rel, beam_mismatches, bf16_tol, load


def _oracle(dtype):
    w = numpy_weights(TINY, seed=0, init="test")
    if dtype == "bf16":
        w = {k: O.bf16(v) for k, v in w.items()}
    return O.HybridOracle(TINY, w, dtype)


def test_bf16_rounding_matches_known_values():
    x = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -3.14159, 65504.0, 1e-40, np.inf], np.float32)
    got = O.bf16(x)
    # 1+2^-8 is a tie -> even (1.0); 1+1.5*2^-8 rounds up to 1+2^-7
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == 1.0078125 and got[3] == 1.0078125
    assert got[4] == np.float32(-3.140625)
    assert got[5] == 65536.0 and np.isinf(got[7])
    assert np.isnan(O.bf16(np.array([np.nan], np.float32)))[0]


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_model_prefill_and_decode_match_reference(dtype):
    g = load(f"model_{dtype}.npz")
    orc = _oracle(dtype)
    logits, layers = orc.prefill(g["ids"])

    def check(a, b, what):
        if dtype == "fp32":
            np.testing.assert_allclose(a, b, atol=2e-3, rtol=0, err_msg=what)
        else:
            assert_close_rel(a, b, what=what)

    check(logits, g["prefill_logits"], "prefill logits")
    for i, (a, b) in enumerate(layers):
        check(a, g[f"layer{i}_a"], f"layer {i} first prefix tensor")
        check(b, g[f"layer{i}_b"], f"layer {i} second prefix tensor")
    ref_layers = [(g[f"layer{i}_a"], g[f"layer{i}_b"]) for i in range(TINY.num_layers)]
    for step in (1, 2):
        hist = g[f"decode{step}_history"]
        got = orc.decode(hist, g["ids"].shape[1], ref_layers)
        check(got, g[f"decode{step}_logits"], f"decode step {step} logits")


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_model_search_matches_reference(dtype):
    g = load(f"model_{dtype}.npz")
    orc = _oracle(dtype)
    tokens, scores, valid = O.grbeam_search(orc, g["ids"], list(g["widths"]))
    if dtype == "fp32":
        np.testing.assert_array_equal(tokens, g["tokens"])
        np.testing.assert_allclose(scores, g["scores"], atol=1e-4)
    else:
        tol = 2 * bf16_tol(g["decode2_logits"])
        assert beam_mismatches(tokens, scores, g["tokens"], g["scores"], tol) == []
    np.testing.assert_array_equal(valid, g["valid"])


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_ops_match_reference(dtype):
    g = load(f"ops_{dtype}.npz")
    r = O.Rounding(dtype)
    small = 1e-5 if dtype == "fp32" else None
    o = O.gated_delta(g["gd_q"], g["gd_k"], g["gd_v"], g["gd_g"], g["gd_beta"], g["gd_s0"],
                      beam_width=int(g["gd_W"]), out_round=r)
    np.testing.assert_allclose(o, g["gd_out"], atol=small or bf16_tol(g["gd_out"], 1, 0), rtol=0)
    o = O.causal_conv1d(g["cv_x"], g["cv_state"], g["cv_w"], beam_width=int(g["cv_W"]), r=r)
    np.testing.assert_allclose(o, g["cv_out"], atol=small or bf16_tol(g["cv_out"], 1, 0), rtol=0)
    args = (g["at_q"], g["at_pk"], g["at_pv"], g["at_sk"], g["at_sv"])
    W = int(g["at_W"])
    o = O.prefix_attention(*args, beam_width=W, out_round=r)
    np.testing.assert_allclose(o, g["at_out"], atol=small or bf16_tol(g["at_out"], 1, 0), rtol=0)
    o = O.prefix_attention(*args, beam_width=W, prefix_mask=g["at_mask"], out_round=r)
    np.testing.assert_allclose(o, g["at_out_masked"], atol=small or bf16_tol(g["at_out"], 1, 0), rtol=0)
    e = O.prefix_attention(g["at_q"], g["at_pk"][:, :0], g["at_pv"][:, :0], g["at_sk"], g["at_sv"],
                           beam_width=W, out_round=r)
    np.testing.assert_allclose(e, g["at_out_empty"], atol=small or bf16_tol(g["at_out"], 1, 0), rtol=0)
    co, cs = O.chunk_gated_delta_rule(g["ch_q"], g["ch_k"], g["ch_v"], g["ch_g"], g["ch_beta"], r)
    if dtype == "fp32":
        np.testing.assert_allclose(co, g["ch_out"], atol=1e-4, rtol=0)
        np.testing.assert_allclose(cs, g["ch_state"], atol=1e-4, rtol=1e-4)
    else:
        # q/k are L2-normalised in BF16 before the fp32 scan (1-ulp differences in
        # the normalised inputs propagate through the whole recurrence)
        assert_close_rel(co, g["ch_out"], what="chunk scan output")
        assert_close_rel(cs, g["ch_state"], what="chunk scan state")


def _run_fixed(steps, widths, allowed=None):
    B = steps.shape[1]
    history = np.zeros((B, 1, 0), np.int64)
    scores = np.zeros((B, 1), np.float32)
    logits = steps[0, :, 0][:, None, :]
    for step, width in enumerate(widths):
        if step:
            logits = steps[step, :, : history.shape[1]]
        mask = None if allowed is None else allowed(history, logits)
        scores, parents, tokens = O.beam_select(logits, scores, width, mask)
        old = (np.take_along_axis(history, np.repeat(parents[..., None], step, -1), axis=1)
               if step else np.zeros((B, width, 0), np.int64))
        history = np.concatenate([old, tokens[..., None]], -1)
    return history, scores


def _allowed(history, logits):
    m = np.ones(logits.shape, bool)
    m[..., 1::3] = False
    if history.shape[2] >= 1:
        m[:, 0, :] = False
    return m


def test_selection_matches_reference():
    g = load("select.npz")
    # continuous logits: no ties, so beams must be identical
    tok, sc = _run_fixed(g["smooth"], [4, 4, 3])
    np.testing.assert_array_equal(tok, g["smooth_tokens"])
    np.testing.assert_allclose(sc, g["smooth_scores"], atol=1e-5)
    tok, sc = _run_fixed(g["smooth"], [4, 4, 4], _allowed)
    np.testing.assert_array_equal(tok[np.isfinite(sc)], g["smooth_masked_tokens"][np.isfinite(sc)])
    np.testing.assert_allclose(sc, g["smooth_masked_scores"], atol=1e-5)
    np.testing.assert_array_equal(np.isfinite(sc), g["smooth_masked_valid"])
    # quarter-step logits: exact ties everywhere; torch.topk orders ties arbitrarily,
    # so only the selected score multiset is comparable
    tok, sc = _run_fixed(g["coarse"], [4, 4, 3])
    np.testing.assert_allclose(sc, g["coarse_scores"], atol=1e-5)
    tok, sc = _run_fixed(g["coarse"], [4, 4, 4], _allowed)
    np.testing.assert_allclose(sc, g["coarse_masked_scores"], atol=1e-5)
