"""Step reuse at depth 2: the two-token decode continued from the one-token step.

A beam's first suffix token at the second decode step is its parent's token of
the first decode step, so the parent's per-layer work (projection rows, q / k /
v) is gathered by parent index instead of recomputed.  These tests hold the
continuation to the full two-token replay: the mixer entry point bit for bit,
the engine's decode and the whole search to the same logits and beams."""

import numpy as np
import pytest
import torch

from oracle import grbeam_oracle as O
from tests.parity import assert_close_rel, beam_mismatches

pytestmark = pytest.mark.gpu


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)


@pytest.mark.parametrize("K,H,HV,B,W,Wp", [(128, 4, 16, 2, 33, 20), (64, 2, 4, 3, 8, 8), (128, 16, 16, 2, 256, 256)])
def test_mixer_continue_equals_two_token_replay(K, H, HV, B, W, Wp):
    """kadllm_gdn_mixer_continue(proj_prev, parent, proj) gives exactly the second
    token's rows of kadllm_gdn_mixer_replay over the assembled two-token rows."""
    from kadllm_b200 import _lib

    rng = np.random.default_rng(K + W + Wp)
    kd, vd = H * K, HV * K
    C = 2 * kd + vd
    ld = C + vd + 2 * HV + 8
    bf = torch.bfloat16
    prev = _t(O.bf16(rng.standard_normal((B * Wp, ld)).astype(np.float32)), bf)
    new = _t(O.bf16(rng.standard_normal((B * W, ld)).astype(np.float32)), bf)
    parent = torch.from_numpy(rng.integers(0, Wp, (B, W)).astype(np.int32)).cuda()
    conv_state = _t(O.bf16(rng.standard_normal((B, C, 4)).astype(np.float32)), bf)
    conv_w = _t(O.bf16(0.5 * rng.standard_normal((C, 4)).astype(np.float32)), bf)
    rec = _t(O.bf16(0.3 * rng.standard_normal((B, HV, K, K)).astype(np.float32)), bf)
    a_log = _t(O.bf16(np.log(rng.uniform(1, 16, HV)).astype(np.float32)), torch.float32)
    dt_bias = _t(O.bf16(rng.uniform(-1, 1, HV).astype(np.float32)), torch.float32)
    nw = _t(O.bf16(1 + 0.1 * rng.standard_normal(K).astype(np.float32)), torch.float32)
    s = _lib.stream(new.device)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # the full replay's rows (beam, t): t = 0 the parent's previous-step row, t = 1 the new row
    gidx = (torch.arange(B, device="cuda")[:, None] * Wp + parent.long()).reshape(-1)
    both = torch.stack([prev[gidx], new], 1).reshape(B * W * 2, ld).contiguous()
    full = torch.empty(B * W * 2, vd, dtype=bf, device="cuda")
    _lib.call("kadllm_gdn_mixer_replay", both.data_ptr(), ld, conv_state.data_ptr(), 4, conv_w.data_ptr(),
              rec.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), nw.data_ptr(), 1e-6, full.data_ptr(), B, W, 2,
              H, HV, K, K, None, status.data_ptr(), s)
    cont = torch.empty(B * W, vd, dtype=bf, device="cuda")
    _lib.call("kadllm_gdn_mixer_continue", prev.data_ptr(), parent.data_ptr(), Wp, new.data_ptr(), ld,
              conv_state.data_ptr(), 4, conv_w.data_ptr(), rec.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
              nw.data_ptr(), 1e-6, cont.data_ptr(), B, W, H, HV, K, K, None, status.data_ptr(), s)
    # the first step over the parents with records, then the new tokens only from them
    records = torch.empty(_lib.lib().kadllm_gdn_mixer_record_bytes(B, Wp, HV, K), dtype=torch.uint8, device="cuda")
    first = torch.empty(B * Wp, vd, dtype=bf, device="cuda")
    plain = torch.empty(B * Wp, vd, dtype=bf, device="cuda")
    _lib.call("kadllm_gdn_mixer_replay", prev.data_ptr(), ld, conv_state.data_ptr(), 4, conv_w.data_ptr(),
              rec.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), nw.data_ptr(), 1e-6, first.data_ptr(), B, Wp, 1,
              H, HV, K, K, records.data_ptr(), status.data_ptr(), s)
    _lib.call("kadllm_gdn_mixer_replay", prev.data_ptr(), ld, conv_state.data_ptr(), 4, conv_w.data_ptr(),
              rec.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), nw.data_ptr(), 1e-6, plain.data_ptr(), B, Wp, 1,
              H, HV, K, K, None, status.data_ptr(), s)
    cont_saved = torch.empty(B * W, vd, dtype=bf, device="cuda")
    _lib.call("kadllm_gdn_mixer_continue", prev.data_ptr(), parent.data_ptr(), Wp, new.data_ptr(), ld,
              conv_state.data_ptr(), 4, conv_w.data_ptr(), rec.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
              nw.data_ptr(), 1e-6, cont_saved.data_ptr(), B, W, H, HV, K, K, records.data_ptr(), status.data_ptr(), s)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(cont, full.view(B * W, 2, vd)[:, 1])
    assert torch.equal(first, plain)  # writing the records leaves the first step's output alone
    assert torch.equal(cont_saved, cont)


def test_gather_rows_by_parent():
    from kadllm_b200 import _lib

    B, Wp, W, n = 3, 5, 7, 24
    src = torch.randn(B * Wp, n, device="cuda").bfloat16()
    parent = torch.randint(0, Wp, (B, W), device="cuda", dtype=torch.int32)
    dst = torch.zeros(B * W, 2, n, dtype=torch.bfloat16, device="cuda")
    _lib.call("kadllm_gather_rows", src.data_ptr(), n * 2, parent.data_ptr(), W, Wp, B * W, n * 2, dst.data_ptr(),
              2 * n * 2, _lib.stream(src.device))
    gidx = (torch.arange(B, device="cuda")[:, None] * Wp + parent.long()).reshape(-1)
    assert torch.equal(dst[:, 0], src[gidx])
    assert int(dst[:, 1].abs().sum()) == 0  # the other slot untouched


@pytest.fixture(scope="module")
def mid_engine():
    from kadllm_b200.model import HybridModel
    from tests.test_model_gpu import MID
    from kadllm_b200.synthetic import numpy_weights

    # the benchmark's weight distributions (N(0, 0.02) projections): realistic logits
    w = {k: O.bf16(v) for k, v in numpy_weights(MID, seed=1, init="spec").items()}
    return HybridModel(MID, {k: torch.from_numpy(v) for k, v in w.items()}, device="cuda"), MID


def test_engine_decode_continuation_matches_full_replay(mid_engine):
    """0.8B head shapes (GDN 16 x 128, attention 8q / 2kv x 256): the two-token decode
    from the one-token step's cache equals the full two-token replay."""
    from kadllm_b200.synthetic import random_prompts

    engine, cfg = mid_engine
    B, Wp, W = 2, 12, 16
    ids = torch.from_numpy(random_prompts(B, 90, cfg.vocab_size, seed=3)).cuda()
    _, state = engine.prefill(ids)
    rng = np.random.default_rng(5)
    h1 = torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, Wp, 1))).cuda()
    cache = {}
    engine.decode(h1, state, cache=cache)
    parent = torch.from_numpy(rng.integers(0, Wp, (B, W)).astype(np.int32)).cuda()
    first = torch.gather(h1[..., 0], 1, parent.long())
    h2 = torch.stack([first, torch.from_numpy(rng.integers(0, cfg.vocab_size, (B, W))).cuda()], -1)
    cont = engine.decode(h2, state, reuse=(cache, parent, Wp))
    full = engine.decode(h2, state)
    engine.check()
    assert_close_rel(cont.float().cpu().numpy(), full.float().cpu().numpy(), rel=2e-3, peak=2e-2,
                     what="continued vs full two-token decode")


@pytest.mark.parametrize("widths", [[16, 16, 16], [8, 8, 8, 8], [16, 16], [16], [16, 40, 8], [4, 64, 33]])
def test_search_with_step_reuse_matches_full_replay(mid_engine, widths):
    """The drop-in search (step reuse through decode_select) against the same search
    through the protocol's decode only (full replay of every suffix token), at depths
    1-4: no decode step, one step, the reused second step, and a third (three-token)
    replay after it; and with widths that change between levels (the second step's
    beams read their parents' rows and records across widths)."""
    from kadllm_b200 import grbeam_search
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.grbeam import PrefillResult
    from kadllm_b200.synthetic import random_prompts

    engine, cfg = mid_engine

    class ProtocolOnly:  # no decode_select: the generic loop, full replays
        def prefill(self, ids):
            logits, state = engine.prefill(ids)
            return PrefillResult(logits, state)

        def decode(self, history, state):
            return engine.decode(history, state)

    ids = torch.from_numpy(random_prompts(2, 70, cfg.vocab_size, seed=8)).cuda()
    a = grbeam_search(NativeGRBeamAdapter(engine), ids, widths)
    b = grbeam_search(ProtocolOnly(), ids, widths)
    assert a.tokens.shape == (2, widths[-1], len(widths))
    assert beam_mismatches(a.tokens.cpu().numpy(), a.scores.cpu().numpy(), b.tokens.cpu().numpy(),
                           b.scores.cpu().numpy(), 1e-3) == []
