"""The reference runner's external-backend path through this package, unchanged:
``benchmarks/grbeam.py --backend external --adapter-factory kadllm_b200.factory:make``
passes the loaded ``Qwen3_5ForConditionalGeneration`` to ``make`` and calls
``search(adapter, ids, [beam] * depth).tokens.tolist()`` with its deterministic
prompts (benchmarks/grbeam.py:219-223,254-257,299).  Here on the tiny BF16
hybrid, checked against the oracle's search and timed eagerly."""

import time

import numpy as np
import pytest
import torch

from kadllm_b200.config import TINY
from kadllm_b200.synthetic import numpy_weights
from oracle import grbeam_oracle as O
from tests.parity import beam_mismatches, bf16_tol

pytestmark = pytest.mark.gpu


def _model():
    from transformers import Qwen3_5Config, Qwen3_5ForConditionalGeneration

    w = {k: O.bf16(v) for k, v in numpy_weights(TINY, seed=0, init="test").items()}
    vision = dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2, out_hidden_size=TINY.hidden_size)
    cfg = Qwen3_5Config(text_config=TINY.to_hf_kwargs(), vision_config=vision, tie_word_embeddings=True)
    model = Qwen3_5ForConditionalGeneration(cfg).to(torch.bfloat16)
    model.model.language_model.load_state_dict({k: torch.from_numpy(v).bfloat16() for k, v in w.items()})
    return model.eval().cuda(), w


def test_runner_external_factory_path():
    from kadllm_b200.factory import make

    model, w = _model()
    adapter, search = make(model)
    B, L, beam, depth = 2, 64, 8, 3
    prompts = [[10 + (i + r * 17) % 100 for i in range(L)] for r in range(B)]
    ids = torch.tensor(prompts, device="cuda")
    with torch.inference_mode():
        tokens = search(adapter, ids, [beam] * depth).tokens.tolist()
        times = []
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            again = search(adapter, ids, [beam] * depth).tokens.tolist()
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
    # the runner's own validation: shape, integer tokens, distinct fixed-depth beams
    assert len(tokens) == B and all(len(req) == beam and all(len(s) == depth for s in req) for req in tokens)
    assert all(len({tuple(s) for s in req}) == beam for req in tokens)
    assert again == tokens  # repeat searches agree
    res = search(adapter, ids, [beam] * depth)
    orc = O.HybridOracle(TINY, w, "bf16")
    ref_tok, ref_sc, _ = O.grbeam_search(orc, np.array(prompts), [beam] * depth)
    tol = 2 * bf16_tol(orc.prefill(np.array(prompts))[0])  # two BF16 ulps of the logits, as the model tests
    assert beam_mismatches(res.tokens.cpu().numpy(), res.scores.cpu().numpy(), ref_tok, ref_sc, tol) == []
    print(f"drop-in search (tiny, B={B}, L={L}, beam {beam}): {1e3 * min(times):.2f} ms eager")
