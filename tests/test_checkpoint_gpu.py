"""Checkpoint loading straight into the engine (no Transformers model at load time):
a tiny Qwen3_5ForConditionalGeneration (text + vision) saved with save_pretrained,
one MLP widened like WideTuning's to_dense merge (wider gate / up rows, down
columns; the config keeps the original width), loaded with load_adapter and
checked against the oracle on the same weights."""

import numpy as np
import pytest
import torch

from kadllm_b200.config import TINY
from kadllm_b200.synthetic import numpy_weights, random_prompts
from oracle import grbeam_oracle as O
from tests.parity import assert_bf16_as_accurate

pytestmark = pytest.mark.gpu
EXTRA = 128  # extra MLP width of layer 1


def _saved_model(tmp_path):
    from transformers import Qwen3_5Config, Qwen3_5ForConditionalGeneration

    cfg = Qwen3_5Config(text_config=TINY.to_hf_kwargs(),
                        vision_config=dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=1,
                                           out_hidden_size=TINY.hidden_size, num_position_embeddings=16,
                                           patch_size=2))
    torch.manual_seed(0)
    with torch.device("cpu"):  # like benchmarks/prepare_model.py: built and saved on the host
        model = Qwen3_5ForConditionalGeneration(cfg).eval().to(torch.bfloat16)
    text = model.model.language_model
    w = numpy_weights(TINY, seed=3, init="test")
    text.load_state_dict({k: torch.from_numpy(v).to(torch.bfloat16) for k, v in w.items()})
    rng = np.random.default_rng(4)
    mlp = text.layers[1].mlp
    H, I = TINY.hidden_size, TINY.intermediate_size
    for name, shape, dim in (("gate_proj", (EXTRA, H), 0), ("up_proj", (EXTRA, H), 0), ("down_proj", (H, EXTRA), 1)):
        old = getattr(mlp, name)
        extra = torch.from_numpy(0.05 * rng.standard_normal(shape).astype(np.float32)).to(torch.bfloat16)
        weight = torch.cat([old.weight.data, extra], dim=dim)
        new = torch.nn.Linear(weight.shape[1], weight.shape[0], bias=False, dtype=torch.bfloat16)
        new.weight.data.copy_(weight)
        setattr(mlp, name, new)
    assert text.layers[1].mlp.gate_proj.weight.shape == (I + EXTRA, H)
    model.save_pretrained(tmp_path)
    weights = {k: v.detach().float().cpu().numpy() for k, v in text.state_dict().items()}
    weights["lm_head.weight"] = model.lm_head.weight.detach().float().cpu().numpy()
    return weights


def test_load_adapter_matches_oracle_with_widened_mlp(tmp_path):
    from kadllm_b200 import grbeam_search
    from kadllm_b200.checkpoint import load_adapter

    weights = _saved_model(tmp_path)
    adapter = load_adapter(tmp_path, device="cuda")
    assert adapter.engine.layers[1].w_gu.shape[0] == 2 * (TINY.intermediate_size + EXTRA)
    ids = random_prompts(2, 40, TINY.vocab_size, seed=8)
    pre = adapter.prefill(torch.from_numpy(ids).cuda())
    orc = O.HybridOracle(TINY, weights, "bf16")
    exact = O.HybridOracle(TINY, weights, "fp32")
    ref_logits, ref_layers = orc.prefill(ids)
    ex_logits, ex_layers = exact.prefill(ids)
    assert_bf16_as_accurate(pre.logits.float().cpu().numpy(), ref_logits, ex_logits, what="prefill logits")
    hist = np.random.default_rng(2).integers(0, TINY.vocab_size, (2, 4, 2))
    got = adapter.decode(torch.from_numpy(hist).cuda(), pre.state).float().cpu().numpy()
    assert_bf16_as_accurate(got, orc.decode(hist, 40, ref_layers), exact.decode(hist, 40, ex_layers),
                            what="decode logits")
    res = grbeam_search(adapter, torch.from_numpy(ids).cuda(), [4, 4])
    assert bool(res.valid.all())
