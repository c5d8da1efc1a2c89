"""Checkpoint parsing on the host: the text model's tensors under Transformers
text-model names, the vision tower left out, per-layer MLP widths kept."""

from tests.test_checkpoint_gpu import EXTRA, _saved_model


def test_load_weights_picks_the_text_model(tmp_path):
    from kadllm_b200.checkpoint import load_weights
    from kadllm_b200.config import TINY

    weights = _saved_model(tmp_path)
    cfg, got = load_weights(tmp_path, device="cpu")
    assert cfg.layer_types == TINY.layer_types and cfg.hidden_size == TINY.hidden_size
    assert set(got) == set(weights)  # text model + lm_head, no vision tensors
    assert not any("visual" in k for k in got)
    assert tuple(got["layers.1.mlp.gate_proj.weight"].shape) == (TINY.intermediate_size + EXTRA, TINY.hidden_size)
    assert tuple(got["layers.0.mlp.gate_proj.weight"].shape) == (TINY.intermediate_size, TINY.hidden_size)
    for k in ("embed_tokens.weight", "norm.weight", "layers.3.self_attn.q_proj.weight", "lm_head.weight"):
        assert (got[k].float().numpy() == weights[k]).all()
