"""Load a Qwen3.5 checkpoint directory straight into the native engine.

The reference runner loads ``Qwen3_5ForConditionalGeneration.from_pretrained``
(``benchmarks/grbeam.py:209-218``) on a directory written by
``benchmarks/prepare_model.py:77-81`` (``save_pretrained``: ``config.json`` plus
safetensors) and then wraps its text model.  :func:`load_adapter` skips the
Transformers model: it reads the text config, picks the text model's tensors
out of the safetensors files (the vision tower is left on disk) and packs them
into :class:`~kadllm_b200.model.HybridModel` on the device.

Each layer's MLP width is taken from its tensors, so checkpoints whose MLPs
were widened by WideTuning and merged with ``to_dense``
(``src/kadllm/widetuning.py:95-127``: the config keeps the original
``intermediate_size``) load as they are.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from .config import HybridConfig
from .model import HybridModel


def _text_config(path: Path) -> HybridConfig:
    raw = json.loads((path / "config.json").read_text())
    text = raw.get("text_config", raw)
    from transformers import Qwen3_5TextConfig

    cfg = HybridConfig.from_hf(Qwen3_5TextConfig(**text))
    tie = raw.get("tie_word_embeddings", text.get("tie_word_embeddings", False))
    return cfg.with_(tie_word_embeddings=bool(tie))


def _tensor_files(path: Path) -> list[Path]:
    index = path / "model.safetensors.index.json"
    if index.exists():
        names = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        return [path / n for n in names]
    files = sorted(path.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors files in {path}")
    return files


def load_weights(path: str | Path, device="cuda") -> tuple[HybridConfig, dict[str, torch.Tensor]]:
    """(config, text-model tensors under Transformers ``Qwen3_5TextModel`` names)."""
    from safetensors import safe_open

    path = Path(path)
    cfg = _text_config(path)
    files = _tensor_files(path)
    keys = {}
    for f in files:
        with safe_open(str(f), framework="pt") as h:
            for k in h.keys():
                keys[k] = f
    # the text model's prefix: whatever precedes its (non-vision) embedding table
    embeds = [k for k in keys if k.endswith("embed_tokens.weight") and "visual" not in k]
    if len(embeds) != 1:
        raise ValueError(f"cannot locate the text model's embedding in {path}")
    prefix = embeds[0][: -len("embed_tokens.weight")]
    wanted = {k[len(prefix):]: k for k in keys if k.startswith(prefix)}
    if not cfg.tie_word_embeddings and "lm_head.weight" in keys:
        wanted["lm_head.weight"] = "lm_head.weight"
    weights: dict[str, torch.Tensor] = {}
    by_file: dict[Path, list[tuple[str, str]]] = {}
    for name, key in wanted.items():
        by_file.setdefault(keys[key], []).append((name, key))
    for f, items in by_file.items():
        with safe_open(str(f), framework="pt", device=str(device)) as h:
            for name, key in items:
                weights[name] = h.get_tensor(key)
    if cfg.tie_word_embeddings is False and "lm_head.weight" not in weights:
        cfg = cfg.with_(tie_word_embeddings=True)  # no separate head stored: the embedding is the head
    return cfg, weights


def load_engine(path: str | Path, device="cuda") -> HybridModel:
    cfg, weights = load_weights(path, device)
    return HybridModel(cfg, weights, device=device)


def load_adapter(path: str | Path, device="cuda"):
    """A GRBeam adapter (``NativeGRBeamAdapter``) over the checkpoint's text model."""
    from .adapters import NativeGRBeamAdapter

    return NativeGRBeamAdapter(load_engine(path, device))
