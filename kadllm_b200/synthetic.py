"""Seeded synthetic weights and inputs (no checkpoints or datasets are available).

Parameter names follow Transformers' ``Qwen3_5TextModel`` so the same dict can be
loaded into that model (``load_state_dict``) and into this package's native
layout.  Two initialisations exist:

``"spec"``  the benchmark initialisation: every matrix (linears, embedding, conv
            taps) N(0, 0.02); RMSNorm ``(1+w)`` weights 0; gated-norm weights 1;
            ``dt_bias`` 1; ``A_log = log(U(0, 16))``.  This matches what
            ``Qwen3_5PreTrainedModel._init_weights`` does, with seed 0 instead of
            the reference runner's 20261024 (``benchmarks/prepare_model.py:78``).
``"test"``  parity-test initialisation with fan-in scaled matrices and non-trivial
            norm / gate parameters, so every term of the arithmetic carries weight
            (N(0, 0.02) weights make most activations vanish and hide errors).
"""

from __future__ import annotations

import numpy as np

from .config import FULL, LINEAR, HybridConfig


def parameter_shapes(cfg: HybridConfig) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every parameter, in a fixed generation order."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    out: list[tuple[str, tuple[int, ...]]] = [("embed_tokens.weight", (cfg.vocab_size, H))]
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers.{i}."
        if kind == LINEAR:
            hv = cfg.linear_num_value_heads
            out += [
                (p + "linear_attn.in_proj_qkv.weight", (cfg.conv_dim, H)),
                (p + "linear_attn.in_proj_z.weight", (cfg.value_dim, H)),
                (p + "linear_attn.in_proj_b.weight", (hv, H)),
                (p + "linear_attn.in_proj_a.weight", (hv, H)),
                (p + "linear_attn.conv1d.weight", (cfg.conv_dim, 1, cfg.linear_conv_kernel_dim)),
                (p + "linear_attn.dt_bias", (hv,)),
                (p + "linear_attn.A_log", (hv,)),
                (p + "linear_attn.norm.weight", (cfg.linear_value_head_dim,)),
                (p + "linear_attn.out_proj.weight", (H, cfg.value_dim)),
            ]
        elif kind == FULL:
            nh, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            out += [
                (p + "self_attn.q_proj.weight", (2 * nh * d, H)),
                (p + "self_attn.k_proj.weight", (nkv * d, H)),
                (p + "self_attn.v_proj.weight", (nkv * d, H)),
                (p + "self_attn.o_proj.weight", (H, nh * d)),
                (p + "self_attn.q_norm.weight", (d,)),
                (p + "self_attn.k_norm.weight", (d,)),
            ]
        out += [
            (p + "mlp.gate_proj.weight", (I, H)),
            (p + "mlp.up_proj.weight", (I, H)),
            (p + "mlp.down_proj.weight", (H, I)),
            (p + "input_layernorm.weight", (H,)),
            (p + "post_attention_layernorm.weight", (H,)),
        ]
    out.append(("norm.weight", (H,)))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (cfg.vocab_size, H)))
    return out


def _kind(name: str) -> str:
    if name.endswith("A_log"):
        return "a_log"
    if name.endswith("dt_bias"):
        return "dt_bias"
    if name.endswith("linear_attn.norm.weight"):
        return "gated_norm"
    if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        return "rms_norm"
    if name.endswith("conv1d.weight"):
        return "conv"
    if name.startswith("embed_tokens") or name.startswith("lm_head"):
        return "embed"
    return "linear"


def numpy_weights(cfg: HybridConfig, seed: int = 0, init: str = "test") -> dict[str, np.ndarray]:
    """Deterministic float32 weights from ``numpy.random.default_rng(seed)``."""
    if init not in ("spec", "test"):
        raise ValueError("init must be 'spec' or 'test'")
    rng = np.random.default_rng(seed)
    weights = {}
    for name, shape in parameter_shapes(cfg):
        kind = _kind(name)
        if kind == "a_log":
            lo = 0.0 if init == "spec" else 1.0
            w = np.log(rng.uniform(lo, 16.0, size=shape).astype(np.float32) + np.float32(1e-30))
        elif kind == "dt_bias":
            w = np.ones(shape, np.float32) if init == "spec" else rng.uniform(-1.0, 1.0, size=shape)
        elif kind == "gated_norm":
            w = np.ones(shape, np.float32) if init == "spec" else 1.0 + 0.1 * rng.standard_normal(shape)
        elif kind == "rms_norm":
            w = np.zeros(shape, np.float32) if init == "spec" else 0.1 * rng.standard_normal(shape)
        elif init == "spec":
            w = 0.02 * rng.standard_normal(shape, dtype=np.float32)
        elif kind == "conv":
            w = 0.5 * rng.standard_normal(shape, dtype=np.float32)
        elif kind == "embed":
            w = 0.5 * rng.standard_normal(shape, dtype=np.float32)
        else:
            w = rng.standard_normal(shape, dtype=np.float32) / np.float32(np.sqrt(shape[-1]))
        weights[name] = np.ascontiguousarray(w, dtype=np.float32)
    return weights


def torch_weights(cfg: HybridConfig, seed: int = 0, device="cuda", dtype=None):
    """Benchmark ("spec") weights generated on ``device`` with a seeded torch generator.

    Faster than :func:`numpy_weights` at 0.8B scale; same distributions as
    ``init="spec"`` but a different random stream.
    """
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    weights = {}
    for name, shape in parameter_shapes(cfg):
        kind = _kind(name)
        if kind == "a_log":
            w = torch.empty(shape, device=device, dtype=torch.float32).uniform_(0.0, 16.0, generator=gen).log_()
        elif kind == "dt_bias" or kind == "gated_norm":
            w = torch.ones(shape, device=device, dtype=torch.float32)
        elif kind == "rms_norm":
            w = torch.zeros(shape, device=device, dtype=torch.float32)
        else:
            w = torch.empty(shape, device=device, dtype=torch.float32).normal_(0.0, 0.02, generator=gen)
        weights[name] = w.to(dtype)
    return weights


def random_prompts(batch: int, length: int, vocab: int, seed: int = 0) -> np.ndarray:
    """Uniform-random token ids ``[batch, length]`` (int64)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=(batch, length), dtype=np.int64)
