"""GRBeam adapter for the dense Qwen3.5 text model (drop-in for Kadllm's).

Same constructor, checks and protocol as ``src/kadllm/adapters/qwen3_5.py``:
pass the Transformers ``Qwen3_5TextModel`` and its LM head.  The weights are
packed once into :class:`~kadllm_b200.model.HybridModel` and every prefill and
decode runs on this package's sm_100a kernels; the Transformers modules are
not called.  The backend switches of the reference (``gdn_backend``,
``conv_backend``, ``attention_backend``, ``gdn_triton_config``) are validated
like the reference validates them, and are otherwise inert: there is a single
CUDA path.  BF16 models only.
"""

from __future__ import annotations

import torch

from ..config import HybridConfig
from ..grbeam import PrefillResult
from ..model import HybridModel, HybridPrefix
from ..ops import _gdn_launch


class Qwen35GRBeamAdapter:
    """Wrap an eval-mode ``Qwen3_5TextModel`` and its matching LM head."""

    def __init__(
        self,
        text_model,
        lm_head,
        *,
        gdn_backend="torch",
        conv_backend="torch",
        attention_backend="torch",
        gdn_triton_config=None,
    ):
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

        if type(text_model) is not Qwen3_5TextModel:
            raise TypeError("pass the dense Qwen3_5TextModel explicitly")
        if text_model.config.rope_parameters["rope_type"] != "default":
            raise ValueError("only default RoPE is supported")
        if text_model.config.hidden_act != "silu":
            raise ValueError("only SiLU convolution is supported")
        if gdn_backend not in ("torch", "auto", "triton") or conv_backend not in ("torch", "auto", "triton"):
            raise ValueError("invalid GDN or convolution backend")
        if attention_backend not in ("torch", "flash_attn"):
            raise ValueError("invalid attention backend")
        if any(kind not in ("linear_attention", "full_attention") for kind in text_model.config.layer_types):
            raise ValueError("unsupported layer type")
        devices = {p.device for module in (text_model, lm_head) for p in module.parameters()}
        if len(devices) != 1:
            raise ValueError("only single-device models are supported")
        _gdn_launch(gdn_triton_config)
        if gdn_triton_config is not None and gdn_backend != "triton":
            raise ValueError("gdn_triton_config requires gdn_backend='triton'")
        dtypes = {p.dtype for module in (text_model, lm_head) for p in module.parameters() if p.is_floating_point()}
        if dtypes - {torch.bfloat16, torch.float32} or text_model.embed_tokens.weight.dtype != torch.bfloat16:
            raise TypeError("kadllm_b200 runs BF16 Qwen3.5 models")
        self.layer_types = tuple(text_model.config.layer_types)
        self.model_ref, self.lm_head_ref = text_model, lm_head
        self.config = HybridConfig.from_hf(text_model.config)
        weights = {k: v.detach() for k, v in text_model.state_dict().items()}
        if lm_head.weight.data_ptr() != text_model.embed_tokens.weight.data_ptr():
            weights["lm_head.weight"] = lm_head.weight.detach()
            self.config = self.config.with_(tie_word_embeddings=False)
        self.engine = HybridModel(self.config, weights, device=next(iter(devices)))
        self._owner = self.engine.owner

    def _check(self, tokens):
        if self.model_ref.training or self.lm_head_ref.training:
            raise RuntimeError("call eval() before replay")
        if tokens.dtype not in (torch.int32, torch.int64):
            raise TypeError("token IDs must be integers")
        if tokens.device != self.engine.device:
            raise ValueError("tokens and model must share a device")

    @torch.no_grad()
    def prefill(self, input_ids):
        self._check(input_ids)
        if input_ids.ndim != 2 or min(input_ids.shape) < 1:
            raise ValueError("input_ids must be nonempty unpadded [B,L]")
        logits, state = self.engine.prefill(input_ids)
        return PrefillResult(logits, state)

    @torch.no_grad()
    def prefill_varlen(self, prompts):
        """Prompts of their own lengths in one packed prefill (no reference counterpart: the
        reference adapter takes unpadded ``[B, L]`` only).  ``prompts``: 1-D integer tensors."""
        for p in prompts:
            self._check(p)
            if p.ndim != 1 or p.numel() < 1:
                raise ValueError("each prompt must be a nonempty 1-D tensor")
        logits, state = self.engine.prefill_varlen(list(prompts))
        return PrefillResult(logits, state)

    def _check_state(self, history, state):
        self._check(history)
        if not isinstance(state, HybridPrefix) or state.owner is not self._owner:
            raise ValueError("prefix belongs to a different adapter")
        if history.ndim != 3 or min(history.shape) < 1 or history.shape[0] != state.batch:
            raise ValueError("history must be nonempty [B,W,T] matching the prefix")

    def check(self) -> None:
        """Raise if a tensor-core kernel of the engine reported a timed-out wait (synchronises)."""
        self.engine.check()

    @torch.no_grad()
    def decode(self, history, state):
        self._check_state(history, state)
        return self.engine.decode(history, state)

    def end_search(self) -> None:
        """Drop the step cache of the search that just finished (``grbeam_search`` calls it)."""
        self._step = None

    @torch.no_grad()
    def decode_select(self, history, state, scores, width, selector):
        """Decode and select in one pass (used by ``kadllm_b200.grbeam_search``).

        Step reuse: a one-token decode keeps its per-layer work (projections, q / k / v)
        and asks the selection for each new beam's parent; when the search then decodes
        exactly the history that selection returned, the two-token replay reuses the
        parent's first token and runs only the new one.  Results are those of a full
        replay of both tokens (the same kernels' arithmetic on the same inputs)."""
        self._check_state(history, state)
        T = history.shape[2]
        ws = selector.workspace if self.engine.fused_select(history.shape[0], history.shape[1]) else None
        select = selector.step_fused if ws is not None else selector.step
        step, self._step = getattr(self, "_step", None), None
        if T == 2 and step is not None and step[0] is history and step[1] is state:
            _, _, cache, parent, prev_width = step
            logits = self.engine.decode(history, state, reuse=(cache, parent, prev_width), select_workspace=ws)
            return select(logits, scores, history, width)
        if T == 1 and self.engine.step_reuse:
            cache = {}
            logits = self.engine.decode(history, state, cache=cache, select_workspace=ws)
            new_scores, new_hist, parent = select(logits, scores, history, width, parents=True)
            del logits
            self._step = (new_hist, state, cache, parent, history.shape[1])
            return new_scores, new_hist
        logits = self.engine.decode(history, state, select_workspace=ws)
        return select(logits, scores, history, width)


class NativeGRBeamAdapter(Qwen35GRBeamAdapter):
    """The same adapter over a :class:`HybridModel` built directly from packed or
    synthetic weights (no Transformers model object needed)."""

    def __init__(self, engine: HybridModel):  # noqa: D107 - deliberately not calling super()
        self.engine = engine
        self.config = engine.config if hasattr(engine, "config") else engine.cfg
        self.layer_types = tuple(self.config.layer_types)
        self._owner = engine.owner

    def _check(self, tokens):
        if tokens.dtype not in (torch.int32, torch.int64):
            raise TypeError("token IDs must be integers")
        if tokens.device != self.engine.device:
            raise ValueError("tokens and model must share a device")
