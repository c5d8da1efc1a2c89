"""Argument validation of the drop-in operators, on the host.

``kadllm_b200.ops`` checks its arguments in the reference's order and with its
exception types (``src/kadllm/ops.py:41-67`` helpers, ``:98-116`` gated_delta,
``:183-202`` causal_conv1d, ``:272-295`` prefix_attention) before it touches a
device, so every rejected call is checked here with CPU (or meta) tensors: empty
dimensions, widths that do not divide the rows, mismatched shapes, dtypes and
devices, unknown launch tuples and activations.  Arguments that pass the checks
reach the CUDA requirement and raise ``RuntimeError`` (the library has no CPU
path).  The adapter's constructor switches are checked the same way on a tiny
CPU model.  No GPU is needed.
"""

import copy

import pytest
import torch

from kadllm_b200 import ops


def _gd(BW=4, T=1, H=2, K=32, HV=2, V=32, B=2, dtype=torch.float32):
    q = torch.zeros(BW, T, H, K, dtype=dtype)
    v = torch.zeros(BW, T, HV, V, dtype=dtype)
    g = torch.zeros(BW, T, HV)
    return [q, q.clone(), v, g, g.clone(), torch.zeros(B, HV, K, V)]


def _conv(BW=4, C=8, T=2, width=4, hist=3, B=2, dtype=torch.float32):
    return [torch.zeros(BW, C, T, dtype=dtype), torch.zeros(B, C, hist, dtype=dtype), torch.zeros(C, width, dtype=dtype)]


def _attn(BW=4, T=2, H=4, D=16, B=2, L=5, HK=2, dtype=torch.bfloat16):
    return [torch.zeros(BW, T, H, D, dtype=dtype), torch.zeros(B, L, HK, D, dtype=dtype),
            torch.zeros(B, L, HK, D, dtype=dtype), torch.zeros(BW, T, HK, D, dtype=dtype),
            torch.zeros(BW, T, HK, D, dtype=dtype)]


@pytest.mark.parametrize("width", [0, -1, True, 2.0, None])
def test_beam_width_must_be_a_positive_integer(width):
    with pytest.raises(ValueError, match="beam_width"):
        ops.gated_delta(*_gd(), beam_width=width)
    with pytest.raises(ValueError, match="beam_width"):
        ops.causal_conv1d(*_conv(), beam_width=width)
    with pytest.raises(ValueError, match="beam_width"):
        ops.prefix_attention(*_attn(), beam_width=width)


@pytest.mark.parametrize("case", [
    dict(BW=0, B=0), dict(T=0), dict(H=0), dict(K=0), dict(HV=0), dict(V=0),
    dict(H=2, HV=3),  # value heads not a multiple of key heads
])
def test_gated_delta_rejects_empty_and_incompatible_dimensions(case):
    with pytest.raises(ValueError, match="empty dimensions or incompatible"):
        ops.gated_delta(*_gd(**case), beam_width=2)


def test_gated_delta_rejects_rows_not_divisible_by_the_width():
    with pytest.raises(ValueError, match="empty dimensions or incompatible"):
        ops.gated_delta(*_gd(BW=4), beam_width=3)


@pytest.mark.parametrize("slot,shape", [
    (2, (4, 2, 2, 32)),   # v with another T
    (3, (4, 1, 3)),       # log_decay heads
    (4, (4, 1)),          # beta rank
    (5, (3, 2, 32, 32)),  # state rows != BW / width
    (5, (2, 2, 32, 16)),  # state value dim
])
def test_gated_delta_rejects_mismatched_shapes(slot, shape):
    args = _gd()
    args[slot] = torch.zeros(shape)
    with pytest.raises(ValueError, match="incompatible state|invalid q/k/v"):
        ops.gated_delta(*args, beam_width=2)


def test_gated_delta_rejects_ranks_dtypes_devices_and_types():
    args = _gd()
    with pytest.raises(ValueError, match="ranks"):
        ops.gated_delta(args[0][..., 0], *args[1:], beam_width=2)
    with pytest.raises(ValueError, match="same dtype"):
        ops.gated_delta(args[0], args[1], args[2].double(), *args[3:], beam_width=2)
    with pytest.raises(ValueError, match="same device"):
        ops.gated_delta(args[0].to("meta"), *args[1:], beam_width=2)
    with pytest.raises(TypeError, match="floating-point"):
        ops.gated_delta(args[0].long(), *args[1:], beam_width=2)


@pytest.mark.parametrize("config", [(7, 1, 1), (8, 3, 1), (8, 1, 4), (8, 1, 1, 3), (8, 1), [8, 1, 1], (8.0, 1, 1)])
def test_gated_delta_rejects_unknown_launch_tuples(config):
    with pytest.raises(ValueError, match="triton_config"):
        ops.gated_delta(*_gd(), beam_width=2, triton_config=config)


def test_gated_delta_backend_names_and_cpu_inputs():
    with pytest.raises(ValueError, match="backend"):
        ops.gated_delta(*_gd(), beam_width=2, backend="bogus")
    with pytest.raises(NotImplementedError):
        ops.gated_delta(*_gd(), beam_width=2, return_final_state=True)
    for name in ("auto", "cuda", "triton", "torch"):
        with pytest.raises(RuntimeError, match="CUDA"):
            ops.gated_delta(*_gd(), beam_width=2, backend=name, triton_config=(32, 4, 2, 2))


@pytest.mark.parametrize("case", [dict(BW=0, B=0), dict(C=0), dict(T=0), dict(width=0), dict(hist=2), dict(B=3)])
def test_causal_conv1d_rejects_empty_and_incompatible_shapes(case):
    with pytest.raises(ValueError, match="incompatible convolution shapes"):
        ops.causal_conv1d(*_conv(**case), beam_width=2)


def test_causal_conv1d_rejects_ranks_dtypes_bias_and_activation():
    x, state, w = _conv()
    with pytest.raises(ValueError, match="ranks"):
        ops.causal_conv1d(x[0], state, w, beam_width=2)
    with pytest.raises(ValueError, match="incompatible convolution shapes"):
        ops.causal_conv1d(x, state, torch.zeros(9, 4), beam_width=2)
    with pytest.raises(ValueError, match="same dtype"):
        ops.causal_conv1d(x, state.double(), w, beam_width=2)
    with pytest.raises(ValueError, match="bias"):
        ops.causal_conv1d(x, state, w, beam_width=2, bias=torch.zeros(7))
    with pytest.raises(ValueError, match="activation"):
        ops.causal_conv1d(x, state, w, beam_width=2, activation="relu")
    with pytest.raises(ValueError, match="backend"):
        ops.causal_conv1d(x, state, w, beam_width=2, backend="bogus")
    # a width-1 filter, no activation and a bias are valid arguments: the CUDA requirement comes next
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.causal_conv1d(*_conv(width=1, hist=1), beam_width=2, bias=torch.zeros(8), activation=None)


@pytest.mark.parametrize("case", [
    dict(BW=0, B=0), dict(T=0), dict(H=0), dict(D=0), dict(HK=0),
    dict(BW=5),        # rows != requests x width
    dict(H=3),         # query heads not a multiple of kv heads
])
def test_prefix_attention_rejects_empty_and_incompatible_shapes(case):
    with pytest.raises(ValueError, match="incompatible attention shapes"):
        ops.prefix_attention(*_attn(**case), beam_width=2)


def test_prefix_attention_rejects_ranks_dtypes_and_masks():
    q, pk, pv, sk, sv = _attn()
    with pytest.raises(ValueError, match="rank 4"):
        ops.prefix_attention(q[0], pk, pv, sk, sv, beam_width=2)
    with pytest.raises(ValueError, match="incompatible attention shapes"):
        ops.prefix_attention(q, pk, pv[:, :4], sk, sv, beam_width=2)
    with pytest.raises(ValueError, match="incompatible attention shapes"):
        ops.prefix_attention(q, pk, pv, sk[:, :1], sv, beam_width=2)
    with pytest.raises(ValueError, match="same dtype"):
        ops.prefix_attention(q, pk.float(), pv, sk, sv, beam_width=2)
    with pytest.raises(ValueError, match="prefix_mask"):
        ops.prefix_attention(q, pk, pv, sk, sv, beam_width=2, prefix_mask=torch.ones(2, 5, dtype=torch.uint8))
    with pytest.raises(ValueError, match="prefix_mask"):
        ops.prefix_attention(q, pk, pv, sk, sv, beam_width=2, prefix_mask=torch.ones(2, 4, dtype=torch.bool))
    with pytest.raises(ValueError, match="backend"):
        ops.prefix_attention(q, pk, pv, sk, sv, beam_width=2, backend="bogus")


@pytest.mark.parametrize("L", [0, 5])
def test_prefix_attention_empty_prefix_is_a_valid_argument(L):
    """An empty prefix (L = 0) passes validation as in the reference, whose rows then
    attend to the suffix only; on CPU tensors the CUDA requirement is what raises."""
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.prefix_attention(*_attn(L=L), beam_width=2, prefix_mask=torch.ones(2, L, dtype=torch.bool))


@pytest.fixture(scope="module")
def tiny_text_model():
    """A random-init BF16 Qwen3_5TextModel with the library's tiny hybrid dims, on CPU."""
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    from kadllm_b200.config import TINY

    torch.manual_seed(0)
    model = Qwen3_5TextModel(Qwen3_5TextConfig(**TINY.to_hf_kwargs())).to(torch.bfloat16).eval()
    head = torch.nn.Linear(TINY.hidden_size, TINY.vocab_size, bias=False).to(torch.bfloat16).eval()
    return model, head


@pytest.mark.parametrize("kwargs", [
    dict(gdn_backend="cuda"), dict(conv_backend="flash_attn"), dict(attention_backend="triton"),
    dict(attention_backend="auto"), dict(gdn_triton_config=(32, 4, 2)),  # a launch tuple needs gdn_backend="triton"
    dict(gdn_backend="triton", gdn_triton_config=(33, 4, 2)),
])
def test_adapter_rejects_backend_switches_like_the_reference(tiny_text_model, kwargs):
    """``Qwen35GRBeamAdapter``'s switches (``src/kadllm/adapters/qwen3_5.py:61-92``)."""
    from kadllm_b200.adapters import Qwen35GRBeamAdapter

    with pytest.raises(ValueError):
        Qwen35GRBeamAdapter(*tiny_text_model, **kwargs)


def test_adapter_rejects_other_modules_and_dtypes(tiny_text_model):
    from kadllm_b200.adapters import Qwen35GRBeamAdapter

    model, head = tiny_text_model
    with pytest.raises(TypeError, match="Qwen3_5TextModel"):
        Qwen35GRBeamAdapter(head, head)
    with pytest.raises(TypeError, match="BF16"):
        Qwen35GRBeamAdapter(model, copy.deepcopy(head).half())
    # valid switches on a CPU model: the engine's CUDA requirement is what raises
    with pytest.raises(RuntimeError, match="CUDA"):
        Qwen35GRBeamAdapter(model, head, gdn_backend="triton", conv_backend="auto", attention_backend="flash_attn",
                            gdn_triton_config=(32, 4, 2, 8))


class _FakeAdapter:
    """Returns fixed prefill logits; decode is never reached on the host."""

    def __init__(self, logits):
        self.logits, self.prefills = logits, 0

    def prefill(self, input_ids):
        from kadllm_b200.grbeam import PrefillResult

        self.prefills += 1
        return PrefillResult(self.logits, None)

    def decode(self, history, state):  # pragma: no cover - validation stops earlier
        raise AssertionError("decode reached")


@pytest.mark.parametrize("ids,widths", [
    (torch.zeros(3, dtype=torch.long), [2]),        # not [B, L]
    (torch.zeros(0, 4, dtype=torch.long), [2]),     # no requests
    (torch.zeros(2, 0, dtype=torch.long), [2]),     # empty prompts
    (torch.zeros(2, 4, dtype=torch.long), []),      # no levels
    (torch.zeros(2, 4, dtype=torch.long), [2, 0]),
    (torch.zeros(2, 4, dtype=torch.long), [True]),
    (torch.zeros(2, 4, dtype=torch.long), [2.0]),
])
def test_grbeam_search_rejects_inputs_before_the_prefill(ids, widths):
    """``grbeam_search``'s checks (``src/kadllm/grbeam.py:60-65``) run before the adapter."""
    from kadllm_b200 import grbeam_search

    adapter = _FakeAdapter(torch.zeros(2, 8))
    with pytest.raises(ValueError):
        grbeam_search(adapter, ids, widths)
    assert adapter.prefills == 0


@pytest.mark.parametrize("logits", [torch.zeros(3, 8), torch.zeros(2, 1, 8), torch.zeros(2, 0)])
def test_grbeam_search_rejects_prefill_logits_of_another_shape(logits):
    """``src/kadllm/grbeam.py:67-72``: [B, V] logits with V >= 1."""
    from kadllm_b200 import grbeam_search

    with pytest.raises(ValueError):
        grbeam_search(_FakeAdapter(logits), torch.zeros(2, 4, dtype=torch.long), [2])


def test_grbeam_search_needs_cuda_logits():
    from kadllm_b200 import grbeam_search

    with pytest.raises(RuntimeError, match="CUDA"):
        grbeam_search(_FakeAdapter(torch.zeros(2, 8)), torch.zeros(2, 4, dtype=torch.long), [2, 2])
