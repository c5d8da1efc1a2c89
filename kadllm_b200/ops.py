"""GRBeam shared-prefix operators on the sm_100a CUDA library.

Same names, layouts, keyword arguments and error types as Kadllm's
``src/kadllm/ops.py``; each call validates its arguments like the reference
and launches a hand-written kernel through the C ABI (``_lib``).  There is no
torch or CPU path: non-CUDA inputs raise ``RuntimeError``.

The reference's ``backend`` switches select between its torch and Triton/FA2
paths.  Here ``"auto"``, ``"cuda"`` and the reference's accelerated names
(``"triton"``, ``"flash_attn"``) all run the CUDA kernels; ``"torch"`` is
rejected because the torch path is the reference's CPU oracle, not part of
this library.
"""

from __future__ import annotations

import math

import torch

from . import _lib

_ACCEL = ("auto", "cuda", "triton")


def _width(width):
    if not isinstance(width, int) or isinstance(width, bool) or width <= 0:
        raise ValueError("beam_width must be a positive integer")


def _same_device(tensors):
    if len({t.device for t in tensors}) != 1:
        raise ValueError("all tensors must be on the same device")
    if not all(t.is_floating_point() for t in tensors):
        raise TypeError("operator inputs must be floating-point tensors")


def _backend(name: str, accepted=_ACCEL) -> None:
    if name == "torch":
        raise ValueError("kadllm_b200 has no torch path; use backend='auto' or 'cuda'")
    if name not in accepted:
        raise ValueError(f"backend must be one of {accepted}")


def _gdn_launch(config):
    """Validate a reference Triton launch tuple (``src/kadllm/ops.py:53-67``).

    Accepted for API compatibility; the CUDA kernel picks its own tiling.
    """
    if config is None:
        return
    if (
        not isinstance(config, tuple)
        or len(config) not in (3, 4)
        or any(type(value) is not int for value in config)
        or config[0] not in (8, 16, 32, 64, 128)
        or config[1] not in (1, 2, 4, 8)
        or config[2] not in (1, 2, 3)
        or (len(config) == 4 and config[3] not in (1, 2, 4, 8, 16))
    ):
        raise ValueError("triton_config must be (tile_v, num_warps, num_stages[, beam_group])")


def gated_delta(
    q,
    k,
    v,
    log_decay,
    beta,
    shared_state,
    *,
    beam_width: int = 1,
    scale: float | None = None,
    backend: str = "auto",
    return_final_state: bool = False,
    triton_config: tuple[int, ...] | None = None,
):
    """Gated delta recurrence replayed from a shared, request-sized state.

    q,k: [B*W,T,H,K]; v: [B*W,T,HV,V]; log_decay, beta: [B*W,T,HV];
    shared_state: [B,HV,K,V] (read-only).  Returns [B*W,T,HV,V] in v's dtype.
    Mirrors ``src/kadllm/ops.py:70-138``.  The state is never copied per beam:
    all beams of a request are multiplied against it at once on the tensor
    cores (``csrc/gdn_replay.cu``).  K == V in {32, 64, 128}, T <= 8.
    """
    _width(beam_width)
    _gdn_launch(triton_config)
    tensors = (q, k, v, log_decay, beta, shared_state)
    _same_device(tensors)
    if q.ndim != 4 or k.shape != q.shape or v.ndim != 4 or shared_state.ndim != 4:
        raise ValueError("invalid q/k/v/state ranks or shapes")
    BW, T, H, K = q.shape
    HV, V = v.shape[-2:]
    if min(BW, T, H, K, HV, V) <= 0 or HV % H or BW % beam_width:
        raise ValueError("empty dimensions or incompatible beam/head counts")
    if (
        v.shape[:2] != (BW, T)
        or log_decay.shape != (BW, T, HV)
        or beta.shape != log_decay.shape
        or shared_state.shape != (BW // beam_width, HV, K, V)
    ):
        raise ValueError("incompatible state, value, or gate shape")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q/k/v must have the same dtype")
    _backend(backend)
    if return_final_state:
        raise NotImplementedError("return_final_state is a reference torch-path facility; "
                                  "prefill states come from the chunked prefill kernel")
    _lib.require_cuda(*tensors)
    scale = K ** -0.5 if scale is None else float(scale)
    q, k, v, log_decay, beta, shared_state = (_lib.aligned(t) for t in tensors)
    out = torch.empty_like(v)
    _lib.call(
        "kadllm_gated_delta_replay",
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.dtype_code(q),
        log_decay.data_ptr(), _lib.dtype_code(log_decay), beta.data_ptr(), _lib.dtype_code(beta),
        shared_state.data_ptr(), _lib.dtype_code(shared_state), out.data_ptr(),
        BW // beam_width, beam_width, T, H, HV, K, V, scale, _lib.stream(q.device),
    )
    return out


def causal_conv1d(
    x,
    shared_state,
    weight,
    *,
    beam_width: int = 1,
    bias=None,
    activation: str | None = "silu",
    backend: str = "auto",
):
    """Stateless depthwise short convolution replayed from a shared prefix.

    x: [B*W,C,T] (strided views accepted); shared_state: [B,C,history];
    weight: [C,width].  Only the last width-1 prefix taps are consumed.
    Returns [B*W,C,T].  Mirrors ``src/kadllm/ops.py:166-214``; width <= 8.
    """
    _width(beam_width)
    tensors = (x, shared_state, weight) + (() if bias is None else (bias,))
    _same_device(tensors)
    if x.ndim != 3 or shared_state.ndim != 3 or weight.ndim != 2:
        raise ValueError("invalid convolution input ranks")
    BW, C, T = x.shape
    width = weight.shape[-1]
    if (
        min(BW, C, T, width) < 1
        or BW % beam_width
        or shared_state.shape[:2] != (BW // beam_width, C)
        or shared_state.shape[-1] < width - 1
        or weight.shape[0] != C
    ):
        raise ValueError("incompatible convolution shapes")
    if len({t.dtype for t in tensors}) != 1:
        raise ValueError("convolution inputs must have the same dtype")
    if bias is not None and bias.shape != (C,):
        raise ValueError("bias must have shape [C]")
    if activation not in (None, "silu"):
        raise ValueError("activation must be None or silu")
    _backend(backend)
    _lib.require_cuda(*tensors)
    weight = weight.contiguous()
    bias = None if bias is None else bias.contiguous()
    out = torch.empty((BW, C, T), dtype=x.dtype, device=x.device)
    _lib.call(
        "kadllm_causal_conv1d_replay",
        x.data_ptr(), *x.stride(), shared_state.data_ptr(), *shared_state.stride(),
        shared_state.shape[-1], weight.data_ptr(), _lib.ptr(bias), out.data_ptr(),
        _lib.dtype_code(x), BW // beam_width, beam_width, C, T, width,
        1 if activation == "silu" else 0, _lib.stream(x.device),
    )
    return out
