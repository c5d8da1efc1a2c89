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
    """The reference's backend switch (``src/kadllm/ops.py:41-52``): "torch" selects its
    eager implementation there; here every accepted name runs the same CUDA kernels (the
    only implementation, no CPU path)."""
    if name != "torch" and name not in accepted:
        raise ValueError(f"backend must be one of {('torch',) + tuple(accepted)}")


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
        BW // beam_width, beam_width, T, H, HV, K, V, scale, _status_word(q.device).data_ptr(),
        _lib.stream(q.device),
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


def merge_attention(prefix_out, prefix_lse, suffix_out, suffix_lse):
    """Merge two independently normalised attention partitions by LSE
    (``src/kadllm/ops.py:243-249``).  The CUDA kernel performs this merge
    internally; the helper is kept for API compatibility."""
    total = torch.logaddexp(prefix_lse, suffix_lse)
    return (
        prefix_out * (prefix_lse - total).exp()[..., None]
        + suffix_out * (suffix_lse - total).exp()[..., None]
    )


def prefix_attention(
    q,
    prefix_k,
    prefix_v,
    suffix_k,
    suffix_v,
    *,
    beam_width: int = 1,
    prefix_mask: torch.Tensor | None = None,
    scale: float | None = None,
    backend: str = "auto",
):
    """Shared-prefix attention plus a causal replay suffix, with GQA support.

    Layout: q [B*W,T,H,D], prefix K/V [B,L,HK,D] (strided views accepted),
    suffix K/V [B*W,T,HK,D].  prefix_mask [B,L] is True for valid keys.
    Mirrors ``src/kadllm/ops.py:252-308``.  Unlike the reference's FlashAttention
    path, padded prefixes (``prefix_mask``) are supported.  BF16 only.
    """
    _width(beam_width)
    tensors = (q, prefix_k, prefix_v, suffix_k, suffix_v)
    _same_device(tensors)
    if any(t.ndim != 4 for t in tensors):
        raise ValueError("attention inputs must all have rank 4")
    BW, T, H, D = q.shape
    B, L, HK, DK = prefix_k.shape
    if (
        min(BW, T, H, D, B, HK) < 1
        or BW != B * beam_width
        or H % HK
        or DK != D
        or prefix_v.shape != prefix_k.shape
        or suffix_k.shape != (BW, T, HK, D)
        or suffix_v.shape != suffix_k.shape
    ):
        raise ValueError("incompatible attention shapes")
    if len({t.dtype for t in tensors}) != 1:
        raise ValueError("attention inputs must have the same dtype")
    if prefix_mask is not None and (
        prefix_mask.shape != (B, L) or prefix_mask.dtype != torch.bool or prefix_mask.device != q.device
    ):
        raise ValueError("prefix_mask must be bool [B,L] on the query device")
    _backend(backend, _ACCEL + ("flash_attn",))
    _lib.require_cuda(*tensors)
    if q.dtype != torch.bfloat16:
        raise ValueError("the CUDA attention kernel requires bfloat16 inputs")
    scale = 1 / math.sqrt(D) if scale is None else float(scale)

    def rows(t):
        # inner dim contiguous, 16-byte aligned rows
        if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    q, prefix_k, prefix_v = rows(q), rows(prefix_k), rows(prefix_v)
    suffix_k, suffix_v = (
        t if t.stride(-1) == 1 and not any(x % 2 for x in t.stride()) and t.data_ptr() % 4 == 0
        else t.contiguous()
        for t in (suffix_k, suffix_v)
    )
    mask = None if prefix_mask is None else prefix_mask.contiguous().view(torch.uint8)
    out = torch.empty((BW, T, H, D), dtype=q.dtype, device=q.device)
    if D == _TILED_D and mask is None and L >= 1 and T <= 8:
        return _prefix_attention_tiled(q, prefix_k, prefix_v, suffix_k.contiguous(), suffix_v.contiguous(), out,
                                       B, beam_width, T, H, HK, L, D, scale)
    _lib.call(
        "kadllm_prefix_attention",
        q.data_ptr(), *q.stride()[:3], prefix_k.data_ptr(), *prefix_k.stride()[:3],
        prefix_v.data_ptr(), *prefix_v.stride()[:3], suffix_k.data_ptr(), *suffix_k.stride()[:3],
        suffix_v.data_ptr(), *suffix_v.stride()[:3], _lib.ptr(mask), None, 0, 0, 0,
        out.data_ptr(), *out.stride()[:3], _lib.dtype_code(q), B, beam_width, T, H, HK, L, D,
        scale, _lib.stream(q.device),
    )
    return out


_TILED_D = 256  # head dim of the tensor-core attention
_status: dict = {}


def _status_word(dev):
    """The device's status word of the tensor-core operators (bit 0: a wait timed out)."""
    status = _status.get(dev)
    if status is None:
        status = _status[dev] = torch.zeros(1, dtype=torch.int32, device=dev)
    return status


def _prefix_attention_tiled(q, prefix_k, prefix_v, suffix_k, suffix_v, out, B, W, T, H, HK, L, D, scale):
    """Head dim 256 without a mask: the tcgen05 attention over a tiled copy of the prefix
    (one re-layout of K / V per call), split over the key blocks when the request count
    leaves SMs idle."""
    lib = _lib.lib()
    dev = q.device
    s = _lib.stream(dev)
    nbytes = lib.kadllm_kv_tile_bytes(B, HK, L, D)
    kt = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    vt = torch.empty_like(kt)
    _lib.call("kadllm_kv_tile", prefix_k.data_ptr(), *prefix_k.stride()[:3], B, HK, L, D, kt.data_ptr(), nbytes, s)
    _lib.call("kadllm_kv_tile", prefix_v.data_ptr(), *prefix_v.stride()[:3], B, HK, L, D, vt.data_ptr(), nbytes, s)
    status = _status_word(dev)
    # CTAs of 128 query rows per (request, kv head); split the key blocks when they leave SMs idle
    ctas = -(-(W * T * (H // HK)) // 128) * B * HK
    sms = _sm_count(dev)
    splits = max(1, min(sms // ctas, -(-L // 64), 64)) if ctas < sms else 1
    ws_bytes = lib.kadllm_attention_split_workspace(B, W, T, 0, H, splits)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    _lib.call("kadllm_attention_tiled_split", q.data_ptr(), *q.stride()[:3], kt.data_ptr(), vt.data_ptr(),
              -(-L // 64), suffix_k.data_ptr(), *suffix_k.stride()[:3], suffix_v.data_ptr(), *suffix_v.stride()[:3],
              None, 0, 0, 0, out.data_ptr(), *out.stride()[:3], status.data_ptr(), B, W, T, 0, H, HK, L, D, scale,
              splits, ws.data_ptr(), ws.numel(), s)
    return out


def check(device=None) -> None:
    """Raise if a tensor-core wait of an operator timed out on ``device`` since the last
    check (synchronises; the operators themselves never wait on the host)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    status = _status.get(dev)
    if status is not None and int(status.item()):
        status.zero_()
        raise RuntimeError("kadllm_b200 operator: a tensor-core pipeline wait timed out")


_sms: dict = {}


def _sm_count(dev) -> int:
    n = _sms.get(dev)
    if n is None:
        n = _sms[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    return n
