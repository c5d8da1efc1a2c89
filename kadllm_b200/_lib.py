"""ctypes binding of the C ABI in ``include/kadllm_b200.h``.

The shared library is built in-tree (``python -m kadllm_b200.build``).  There
is no fallback: importing an operator without the library, or calling one on
non-CUDA tensors, raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libkadllm_b200.so")

P, I, L, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float

# entry point -> argument types (all return int status)
SIGNATURES: dict[str, list] = {
    "kadllm_embed_rmsnorm": [P, P, L, P, F, P, P, L, L, P],
    "kadllm_add_rmsnorm": [P, P, L, P, F, P, L, L, L, L, P],
    "kadllm_silu_mul": [P, L, L, P, L, P],
    "kadllm_qk_norm_rope": [P, L, L, L, L, P, P, F, P, P, L, P, L, L, P, L, L, P, L, L, L, P, L, L, L, L, P],
    "kadllm_gdn_prefill_split": [P, L, P, P, P, P, P, F, P, L, P, P, L, L, L, L, L, L, L, P],
    "kadllm_kv_tile": [P, L, L, L, L, L, L, L, P, L, P],
    "kadllm_kv_tile_varlen": [P, L, L, P, L, L, L, L, P, L, P],
    "kadllm_diag_wait_timeout": [P, L, P],
    "kadllm_gdn_prefill_split_varlen": [P, L, P, P, P, P, P, F, P, L, P, P, L, P, L, L, L, L, L, L, L, P],
    "kadllm_attention_tiled": [P, L, L, L, P, P, L, P, L, L, L, P, L, L, L, P, L, L, L, P, L, L, L, P,
                               L, L, L, L, L, L, L, L, F, I, P],
    "kadllm_attention_tiled_varlen": [P, L, L, L, P, P, L, P, L, L, L, P, L, L, L, P, L, L, L, P, L, L, L, P,
                                      P, L, L, L, L, L, L, L, L, F, I, P],
    "kadllm_attention_tiled_split": [P, L, L, L, P, P, L, P, L, L, L, P, L, L, L, P, L, L, L, P, L, L, L, P,
                                     L, L, L, L, L, L, L, L, F, L, P, L, P],
    "kadllm_causal_attention": [P, L, L, P, L, L, L, P, L, L, L, P, L, L, P, L, L, L, L, L, L, L, F, P],
    "kadllm_beam_select": [P, I, L, P, P, P, P, P, P, P, L, L, L, L, L, L, P],
    "kadllm_beam_select_status": [P, L, L, P, P],
    "kadllm_beam_select_noalloc": [P, I, L, P, P, P, P, P, P, L, L, L, L, L, P],
    "kadllm_gated_delta_replay": [P, P, P, I, P, I, P, I, P, I, P, L, L, L, L, L, L, L, F, P, P],
    "kadllm_gdn_mixer_replay": [P, L, P, L, P, P, P, P, P, F, P, L, L, L, L, L, L, L, P, P, P],
    "kadllm_causal_conv1d_replay": [P, L, L, L, P, L, L, L, L, P, P, P, I, L, L, L, L, L, I, P],
    "kadllm_gemm": [P, L, P, L, P, L, P, L, L, L, L, L, I, P, P],
    "kadllm_gemm_logits": [P, L, P, L, P, L, L, L, L, P, L, L, L, P, P],
    "kadllm_beam_select_fused": [P, L, P, P, P, P, P, P, L, L, L, L, L, L, P],
    "kadllm_gather_rows": [P, L, P, L, L, L, L, P, L, P],
    "kadllm_gdn_mixer_continue": [P, P, L, P, L, P, L, P, P, P, P, P, F, P, L, L, L, L, L, L, P, P, P],
    "kadllm_prefix_attention": [P, L, L, L, P, L, L, L, P, L, L, L, P, L, L, L, P, L, L, L, P, P,
                                L, L, L, P, L, L, L, I, L, L, L, L, L, L, L, F, P],
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"kadllm_b200 CUDA library missing ({LIB_PATH.name}); build it with "
                "`python -m kadllm_b200.build`"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        handle.kadllm_last_error.restype = ctypes.c_char_p
        handle.kadllm_last_error.argtypes = []
        handle.kadllm_abi_version.restype = ctypes.c_int
        handle.kadllm_beam_select_workspace.restype = ctypes.c_int64
        handle.kadllm_beam_select_workspace.argtypes = [L, L]
        handle.kadllm_beam_select_workspace_fused.restype = ctypes.c_int64
        handle.kadllm_beam_select_workspace_fused.argtypes = [L, L]
        handle.kadllm_gdn_prefill_workspace.restype = ctypes.c_int64
        handle.kadllm_gdn_prefill_workspace.argtypes = [L, L, L, L, L]
        handle.kadllm_attention_split_workspace.restype = ctypes.c_int64
        handle.kadllm_attention_split_workspace.argtypes = [L, L, L, L, L, L]
        handle.kadllm_kv_tile_bytes.restype = ctypes.c_int64
        handle.kadllm_kv_tile_bytes.argtypes = [L, L, L, L]
        handle.kadllm_gdn_mixer_record_bytes.restype = ctypes.c_int64
        handle.kadllm_gdn_mixer_record_bytes.argtypes = [L, L, L, L]
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = handle
    return _lib


_ERRORS = {1: ValueError, 2: TypeError, 3: NotImplementedError, 4: RuntimeError}


# kernels launched per successful call of each entry point (for launch accounting)
LAUNCHES_PER_CALL = {"kadllm_beam_select": 4, "kadllm_beam_select_noalloc": 4, "kadllm_beam_select_status": 0,
                     "kadllm_beam_select_fused": 4, "kadllm_attention_tiled_split": 2,
                     "kadllm_gdn_prefill_split": 2, "kadllm_gdn_prefill_split_varlen": 2}
launch_count = 0
_count_lock = threading.Lock()


def call(name: str, *args) -> None:
    """Invoke an entry point and map a nonzero status to the reference's exception types."""
    global launch_count
    rc = getattr(lib(), name)(*args)
    if not rc:
        with _count_lock:  # callers may drive several streams from several threads
            launch_count += LAUNCHES_PER_CALL.get(name, 1)
    if rc:
        msg = lib().kadllm_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, RuntimeError)(msg)


DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, float16 or bfloat16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> None:
    if not all(t.is_cuda for t in tensors):
        raise RuntimeError("kadllm_b200 operators run only on CUDA tensors (no CPU path)")
    if len({t.device for t in tensors}) != 1:
        raise ValueError("all tensors must be on the same device")


def aligned(t: torch.Tensor, nbytes: int = 16) -> torch.Tensor:
    """Contiguous tensor whose data pointer is ``nbytes``-aligned (copies only if needed)."""
    t = t.contiguous()
    if t.data_ptr() % nbytes:
        t = t.clone()
    return t
