"""The tcgen05 projection GEMM (``kadllm_gemm``) against a torch fp32 product of
the same BF16 operands: plain product, the MLP's SiLU-mul epilogue and the
residual-update epilogue, at ragged and at the benchmark's shapes."""

import pytest
import torch

from kadllm_b200 import _lib
from kadllm_b200.model import GEMM_ADD, GEMM_SILU_MUL, GEMM_STORE, interleave_gate_up

pytestmark = pytest.mark.gpu

# fp32 accumulation in a different order, then one BF16 rounding: 2 BF16 ulps
# relative, plus an absolute term for sums that cancel
RTOL = 2.0 ** -7


def _atol(ref: torch.Tensor) -> float:
    return 2.0 ** -9 * float(ref.abs().mean())


def _gemm(a, b, *, resid=None, silu_inter=None, status=None):
    M, K = a.shape
    N = b.shape[0]
    if silu_inter is not None:
        epi, n_out = GEMM_SILU_MUL, silu_inter
        out = torch.empty(M, n_out, dtype=torch.bfloat16, device=a.device)
    elif resid is not None:
        epi, n_out, out = GEMM_ADD, N, resid
    else:
        epi, n_out = GEMM_STORE, N
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    status = torch.zeros(1, dtype=torch.int32, device=a.device) if status is None else status
    _lib.call("kadllm_gemm", a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0),
              _lib.ptr(resid), 0 if resid is None else resid.stride(0), M, N, K, n_out, epi, status.data_ptr(),
              _lib.stream(a.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "a bounded wait of the GEMM timed out"
    return out


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    return a, b


@pytest.mark.parametrize("M,N,K", [
    (256, 256, 64), (1, 256, 64), (300, 520, 128), (192, 320, 96), (1000, 1024, 2048),
    (4096, 8224, 1024), (513, 5120, 1024), (8192, 1024, 3584), (64, 248320, 1024)])
def test_gemm_matches_fp32_product(M, N, K):
    """Partial M / N / K tiles (zero fill past the edges), a single row, N = 8224
    (the GDN input projection, 32 columns into a last tile), several waves of tiles
    over the CTA pairs, and the full vocabulary's LM-head width."""
    a, b = _operands(M, N, K, seed=M + N + K)
    ref = a.float() @ b.float().T
    out = _gemm(a, b)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=_atol(ref))


@pytest.mark.parametrize("M,I,K", [(300, 384, 256), (257, 200, 128), (2048, 3584, 1024)])
def test_gemm_silu_mul_epilogue(M, I, K):
    """act = bf16(bf16(silu(bf16(gate))) * bf16(up)) from the interleaved gate / up
    weight, including a width that is not a multiple of 128 (zero-padded blocks)."""
    g = torch.Generator(device="cuda").manual_seed(I)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    gate = (torch.randn(I, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    up = (torch.randn(I, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    w = interleave_gate_up(gate, up)
    out = _gemm(a, w, silu_inter=I)
    gf = (a.float() @ gate.float().T).bfloat16()
    uf = (a.float() @ up.float().T).bfloat16()
    ref = (torch.nn.functional.silu(gf.float()).bfloat16().float() * uf.float())
    # the gate and up roundings can each move by an ulp, and SiLU runs on the fast exp2
    torch.testing.assert_close(out.float(), ref, rtol=2 * RTOL, atol=2 * _atol(ref))


@pytest.mark.parametrize("M,N,K", [(300, 1024, 2048), (8192, 1024, 3584), (77, 136, 64)])
def test_gemm_residual_epilogue_in_place(M, N, K):
    """x = bf16(x + bf16(a . b^T)) written over x."""
    a, b = _operands(M, N, K, seed=7 * M)
    x = torch.randn(M, N, device="cuda").bfloat16()
    x0 = x.clone()
    _gemm(a, b, resid=x)
    prod = a.float() @ b.float().T
    ref = x0.float() + prod.bfloat16().float()
    # the product's BF16 rounding may differ by an ulp (accumulation order) and the sum
    # is rounded again: an ulp of |product| plus an ulp of |sum|, elementwise
    bound = RTOL * (prod.abs() + ref.abs()) + _atol(prod)
    err = (x.float() - ref).abs()
    assert bool((err <= bound).all()), f"max error {float(err.max())}, worst excess {float((err - bound).max())}"


@pytest.mark.parametrize("M,N,K,ld", [(20000, 1000, 128, 1008), (77, 136, 64, 200)])
def test_gemm_residual_epilogue_ragged_row(M, N, K, ld):
    """Rows that end inside a 64-column residual / output box (padded row stride) and
    several tiles per CTA pair: the padding past N is neither read into the sum nor
    written."""
    a, b = _operands(M, N, K, seed=N + K)
    store = torch.randn(M, ld, device="cuda").bfloat16()
    x = store[:, :N]
    x0, pad0 = x.clone(), store[:, N:].clone()
    _gemm(a, b, resid=x)
    prod = a.float() @ b.float().T
    ref = x0.float() + prod.bfloat16().float()
    bound = RTOL * (prod.abs() + ref.abs()) + _atol(prod)
    err = (x.float() - ref).abs()
    assert bool((err <= bound).all()), f"max error {float(err.max())}, worst excess {float((err - bound).max())}"
    assert torch.equal(store[:, N:], pad0)


def test_gemm_rejects_bad_arguments():
    a, b = _operands(64, 64, 64, seed=0)
    out = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = _lib.stream(a.device)
    with pytest.raises(ValueError):  # empty K
        _lib.call("kadllm_gemm", a.data_ptr(), 64, b.data_ptr(), 64, out.data_ptr(), 64, None, 0, 64, 64, 0, 64,
                  GEMM_STORE, st.data_ptr(), s)
    with pytest.raises(ValueError):  # leading dimension not a multiple of 8
        _lib.call("kadllm_gemm", a.data_ptr(), 63, b.data_ptr(), 64, out.data_ptr(), 64, None, 0, 64, 64, 60, 64,
                  GEMM_STORE, st.data_ptr(), s)
    with pytest.raises(ValueError):  # SiLU-mul needs whole 256-row gate / up block pairs
        _lib.call("kadllm_gemm", a.data_ptr(), 64, b.data_ptr(), 64, out.data_ptr(), 64, None, 0, 64, 64, 64, 32,
                  GEMM_SILU_MUL, st.data_ptr(), s)
