"""GPU parity of the shared-prefix decode attention kernel."""

import numpy as np
import pytest
import torch

from oracle import grbeam_oracle as O
from tests import torch_ref
from tests.parity import assert_close_rel, bf16_tol, load

pytestmark = pytest.mark.gpu
bf = torch.bfloat16


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(bf)


def test_matches_golden_including_masks_and_empty_prefix():
    from kadllm_b200 import ops

    g = load("ops_bf16.npz")
    W = int(g["at_W"])
    args = [_t(g[k]) for k in ("at_q", "at_pk", "at_pv", "at_sk", "at_sv")]
    tol = bf16_tol(g["at_out"], 1, 0)
    out = ops.prefix_attention(*args, beam_width=W)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["at_out"], atol=tol, rtol=0)
    mask = torch.from_numpy(g["at_mask"]).cuda()
    out = ops.prefix_attention(*args, beam_width=W, prefix_mask=mask)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["at_out_masked"], atol=tol, rtol=0)
    out = ops.prefix_attention(args[0], args[1][:, :0], args[2][:, :0], args[3], args[4], beam_width=W)
    np.testing.assert_allclose(out.float().cpu().numpy(), g["at_out_empty"], atol=tol, rtol=0)


@pytest.mark.parametrize("D", [32, 64, 128, 256])
@pytest.mark.parametrize("L,T", [(1, 1), (33, 2), (100, 3), (64, 8)])
def test_matches_oracle(D, L, T):
    from kadllm_b200 import ops

    rng = np.random.default_rng(D + L + T)
    B, W, H, HK = 2, 7, 8, 2
    r = lambda *s: O.bf16(rng.standard_normal(s).astype(np.float32))
    q, sk, sv = r(B * W, T, H, D), r(B * W, T, HK, D), r(B * W, T, HK, D)
    pk_store, pv_store = r(B, HK, L, D), r(B, HK, L, D)  # [B,HK,L,D] storage, passed as views
    pk = _t(pk_store).transpose(1, 2)
    pv = _t(pv_store).transpose(1, 2)
    before = pk.clone()
    out = ops.prefix_attention(_t(q), pk, pv, _t(sk), _t(sv), beam_width=W)
    ref = O.prefix_attention(q, pk_store.transpose(0, 2, 1, 3), pv_store.transpose(0, 2, 1, 3), sk, sv,
                             beam_width=W)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=bf16_tol(ref, 2, 0), rtol=0)
    assert torch.equal(pk, before)


@pytest.mark.parametrize("B,W,T,L", [(32, 256, 1, 1024), (32, 256, 2, 1024), (1, 256, 3, 4096)])
def test_full_size_matches_torch_fp32(B, W, T, L):
    """0.8B decode shapes (8 q / 2 kv heads, d = 256) and the decode-attention microbenchmark."""
    from kadllm_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(L + T)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen).to(bf)
    H, HK, D = 8, 2, 256
    q, sk, sv = n(B * W, T, H, D), n(B * W, T, HK, D), n(B * W, T, HK, D)
    pk, pv = n(B, L, HK, D), n(B, L, HK, D)
    out = ops.prefix_attention(q, pk, pv, sk, sv, beam_width=W)
    ref = torch_ref.prefix_attention(q, pk, pv, sk, sv, W)
    assert_close_rel(out.float().cpu().numpy(), ref.cpu().numpy(), rel=5e-3, what="attention")


def test_masked_prefix_matches_torch_fp32():
    from kadllm_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(5)
    B, W, T, L, H, HK, D = 4, 16, 2, 300, 8, 2, 256
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen).to(bf)
    q, sk, sv = n(B * W, T, H, D), n(B * W, T, HK, D), n(B * W, T, HK, D)
    pk, pv = n(B, L, HK, D), n(B, L, HK, D)
    lengths = torch.tensor([300, 17, 0, 160], device="cuda")
    mask = torch.arange(L, device="cuda")[None, :] < lengths[:, None]
    out = ops.prefix_attention(q, pk, pv, sk, sv, beam_width=W, prefix_mask=mask)
    ref = torch_ref.prefix_attention(q, pk, pv, sk, sv, W, mask=mask)
    assert_close_rel(out.float().cpu().numpy(), ref.cpu().numpy(), rel=5e-3, what="masked attention")
