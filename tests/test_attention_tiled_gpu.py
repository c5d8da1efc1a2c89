"""Tensor-core attention over a tiled prefix (kadllm_attention_tiled) against a
plain PyTorch fp32 restatement of the same op (src/kadllm/ops.py:252-341 for
decode; causal SDPA for prefill), with the fused output gate."""

import pytest
import torch

from kadllm_b200 import _lib
from tests.parity import assert_close_rel

pytestmark = pytest.mark.gpu
bf = torch.bfloat16
D = 256


def _tiles(cache):  # cache [B, HK, L, D]
    B, HK, L, _ = cache.shape
    nbytes = _lib.lib().kadllm_kv_tile_bytes(B, HK, L, D)
    t = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("kadllm_kv_tile", cache.data_ptr(), HK * L * D, D, L * D, B, HK, L, D, t.data_ptr(), nbytes,
              _lib.stream(cache.device))
    return t, -(-L // 64)


def _gate(o, g):  # bf16(bf16(o) * bf16(sigmoid(g)))
    return (o.to(bf).float() * torch.sigmoid(g.float()).to(bf).float()).to(bf)


@pytest.mark.parametrize("B,W,T,L,trend", [(2, 5, 2, 100, 0.0), (1, 40, 1, 64, 0.0), (1, 7, 3, 1100, 3.0)])
def test_decode_matches_torch(B, W, T, L, trend):
    hq, hk = 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(L + W)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = n(B * W, T, hq, D).to(bf)
    kc = n(B, hk, L, D)
    if trend:  # later keys align with the queries: row maxima keep rising (reference moves, O rescales)
        kc = kc + trend * torch.linspace(0, 1, L, device="cuda")[None, None, :, None] * q.float().mean((0, 1, 2))
    kc = kc.to(bf)
    vc = n(B, hk, L, D).to(bf)
    ks, vs = n(B * W, T, hk, D).to(bf), n(B * W, T, hk, D).to(bf)
    gate = n(B * W, T, hq, D).to(bf)
    out = torch.empty(B * W, T, hq, D, dtype=bf, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kt, nblk = _tiles(kc)
    vt, _ = _tiles(vc)
    _lib.call("kadllm_attention_tiled", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(), vt.data_ptr(), nblk,
              ks.data_ptr(), T * hk * D, hk * D, D, vs.data_ptr(), T * hk * D, hk * D, D, gate.data_ptr(),
              T * hq * D, hq * D, D, out.data_ptr(), T * hq * D, hq * D, D, status.data_ptr(), B, W, T, hq, hk, L, D,
              D ** -0.5, 0, _lib.stream(q.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # reference: per beam row, prefix keys then suffix keys s <= t
    ref = torch.empty(B * W, T, hq, D, device="cuda")
    for b in range(B):
        for w in range(W):
            r = b * W + w
            for t in range(T):
                for h in range(hq):
                    kv = h // G
                    keys = torch.cat([kc[b, kv].float(), ks[r, :t + 1, kv].float()])
                    vals = torch.cat([vc[b, kv].float(), vs[r, :t + 1, kv].float()])
                    p = torch.softmax(keys @ q[r, t, h].float() * D ** -0.5, 0)
                    ref[r, t, h] = p @ vals
    want = _gate(ref, gate)
    assert_close_rel(out.float().cpu().numpy(), want.float().cpu().numpy(), rel=1e-2, what="tiled decode attention")


@pytest.mark.parametrize("B,L", [(2, 130), (1, 64)])
def test_causal_matches_torch(B, L):
    hq, hk = 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(L)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = n(B * L, hq, D).to(bf)
    kc, vc = n(B, hk, L, D).to(bf), n(B, hk, L, D).to(bf)
    gate = n(B * L, hq, D).to(bf)
    out = torch.empty(B * L, hq, D, dtype=bf, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kt, nblk = _tiles(kc)
    vt, _ = _tiles(vc)
    _lib.call("kadllm_attention_tiled", q.data_ptr(), hq * D, 0, D, kt.data_ptr(), vt.data_ptr(), nblk, None, 0, 0, 0,
              None, 0, 0, 0, gate.data_ptr(), hq * D, 0, D, out.data_ptr(), hq * D, 0, D, status.data_ptr(), B, 1, 1,
              hq, hk, L, D, D ** -0.5, 1, _lib.stream(q.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    qh = q.float().view(B, L, hq, D).permute(0, 2, 1, 3)
    kh = kc.float().repeat_interleave(G, 1)
    vh = vc.float().repeat_interleave(G, 1)
    s = qh @ kh.transpose(-1, -2) * D ** -0.5
    s = s.masked_fill(~torch.tril(torch.ones(L, L, dtype=torch.bool, device="cuda")), float("-inf"))
    ref = (torch.softmax(s, -1) @ vh).permute(0, 2, 1, 3).reshape(B * L, hq, D)
    want = _gate(ref, gate)
    assert_close_rel(out.float().cpu().numpy(), want.float().cpu().numpy(), rel=1e-2, what="tiled causal attention")
