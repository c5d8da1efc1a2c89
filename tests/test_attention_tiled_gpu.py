"""Tensor-core attention over a tiled prefix (kadllm_attention_tiled) against a
plain PyTorch fp32 restatement of the same op (src/kadllm/ops.py:252-341 for
decode; causal SDPA for prefill), with the fused output gate."""

import numpy as np
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


@pytest.mark.parametrize("B,W,T,L,trend,t0", [(2, 5, 2, 100, 0.0, 0), (1, 40, 1, 64, 0.0, 0), (1, 7, 3, 1100, 3.0, 0),
                                               (2, 5, 2, 100, 0.0, 1), (1, 7, 3, 1100, 3.0, 2)])
def test_decode_matches_torch(B, W, T, L, trend, t0):
    """Decode rows (beam, t) against prefix + suffix keys s <= t; with first_step t0 > 0
    only the steps t >= t0 have query rows (earlier suffix tokens stay keys)."""
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
    out = torch.zeros(B * W, T, hq, D, dtype=bf, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kt, nblk = _tiles(kc)
    vt, _ = _tiles(vc)
    _lib.call("kadllm_attention_tiled", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(), vt.data_ptr(), nblk,
              ks.data_ptr(), T * hk * D, hk * D, D, vs.data_ptr(), T * hk * D, hk * D, D, gate.data_ptr(),
              T * hq * D, hq * D, D, out.data_ptr(), T * hq * D, hq * D, D, status.data_ptr(), B, W, T, t0, hq, hk, L,
              D, D ** -0.5, 0, _lib.stream(q.device))
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
    assert_close_rel(out[:, t0:].float().cpu().numpy(), want[:, t0:].float().cpu().numpy(), rel=1e-2,
                     what="tiled decode attention")
    assert int(out[:, :t0].abs().sum()) == 0  # no rows for the steps before t0


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
              0, hq, hk, L, D, D ** -0.5, 1, _lib.stream(q.device))
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


def test_decode_at_the_benchmark_shape_sampled():
    """The timed decode launch: 32 requests x 256 beams, T = 2, prefix 1024 (1024
    CTAs of 128 query rows, every K/V buffer phase reused over 16 key blocks), plus the
    continuation form (first_step 1: queries of the newest token only), checked
    against fp32 torch on sampled (request, beam, head) rows."""
    B, W, T, L, hq, hk = 32, 256, 2, 1024, 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(11)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = n(B * W, T, hq, D).to(bf)
    kc, vc = n(B, hk, L, D).to(bf), n(B, hk, L, D).to(bf)
    ks, vs = n(B * W, T, hk, D).to(bf), n(B * W, T, hk, D).to(bf)
    gate = n(B * W, T, hq, D).to(bf)
    kt, nblk = _tiles(kc)
    vt, _ = _tiles(vc)
    rng = np.random.default_rng(0)
    for t0 in (0, 1):
        out = torch.zeros(B * W, T, hq, D, dtype=bf, device="cuda")
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.call("kadllm_attention_tiled", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(), vt.data_ptr(),
                  nblk, ks.data_ptr(), T * hk * D, hk * D, D, vs.data_ptr(), T * hk * D, hk * D, D, gate.data_ptr(),
                  T * hq * D, hq * D, D, out.data_ptr(), T * hq * D, hq * D, D, status.data_ptr(), B, W, T, t0, hq,
                  hk, L, D, D ** -0.5, 0, _lib.stream(q.device))
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        got, want = [], []
        for _ in range(48):
            b, w, h = int(rng.integers(B)), int(rng.integers(W)), int(rng.integers(hq))
            t = int(rng.integers(t0, T))
            r, kv = b * W + w, h // G
            keys = torch.cat([kc[b, kv].float(), ks[r, :t + 1, kv].float()])
            vals = torch.cat([vc[b, kv].float(), vs[r, :t + 1, kv].float()])
            p = torch.softmax(keys @ q[r, t, h].float() * D ** -0.5, 0)
            want.append(_gate((p @ vals)[None], gate[r, t, h][None])[0].float())
            got.append(out[r, t, h].float())
        assert_close_rel(torch.stack(got).cpu().numpy(), torch.stack(want).cpu().numpy(), rel=1e-2,
                         what=f"decode attention at the benchmark shape (first_step {t0})")


def test_causal_at_the_benchmark_shape_sampled():
    """The timed prefill launch: 32 requests x 1024 tokens (causal), sampled rows."""
    B, L, hq, hk = 32, 1024, 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(12)
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
              0, hq, hk, L, D, D ** -0.5, 1, _lib.stream(q.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    rng = np.random.default_rng(1)
    got, want = [], []
    for _ in range(64):
        b, pos, h = int(rng.integers(B)), int(rng.integers(L)), int(rng.integers(hq))
        kv = h // G
        p = torch.softmax(kc[b, kv, :pos + 1].float() @ q[b * L + pos, h].float() * D ** -0.5, 0)
        want.append(_gate((p @ vc[b, kv, :pos + 1].float())[None], gate[b * L + pos, h][None])[0].float())
        got.append(out[b * L + pos, h].float())
    assert_close_rel(torch.stack(got).cpu().numpy(), torch.stack(want).cpu().numpy(), rel=1e-2,
                     what="causal attention at the benchmark shape")


@pytest.mark.parametrize("B,W,T,L,t0,splits", [(1, 40, 3, 1100, 0, 3), (2, 5, 2, 100, 1, 2), (1, 7, 1, 4096, 0, 64)])
def test_split_decode_matches_torch(B, W, T, L, t0, splits):
    """kadllm_attention_tiled_split: key blocks split over CTAs, partials merged with the
    suffix keys and the gate by the combine kernel (one split per key block at most)."""
    hq, hk = 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(L + W + splits)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen)
    q = n(B * W, T, hq, D).to(bf)
    kc, vc = n(B, hk, L, D).to(bf), n(B, hk, L, D).to(bf)
    ks, vs = n(B * W, T, hk, D).to(bf), n(B * W, T, hk, D).to(bf)
    gate = n(B * W, T, hq, D).to(bf)
    out = torch.zeros(B * W, T, hq, D, dtype=bf, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kt, nblk = _tiles(kc)
    vt, _ = _tiles(vc)
    nbytes = _lib.lib().kadllm_attention_split_workspace(B, W, T, t0, hq, splits)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
    _lib.call("kadllm_attention_tiled_split", q.data_ptr(), T * hq * D, hq * D, D, kt.data_ptr(), vt.data_ptr(), nblk,
              ks.data_ptr(), T * hk * D, hk * D, D, vs.data_ptr(), T * hk * D, hk * D, D, gate.data_ptr(),
              T * hq * D, hq * D, D, out.data_ptr(), T * hq * D, hq * D, D, status.data_ptr(), B, W, T, t0, hq, hk, L,
              D, D ** -0.5, splits, ws.data_ptr(), ws.numel(), _lib.stream(q.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = torch.zeros(B * W, T, hq, D, device="cuda")
    for b in range(B):
        for w in range(W):
            r = b * W + w
            for t in range(t0, T):
                for h in range(hq):
                    kv = h // G
                    keys = torch.cat([kc[b, kv].float(), ks[r, :t + 1, kv].float()])
                    vals = torch.cat([vc[b, kv].float(), vs[r, :t + 1, kv].float()])
                    p = torch.softmax(keys @ q[r, t, h].float() * D ** -0.5, 0)
                    ref[r, t, h] = p @ vals
    want = _gate(ref, gate)
    assert_close_rel(out[:, t0:].float().cpu().numpy(), want[:, t0:].float().cpu().numpy(), rel=1e-2,
                     what="split decode attention")


def test_public_op_long_prefix_few_requests():
    """ops.prefix_attention at the kernel microbenchmark's shape (1 request x 256 beams x
    3 steps, 4096 prefix keys: the split path), sampled rows against fp32 torch."""
    from kadllm_b200 import ops

    B, W, T, L, hq, hk = 1, 256, 3, 4096, 8, 2
    G = hq // hk
    gen = torch.Generator(device="cuda").manual_seed(5)
    n = lambda *s: torch.randn(*s, device="cuda", generator=gen).to(bf)
    q, sk, sv = n(B * W, T, hq, D), n(B * W, T, hk, D), n(B * W, T, hk, D)
    pk, pv = n(B, L, hk, D), n(B, L, hk, D)
    out = ops.prefix_attention(q, pk, pv, sk, sv, beam_width=W)
    rng = np.random.default_rng(2)
    got, want = [], []
    for _ in range(32):
        w, t, h = int(rng.integers(W)), int(rng.integers(T)), int(rng.integers(hq))
        kv = h // G
        keys = torch.cat([pk[0, :, kv].float(), sk[w, :t + 1, kv].float()])
        vals = torch.cat([pv[0, :, kv].float(), sv[w, :t + 1, kv].float()])
        p = torch.softmax(keys @ q[w, t, h].float() * D ** -0.5, 0)
        want.append(p @ vals)
        got.append(out[w, t, h].float())
    assert_close_rel(torch.stack(got).cpu().numpy(), torch.stack(want).cpu().numpy(), rel=1e-2,
                     what="public prefix attention, long prefix")
