"""Per-kernel GPU parity of the model building blocks against the oracle's pieces."""

import numpy as np
import pytest
import torch

from kadllm_b200 import _lib
from oracle import grbeam_oracle as O
from tests.parity import assert_close_rel

pytestmark = pytest.mark.gpu
bf = torch.bfloat16
R = O.Rounding("bf16")


def T(a, dtype=bf):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(dtype)


def N(t):
    return t.float().cpu().numpy()


def S():
    return _lib.stream(torch.device("cuda"))


@pytest.mark.parametrize("H", [128, 1024])
def test_embed_and_add_rmsnorm(H):
    rng = np.random.default_rng(H)
    V, rows = 300, 37
    table = O.bf16(rng.standard_normal((V, H)).astype(np.float32))
    w = O.bf16(0.1 * rng.standard_normal(H).astype(np.float32))
    ids = rng.integers(0, V, rows)
    x = torch.empty(rows, H, dtype=bf, device="cuda")
    nrm = torch.empty_like(x)
    tid = torch.from_numpy(ids).cuda()
    ttab, wt = T(table), T(w, torch.float32)
    _lib.call("kadllm_embed_rmsnorm", tid.data_ptr(), ttab.data_ptr(), V, wt.data_ptr(), 1e-6,
              x.data_ptr(), nrm.data_ptr(), rows, H, S())
    np.testing.assert_array_equal(N(x), table[ids])
    assert_close_rel(N(nrm), O.rms_norm(table[ids], w, 1e-6, R), rel=5e-3, what="embed norm")
    delta = O.bf16(rng.standard_normal((rows, H)).astype(np.float32))
    td = T(delta)
    _lib.call("kadllm_add_rmsnorm", x.data_ptr(), td.data_ptr(), H, wt.data_ptr(), 1e-6, nrm.data_ptr(), rows,
              1, 0, H, S())
    xr = R(table[ids] + delta)
    np.testing.assert_array_equal(N(x), xr)
    assert_close_rel(N(nrm), O.rms_norm(xr, w, 1e-6, R), rel=5e-3, what="add norm")
    last = torch.empty(3, H, dtype=bf, device="cuda")
    _lib.call("kadllm_add_rmsnorm", x.data_ptr(), None, 0, wt.data_ptr(), 1e-6, last.data_ptr(), 3, 12, 11, H, S())
    assert_close_rel(N(last), O.rms_norm(xr[11::12][:3], w, 1e-6, R), rel=5e-3, what="strided norm")


def test_silu_mul():
    rng = np.random.default_rng(0)
    rows, inter = 19, 384
    gu = O.bf16(rng.standard_normal((rows, 2 * inter)).astype(np.float32))
    out = torch.empty(rows, inter, dtype=bf, device="cuda")
    tgu = T(gu)
    _lib.call("kadllm_silu_mul", tgu.data_ptr(), 2 * inter, inter, out.data_ptr(), rows, S())
    ref = R(R(O.silu(gu[:, :inter])) * gu[:, inter:])
    assert_close_rel(N(out), ref, rel=5e-3, what="silu_mul")


@pytest.mark.parametrize("D,hq,hk,factor,B,L", [
    (32, 4, 2, 0.25, 2, 9),
    (256, 8, 2, 0.25, 2, 9),     # 64 rotary dims: the two-dims-per-lane kernel
    (256, 8, 2, 0.25, 3, 701),   # ... over many row blocks; sequences end inside a warp's rows
    (256, 8, 2, 0.125, 2, 9),    # 32 rotary dims: the eight-dims-per-lane kernel
])
def test_qk_norm_rope_prefill_and_decode(D, hq, hk, factor, B, L):
    from kadllm_b200.config import TINY

    cfg = TINY.with_(head_dim=D, num_attention_heads=hq, num_key_value_heads=hk, rope_theta=1e7,
                     partial_rotary_factor=factor)
    rng = np.random.default_rng(D + L)
    rows = B * L
    ld = (2 * hq + 2 * hk) * D
    P = O.bf16(rng.standard_normal((rows, ld)).astype(np.float32))
    qw = O.bf16(0.1 * rng.standard_normal(D).astype(np.float32))
    kw = O.bf16(0.1 * rng.standard_normal(D).astype(np.float32))
    rot = cfg.rotary_dim
    pos = torch.arange(L + 5, device="cuda", dtype=torch.float32)
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, device="cuda").float() / rot))
    emb = torch.cat([pos[:, None] * inv, pos[:, None] * inv], -1)
    cos, sin = emb.cos().to(bf).contiguous(), emb.sin().to(bf).contiguous()
    q = torch.empty(rows, hq, D, dtype=bf, device="cuda")
    kc = torch.zeros(B, hk, L, D, dtype=bf, device="cuda")
    vc = torch.zeros_like(kc)
    st = (hk * L * D, D, L * D)
    tP, tqw, tkw = T(P), T(qw, torch.float32), T(kw, torch.float32)
    _lib.call("kadllm_qk_norm_rope", tP.data_ptr(), ld, hq, hk, D, tqw.data_ptr(),
              tkw.data_ptr(), 1e-6, cos.data_ptr(), sin.data_ptr(), rot, None, 5, L,
              q.data_ptr(), hq * D, D, kc.data_ptr(), *st, vc.data_ptr(), *st, rows, S())
    c_np, s_np = N(cos)[5:5 + L], N(sin)[5:5 + L]
    x = P.reshape(B, L, -1)
    qs = x[..., : 2 * hq * D].reshape(B, L, hq, 2 * D)[..., :D]
    ks = x[..., 2 * hq * D: 2 * hq * D + hk * D].reshape(B, L, hk, D)
    vs = x[..., 2 * hq * D + hk * D:].reshape(B, L, hk, D)
    rq = O.apply_rotary(O.rms_norm(qs, qw, 1e-6, R), c_np, s_np, R)
    rk = O.apply_rotary(O.rms_norm(ks, kw, 1e-6, R), c_np, s_np, R)
    assert_close_rel(N(q).reshape(B, L, hq, D), rq, rel=5e-3, what="q")
    assert_close_rel(N(kc).transpose(0, 2, 1, 3), rk, rel=5e-3, what="k")
    np.testing.assert_array_equal(N(vc).transpose(0, 2, 1, 3), vs)


@pytest.mark.parametrize("D,hq,hk,L", [(32, 4, 2, 64), (256, 8, 2, 100)])
def test_causal_attention_prefill(D, hq, hk, L):
    rng = np.random.default_rng(D + L)
    B = 2
    q = O.bf16(rng.standard_normal((B * L, hq, D)).astype(np.float32))
    k = O.bf16(rng.standard_normal((B, hk, L, D)).astype(np.float32))
    v = O.bf16(rng.standard_normal((B, hk, L, D)).astype(np.float32))
    gate = O.bf16(rng.standard_normal((B * L, hq, 2 * D)).astype(np.float32))  # gate at [..., D:]
    tq, tk, tv, tg = T(q), T(k), T(v), T(gate)
    out = torch.empty(B * L, hq * D, dtype=bf, device="cuda")
    gp = tg[..., D:]
    # k / v [B, HK, L, D]: strides passed as (request, position, head)
    _lib.call("kadllm_causal_attention", tq.data_ptr(), hq * D, D, tk.data_ptr(), tk.stride(0), tk.stride(2),
              tk.stride(1), tv.data_ptr(), tv.stride(0), tv.stride(2), tv.stride(1), gp.data_ptr(), hq * 2 * D, 2 * D,
              out.data_ptr(), hq * D, D, B, L, hq, hk, D, D ** -0.5, S())
    qh = q.reshape(B, L, hq, D).transpose(0, 2, 1, 3)
    kh = np.repeat(k, hq // hk, axis=1)
    vh = np.repeat(v, hq // hk, axis=1)
    s = np.matmul(qh, kh.transpose(0, 1, 3, 2)) * np.float32(D ** -0.5)
    s = np.where(np.tril(np.ones((L, L), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    o = R(np.matmul(p / p.sum(-1, keepdims=True), vh)).transpose(0, 2, 1, 3).reshape(B * L, hq * D)
    ref = R(o * R(O.sigmoid(gate[..., D:].reshape(B * L, hq * D))))
    assert_close_rel(N(out), ref, rel=1e-2, what="causal attention")


@pytest.mark.parametrize("K,H,L", [(32, 4, 100), (128, 2, 130), (128, 2, 64), (64, 2, 3), (128, 2, 300),
                                   (128, 1, 1024)])
def test_gdn_prefill_matches_oracle(K, H, L):
    """Conv + gates + chunked rule (WY form) + gated norm from the packed
    projection, and the conv / recurrent prefix states, against the oracle's
    restatement.  L = 300 and 1024 run 5 and 16 chunks, so both pipeline stages
    of the scan are reused many times."""
    rng = np.random.default_rng(K + L + 7)
    B, HV = 2, H
    kd, vd = H * K, HV * K
    C = 2 * kd + vd
    ld = (C + vd + 2 * HV + 7) // 8 * 8  # projection rows padded to 16 bytes
    P = O.bf16(rng.standard_normal((B * L, ld)).astype(np.float32))
    cw = O.bf16(0.5 * rng.standard_normal((C, 4)).astype(np.float32))
    a_log = O.bf16(np.log(rng.uniform(1, 16, HV)).astype(np.float32))
    dtb = O.bf16(rng.uniform(-1, 1, HV).astype(np.float32))
    nw = O.bf16(1 + 0.1 * rng.standard_normal(K).astype(np.float32))
    keep = [T(P), T(cw), T(a_log, torch.float32), T(dtb, torch.float32), T(nw, torch.float32)]
    out = torch.empty(B * L, vd, dtype=bf, device="cuda")
    state = torch.empty(B, HV, K, K, dtype=bf, device="cuda")
    cstate = torch.empty(B, C, 4, dtype=bf, device="cuda")
    nbytes = _lib.lib().kadllm_gdn_prefill_workspace(B, L, HV, K, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("kadllm_gdn_prefill_split", keep[0].data_ptr(), ld, keep[1].data_ptr(), cstate.data_ptr(),
              keep[2].data_ptr(), keep[3].data_ptr(), keep[4].data_ptr(), 1e-6, out.data_ptr(), vd,
              state.data_ptr(), ws.data_ptr(), nbytes, B, L, H, HV, K, K, S())
    x = P[:, :C].reshape(B, L, C).transpose(0, 2, 1)  # B C L
    xp = np.concatenate([np.zeros((B, C, 3), np.float32), x], -1)
    conv = R(O.silu(sum(xp[:, :, j:j + L] * cw[None, :, j:j + 1] for j in range(4)))).transpose(0, 2, 1)
    q = conv[..., :kd].reshape(B, L, H, K)
    k = conv[..., kd:2 * kd].reshape(B, L, H, K)
    v = conv[..., 2 * kd:].reshape(B, L, HV, K)
    Pz = P.reshape(B, L, ld)
    beta = R(O.sigmoid(Pz[..., C + vd:C + vd + HV]))
    g = (-np.exp(a_log) * O.softplus(Pz[..., C + vd + HV:C + vd + 2 * HV] + dtb)).astype(np.float32)
    o, st = O.chunk_gated_delta_rule(q, k, v, g, beta, O.Rounding("fp32"))
    ref = O.rms_norm_gated(R(o).reshape(-1, K), Pz[..., C:C + vd].reshape(-1, K), nw, 1e-6, R).reshape(B * L, vd)
    pad = np.concatenate([np.zeros((B, C, 4), np.float32), x], -1)[:, :, -4:]
    np.testing.assert_array_equal(N(cstate), pad)
    assert_close_rel(N(state), st, rel=1e-2, what="final state")
    assert_close_rel(N(out), ref, rel=1e-2, what="gated output")


def test_gdn_prefill_benchmark_shape_sampled_heads():
    """The benchmark's prefill launch (32 requests x 1024 tokens, 16 heads of 128: 8192
    prep CTAs, 512 scan CTAs over several waves) against the oracle on sampled
    (request, head) pairs: output, final state and conv state."""
    B, L, H, HV, K = 32, 1024, 16, 16, 128
    kd, vd = H * K, HV * K
    C = 2 * kd + vd
    ld = C + vd + 2 * HV
    g = torch.Generator(device="cuda").manual_seed(11)
    P = torch.randn(B * L, ld, device="cuda", generator=g).to(bf)
    cw = (0.5 * torch.randn(C, 4, device="cuda", generator=g)).to(bf)
    a_log = torch.log(1 + 15 * torch.rand(HV, device="cuda", generator=g)).to(bf).float()
    dtb = (2 * torch.rand(HV, device="cuda", generator=g) - 1).to(bf).float()
    nw = (1 + 0.1 * torch.randn(K, device="cuda", generator=g)).to(bf).float()
    out = torch.empty(B * L, vd, dtype=bf, device="cuda")
    state = torch.empty(B, HV, K, K, dtype=bf, device="cuda")
    cstate = torch.empty(B, C, 4, dtype=bf, device="cuda")
    nbytes = _lib.lib().kadllm_gdn_prefill_workspace(B, L, HV, K, K)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("kadllm_gdn_prefill_split", P.data_ptr(), ld, cw.data_ptr(), cstate.data_ptr(), a_log.data_ptr(),
              dtb.data_ptr(), nw.data_ptr(), 1e-6, out.data_ptr(), vd, state.data_ptr(), ws.data_ptr(), nbytes,
              B, L, H, HV, K, K, S())
    torch.cuda.synchronize()
    cwn, aln, dtn, nwn = N(cw), N(a_log), N(dtb), N(nw)
    for b, h in [(0, 0), (13, 7), (31, 15)]:
        cols = np.r_[h * K:(h + 1) * K, kd + h * K:kd + (h + 1) * K, 2 * kd + h * K:2 * kd + (h + 1) * K]
        Pb = N(P[b * L:(b + 1) * L])
        x = Pb[:, cols].T[None]  # 1 x 3K x L
        xp = np.concatenate([np.zeros((1, 3 * K, 3), np.float32), x], -1)
        conv = R(O.silu(sum(xp[:, :, j:j + L] * cwn[cols][None, :, j:j + 1] for j in range(4)))).transpose(0, 2, 1)
        q, k, v = (conv[..., i * K:(i + 1) * K].reshape(1, L, 1, K) for i in range(3))
        beta = R(O.sigmoid(Pb[:, C + vd + h]))[None, :, None]
        gg = (-np.exp(aln[h]) * O.softplus(Pb[:, C + vd + HV + h] + dtn[h])).astype(np.float32)[None, :, None]
        o, st = O.chunk_gated_delta_rule(q, k, v, gg, beta, O.Rounding("fp32"))
        ref = O.rms_norm_gated(R(o).reshape(-1, K), Pb[:, C + h * K:C + (h + 1) * K], nwn, 1e-6, R)
        got = N(out[b * L:(b + 1) * L, h * K:(h + 1) * K])
        assert_close_rel(got, ref, rel=1e-2, what=f"gated output (request {b}, head {h})")
        assert_close_rel(N(state[b, h]), st[0, 0], rel=1e-2, what=f"final state (request {b}, head {h})")
        np.testing.assert_array_equal(N(cstate[b, cols]), x[0, :, -4:])
