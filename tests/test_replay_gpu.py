"""GPU parity of the beam-replay kernels (gated delta, conv1d, fused GDN mixer)."""

import numpy as np
import pytest
import torch

from oracle import grbeam_oracle as O
from tests import torch_ref
from tests.parity import assert_close_rel, bf16_tol, load

pytestmark = pytest.mark.gpu
DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def _t(a, dtype, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_gated_delta_matches_golden(dtype):
    from kadllm_b200 import ops

    g = load(f"ops_{dtype}.npz")
    d = DT[dtype]
    out = ops.gated_delta(_t(g["gd_q"], d), _t(g["gd_k"], d), _t(g["gd_v"], d),
                          _t(g["gd_g"], torch.float32), _t(g["gd_beta"], torch.float32),
                          _t(g["gd_s0"], d), beam_width=int(g["gd_W"]))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    if dtype == "fp32":
        np.testing.assert_allclose(got, g["gd_out"], atol=1e-4, rtol=1e-4)
    else:
        np.testing.assert_allclose(got, g["gd_out"], atol=bf16_tol(g["gd_out"], 1, 0), rtol=0)


@pytest.mark.parametrize("T", [1, 2, 3, 8])
@pytest.mark.parametrize("dims", [(2, 2, 128), (1, 2, 64)])
def test_gated_delta_matches_oracle(T, dims):
    from kadllm_b200 import ops

    H, rep, K = dims
    HV = H * rep
    B, W = 2, 37  # ragged beam chunks
    rng = np.random.default_rng(T)
    q = rng.standard_normal((B * W, T, H, K)).astype(np.float32)
    k = rng.standard_normal((B * W, T, H, K)).astype(np.float32)
    v = rng.standard_normal((B * W, T, HV, K)).astype(np.float32)
    g = -rng.uniform(0, 1, (B * W, T, HV)).astype(np.float32)
    beta = rng.uniform(0, 1, (B * W, T, HV)).astype(np.float32)
    s0 = O.bf16(0.3 * rng.standard_normal((B, HV, K, K)).astype(np.float32))
    bf = torch.bfloat16
    qb, kb, vb = (O.bf16(x) for x in (q, k, v))
    out = ops.gated_delta(_t(qb, bf), _t(kb, bf), _t(vb, bf), _t(g, torch.float32),
                          _t(O.bf16(beta), bf), _t(s0, bf), beam_width=W)
    ref = O.gated_delta(qb, kb, vb, g, O.bf16(beta), s0, beam_width=W)
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, ref, atol=bf16_tol(ref, 1, 0), rtol=0)
    # fp32 inputs and state: the hi/lo split keeps ~fp32 accuracy
    out32 = ops.gated_delta(_t(q, torch.float32), _t(k, torch.float32), _t(v, torch.float32),
                            _t(g, torch.float32), _t(beta, torch.float32),
                            _t(s0 + 1e-3, torch.float32), beam_width=W)
    ref32 = O.gated_delta(q, k, v, g, beta, s0 + np.float32(1e-3), beam_width=W)
    np.testing.assert_allclose(out32.cpu().numpy(), ref32, atol=2e-4, rtol=2e-4)


def test_gated_delta_full_size_matches_torch_fp32():
    """Step shape: 32 requests x 256 beams, 16 heads of 128, T = 1 and 2."""
    from kadllm_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(0)
    B, W, H, K = 32, 256, 16, 128
    for T in (1, 2):
        n = lambda *s: torch.randn(*s, device="cuda", generator=gen)
        q, k, v = (n(B * W, T, H, K).bfloat16() for _ in range(3))
        g = -torch.rand(B * W, T, H, device="cuda", generator=gen)
        beta = torch.rand(B * W, T, H, device="cuda", generator=gen).bfloat16()
        s0 = (0.1 * n(B, H, K, K)).bfloat16()
        snapshot = s0.clone()
        out = ops.gated_delta(q, k, v, g, beta, s0, beam_width=W)
        ref = torch_ref.gated_delta(q, k, v, g, beta, s0, W)
        assert torch.equal(s0, snapshot), "shared state was modified"
        assert_close_rel(out.float().cpu().numpy(), ref.cpu().numpy(), rel=5e-3, what=f"T={T}")


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_causal_conv1d_matches_golden(dtype):
    from kadllm_b200 import ops

    g = load(f"ops_{dtype}.npz")
    d = DT[dtype]
    out = ops.causal_conv1d(_t(g["cv_x"], d), _t(g["cv_state"], d), _t(g["cv_w"], d),
                            beam_width=int(g["cv_W"]))
    got = out.float().cpu().numpy()
    tol = 1e-5 if dtype == "fp32" else bf16_tol(g["cv_out"], 1, 0)
    np.testing.assert_allclose(got, g["cv_out"], atol=tol, rtol=0)


def test_causal_conv1d_strided_input_and_variants():
    from kadllm_b200 import ops

    rng = np.random.default_rng(0)
    B, W, C, T = 3, 5, 200, 3
    proj = rng.standard_normal((B * W, T, C + 16)).astype(np.float32)
    x = _t(proj, torch.float32)[:, :, 8:8 + C].transpose(1, 2)  # strided view
    state = _t(rng.standard_normal((B, C, 6)).astype(np.float32), torch.float32)
    w = _t(0.5 * rng.standard_normal((C, 4)).astype(np.float32), torch.float32)
    out = ops.causal_conv1d(x, state, w, beam_width=W)
    ref = O.causal_conv1d(x.cpu().numpy(), state.cpu().numpy(), w.cpu().numpy(), beam_width=W)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-5)
    before = state.clone()
    bias = _t(rng.standard_normal(C).astype(np.float32), torch.float32)
    out = ops.causal_conv1d(x, state, w, beam_width=W, bias=bias, activation=None)
    ref = O.causal_conv1d(x.cpu().numpy(), state.cpu().numpy(), w.cpu().numpy(), beam_width=W,
                          activation=None) + bias.cpu().numpy()[None, :, None]
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=1e-5)
    assert torch.equal(state, before)


@pytest.mark.parametrize("B,W,C,T", [(2, 1, 2048, 1024), (2, 3, 136, 100), (1, 2, 64, 16)])
def test_causal_conv1d_long_bf16_channel_contiguous(B, W, C, T):
    """The vectorised sliding window for long BF16 suffixes in the reference's layout
    (x = proj.transpose(1, 2), channels contiguous): the kernel microbenchmark's shape
    (2048 channels x 1024 steps), ragged channel / step tiles, T not a multiple of 8."""
    from kadllm_b200 import ops

    rng = np.random.default_rng(C + T)
    bf = torch.bfloat16
    proj = O.bf16(rng.standard_normal((B * W, T, C)).astype(np.float32))
    x = _t(proj, bf).transpose(1, 2)
    state = _t(O.bf16(rng.standard_normal((B, C, 4)).astype(np.float32)), bf)
    w = _t(O.bf16(0.5 * rng.standard_normal((C, 4)).astype(np.float32)), bf)
    bias = _t(O.bf16(rng.standard_normal(C).astype(np.float32)), bf)
    for b_, act in ((None, "silu"), (bias, None)):
        out = ops.causal_conv1d(x, state, w, beam_width=W, bias=b_, activation=act)
        xf, sf, wf = (t.float().cpu().numpy() for t in (x, state, w))
        ref = O.causal_conv1d(xf, sf, wf, beam_width=W, activation=None)
        if b_ is not None:
            ref = ref + b_.float().cpu().numpy()[None, :, None]
        if act == "silu":
            ref = ref / (1 + np.exp(-ref))
        ref = O.bf16(ref.astype(np.float32))  # one rounding of the fp32 result
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-3)


def test_operator_errors_match_reference_conventions():
    from kadllm_b200 import ops

    q = torch.zeros(4, 1, 2, 32, device="cuda")
    s = torch.zeros(2, 2, 32, 32, device="cuda")
    g = torch.zeros(4, 1, 2, device="cuda")
    with pytest.raises(ValueError):
        ops.gated_delta(q, q, q, g, g, s, beam_width=3)
    with pytest.raises(ValueError):
        ops.gated_delta(q, q, q.half(), g, g, s, beam_width=2)
    with pytest.raises(ValueError):
        ops.gated_delta(q, q, q, g, g, s, beam_width=2, triton_config=(7, 1, 1))
    with pytest.raises(RuntimeError):
        ops.gated_delta(q.cpu(), q.cpu(), q.cpu(), g.cpu(), g.cpu(), s.cpu(), beam_width=2)
    with pytest.raises(NotImplementedError):
        ops.gated_delta(torch.zeros(4, 9, 2, 32, device="cuda"), torch.zeros(4, 9, 2, 32, device="cuda"),
                        torch.zeros(4, 9, 2, 32, device="cuda"), torch.zeros(4, 9, 2, device="cuda"),
                        torch.zeros(4, 9, 2, device="cuda"), s, beam_width=2)


@pytest.mark.parametrize("K,H,HV", [(64, 2, 4), (128, 2, 4), (128, 4, 16)])
@pytest.mark.parametrize("T", [1, 2, 3])
def test_gdn_mixer_matches_oracle_composition(T, K, H, HV):
    """Fused conv + gates + replay + gated RMSNorm against the oracle's op chain
    (W = 33: a ragged last beam octet; the 0.8B head shape is K = 128, HV = 16)."""
    _mixer_case(T, K, H, HV, 2, 33)


@pytest.mark.parametrize("T", [1, 2])
def test_gdn_mixer_many_octets_per_warp(T):
    """160 (request, head) pairs x 250 beams: each warp of the staged kernel runs
    several beam octets through its two-part staging buffer, the last one ragged."""
    _mixer_case(T, 128, 4, 16, 10, 250)


def _mixer_case(T, K, H, HV, B, W):
    from kadllm_b200 import _lib

    rng = np.random.default_rng(10 + T + K + HV + W)
    kd, vd = H * K, HV * K
    C = 2 * kd + vd
    ld = C + vd + 2 * HV + 8
    BW = B * W
    proj = O.bf16(rng.standard_normal((BW * T, ld)).astype(np.float32))
    conv_state = O.bf16(rng.standard_normal((B, C, 4)).astype(np.float32))
    conv_w = O.bf16(0.5 * rng.standard_normal((C, 4)).astype(np.float32))
    rec = O.bf16(0.3 * rng.standard_normal((B, HV, K, K)).astype(np.float32))
    a_log = np.log(rng.uniform(1, 16, HV)).astype(np.float32)
    dt_bias = O.bf16(rng.uniform(-1, 1, HV).astype(np.float32))
    a_log = O.bf16(a_log)
    nw = O.bf16(1 + 0.1 * rng.standard_normal(K).astype(np.float32))
    bf = torch.bfloat16
    out = torch.empty(BW * T, vd, dtype=bf, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    tp = _t(proj, bf)
    args = [_t(conv_state, bf), _t(conv_w, bf), _t(rec, bf), _t(a_log, torch.float32),
            _t(dt_bias, torch.float32), _t(nw, torch.float32)]
    _lib.call("kadllm_gdn_mixer_replay", tp.data_ptr(), ld, args[0].data_ptr(), 4, args[1].data_ptr(),
              args[2].data_ptr(), args[3].data_ptr(), args[4].data_ptr(), args[5].data_ptr(), 1e-6,
              out.data_ptr(), B, W, T, H, HV, K, K, None, status.data_ptr(), _lib.stream(tp.device))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # oracle chain (src/kadllm/adapters/qwen3_5.py:144-177)
    r = O.Rounding("bf16")
    P = proj.reshape(BW, T, ld)
    x = np.swapaxes(P[..., :C], 1, 2)
    conv = np.swapaxes(O.causal_conv1d(x, conv_state, conv_w, beam_width=W, r=r), 1, 2)
    q = conv[..., :kd].reshape(BW, T, H, K)
    k = conv[..., kd:2 * kd].reshape(BW, T, H, K)
    v = conv[..., 2 * kd:].reshape(BW, T, HV, K)
    bcol, acol = P[..., C + vd:C + vd + HV], P[..., C + vd + HV:C + vd + 2 * HV]
    decay = (-np.exp(a_log) * O.softplus(acol + dt_bias)).astype(np.float32)
    beta = r(O.sigmoid(bcol))
    o = O.gated_delta(q, k, v, decay, beta, rec, beam_width=W, out_round=r)
    z = P[..., C:C + vd].reshape(-1, K)
    ref = O.rms_norm_gated(o.reshape(-1, K), z, nw, 1e-6, r).reshape(BW * T, vd)
    assert_close_rel(out.float().cpu().numpy(), ref, rel=1e-2, what="gdn mixer")
