"""Kernel microbenchmarks at the benchmark shapes (seeded synthetic inputs).

    python -m kadllm_b200.kernel_bench --case CASE [--reps N]

Cases (the kernel microbenchmark shapes and the GRBeam step shapes):
  prefill  chunked gated-delta prefill (conv + gates + UT transform + scan +
           gated norm) from the packed projection: B=32, T=1024, 16 heads of 128
  conv     causal conv1d width 4 + SiLU over T=1024, 2048 channels (B=32)
  attn     shared-prefix decode attention: 256 beams x 8 q / 2 kv heads x d=256
           against a 4096-token prefix plus a 3-token causal suffix, through the
           public op (prefix re-layout included; attn_split: the kernels alone;
           attn_tiled:
           the tcgen05 kernel over the tiled prefix; attn_step: the GRBeam
           step's second decode, 32 requests x 256 beams, prefix 1024, T=2;
           attn_causal: the prefill's causal attention, 32 x 1024 tokens)
  mixer    fused GDN decode mixer: 32 requests x 256 beams, T = 1 and 2
  select   one selection step over 32 x 256 x 248320 bf16 logits
  gemm_*   the tcgen05 projection GEMM at the step's shapes (cuBLAS timed beside it)
Each prints one JSON line: device time per call (CUDA events, after warm-up),
algorithmic work, achieved rate and the fraction of the measured B200 peak.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from . import _lib, ops

ROOT = Path(__file__).resolve().parent.parent


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def _time(fn, reps: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def _time_graph(fn, reps: int, warmup: int = 3) -> float:
    """Per-call device time of `reps` calls replayed from one CUDA graph, so
    that the host's launch cost of a short kernel stays out of the number."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def case_prefill(gen, reps, B=32):
    dev, bf = torch.device("cuda"), torch.bfloat16
    L, H, HV, K = 1024, 16, 16, 128
    C = 2 * H * K + HV * K
    ld = C + HV * K + 2 * HV
    P = torch.randn(B * L, ld, device=dev, generator=gen).to(bf)
    cw = (0.3 * torch.randn(C, 4, device=dev, generator=gen)).to(bf)
    al = torch.rand(HV, device=dev, generator=gen) * 2
    dt = torch.rand(HV, device=dev, generator=gen)
    nw = torch.ones(K, device=dev)
    out = torch.empty(B * L, HV * K, device=dev, dtype=bf)
    st = torch.empty(B, HV, K, K, device=dev, dtype=bf)
    cs = torch.empty(B, C, 4, device=dev, dtype=bf)
    nb = _lib.lib().kadllm_gdn_prefill_workspace(B, L, HV, K, K)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    s = _lib.stream(dev)

    def run():
        _lib.call("kadllm_gdn_prefill_split", P.data_ptr(), ld, cw.data_ptr(), cs.data_ptr(), al.data_ptr(),
                  dt.data_ptr(), nw.data_ptr(), 1e-6, out.data_ptr(), HV * K, st.data_ptr(), ws.data_ptr(), nb,
                  B, L, H, HV, K, K, s)

    ms = _time(run, reps)
    # compulsory HBM bytes: projection read once, output and both states written
    return ms, "hbm", B * L * ld * 2 + B * L * HV * K * 2 + B * HV * K * K * 2 + B * C * 4 * 2


def case_conv(gen, reps):
    dev, bf = torch.device("cuda"), torch.bfloat16
    B, C, T = 32, 2048, 1024
    x = torch.randn(B, T, C, device=dev, generator=gen).to(bf).transpose(1, 2)  # [B, C, T] view
    state = torch.zeros(B, C, 3, device=dev, dtype=bf)
    w = (0.3 * torch.randn(C, 4, device=dev, generator=gen)).to(bf)
    ms = _time(lambda: ops.causal_conv1d(x, state, w, beam_width=1), reps)
    return ms, "hbm", B * C * T * 2 * 2


def case_attn(gen, reps):
    dev, bf = torch.device("cuda"), torch.bfloat16
    B, W, T, L, Hq, HK, D = 1, 256, 3, 4096, 8, 2, 256
    n = lambda *s: torch.randn(*s, device=dev, generator=gen).to(bf)
    q, sk, sv = n(B * W, T, Hq, D), n(B * W, T, HK, D), n(B * W, T, HK, D)
    pk, pv = n(B, L, HK, D), n(B, L, HK, D)
    ms = _time(lambda: ops.prefix_attention(q, pk, pv, sk, sv, beam_width=W), reps)
    return ms, "tensor", 4 * B * W * T * Hq * D * L + 4 * B * W * Hq * D * T * (T + 1) / 2


def case_attn_split(gen, reps, B=1, W=256, T=3, L=4096):
    """The decode attention kernels alone at the microbenchmark shape (prefix tiled once
    outside the timed loop): the key-block split over 3 CTAs per row tile + the combine."""
    dev, bf = torch.device("cuda"), torch.bfloat16
    Hq, HK, D = 8, 2, 256
    n = lambda *s: torch.randn(*s, device=dev, generator=gen).to(bf)
    q = n(B * W, T, Hq, D)
    sk, sv = n(B * W, T, HK, D), n(B * W, T, HK, D)
    kc, vc = n(B, HK, L, D), n(B, HK, L, D)
    nbytes = _lib.lib().kadllm_kv_tile_bytes(B, HK, L, D)
    kt = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    vt = torch.empty_like(kt)
    s = _lib.stream(dev)
    _lib.call("kadllm_kv_tile", kc.data_ptr(), HK * L * D, D, L * D, B, HK, L, D, kt.data_ptr(), nbytes, s)
    _lib.call("kadllm_kv_tile", vc.data_ptr(), HK * L * D, D, L * D, B, HK, L, D, vt.data_ptr(), nbytes, s)
    out = torch.empty(B * W, T, Hq, D, dtype=bf, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    ctas = -(-(W * T * (Hq // HK)) // 128) * B * HK
    splits = max(1, min(sms // ctas, -(-L // 64), 64))
    ws = torch.empty(max(_lib.lib().kadllm_attention_split_workspace(B, W, T, 0, Hq, splits), 16), dtype=torch.uint8,
                     device=dev)

    def run():
        _lib.call("kadllm_attention_tiled_split", q.data_ptr(), T * Hq * D, Hq * D, D, kt.data_ptr(), vt.data_ptr(),
                  -(-L // 64), sk.data_ptr(), T * HK * D, HK * D, D, sv.data_ptr(), T * HK * D, HK * D, D, None, 0, 0,
                  0, out.data_ptr(), T * Hq * D, Hq * D, D, status.data_ptr(), B, W, T, 0, Hq, HK, L, D, D ** -0.5,
                  splits, ws.data_ptr(), ws.numel(), s)

    ms = _time(run, reps)
    if int(status.item()):
        raise RuntimeError("tiled attention reported a timed-out wait")
    return ms, "tensor", 4 * B * W * T * Hq * D * L + 4 * B * W * Hq * D * T * (T + 1) / 2, {"splits": splits}


def case_attn_tiled(gen, reps, B=1, W=256, T=3, L=4096, causal=False):
    dev, bf = torch.device("cuda"), torch.bfloat16
    Hq, HK, D = 8, 2, 256
    n = lambda *s: torch.randn(*s, device=dev, generator=gen).to(bf)
    R = B * L if causal else B * W  # causal: one query row per prefix token
    q, gate = n(R, T, Hq, D), n(R, T, Hq, D)
    sk, sv = n(B * W, T, HK, D), n(B * W, T, HK, D)
    kc, vc = n(B, HK, L, D), n(B, HK, L, D)
    nbytes = _lib.lib().kadllm_kv_tile_bytes(B, HK, L, D)
    kt = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    vt = torch.empty_like(kt)
    s = _lib.stream(dev)
    _lib.call("kadllm_kv_tile", kc.data_ptr(), HK * L * D, D, L * D, B, HK, L, D, kt.data_ptr(), nbytes, s)
    _lib.call("kadllm_kv_tile", vc.data_ptr(), HK * L * D, D, L * D, B, HK, L, D, vt.data_ptr(), nbytes, s)
    out = torch.empty(R, T, Hq, D, dtype=bf, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    nblk = -(-L // 64)

    def run():
        if causal:
            _lib.call("kadllm_attention_tiled", q.data_ptr(), Hq * D, 0, D, kt.data_ptr(), vt.data_ptr(), nblk,
                      None, 0, 0, 0, None, 0, 0, 0, gate.data_ptr(), Hq * D, 0, D, out.data_ptr(), Hq * D, 0, D,
                      status.data_ptr(), B, 1, 1, 0, Hq, HK, L, D, D ** -0.5, 1, s)
        else:
            _lib.call("kadllm_attention_tiled", q.data_ptr(), T * Hq * D, Hq * D, D, kt.data_ptr(), vt.data_ptr(),
                      nblk, sk.data_ptr(), T * HK * D, HK * D, D, sv.data_ptr(), T * HK * D, HK * D, D,
                      gate.data_ptr(), T * Hq * D, Hq * D, D, out.data_ptr(), T * Hq * D, Hq * D, D,
                      status.data_ptr(), B, W, T, 0, Hq, HK, L, D, D ** -0.5, 0, s)

    ms = _time(run, reps)
    if int(status.item()):
        raise RuntimeError("tiled attention reported a timed-out wait")
    if causal:
        return ms, "tensor", 4 * B * Hq * D * L * (L + 1) / 2
    return ms, "tensor", 4 * B * W * T * Hq * D * L + 4 * B * W * Hq * D * T * (T + 1) / 2


def case_mixer(gen, reps, T=1):
    dev, bf = torch.device("cuda"), torch.bfloat16
    B, W, H, HV, K = 32, 256, 16, 16, 128
    C = 2 * H * K + HV * K
    ld = C + HV * K + 2 * HV
    proj = (0.5 * torch.randn(B * W * T, ld, device=dev, generator=gen)).to(bf)
    cs = torch.randn(B, C, 4, device=dev, generator=gen).to(bf)
    cw = (0.3 * torch.randn(C, 4, device=dev, generator=gen)).to(bf)
    rec = (0.1 * torch.randn(B, HV, K, K, device=dev, generator=gen)).to(bf)
    al = torch.rand(HV, device=dev, generator=gen) * 2
    dt = torch.rand(HV, device=dev, generator=gen)
    nw = torch.ones(K, device=dev)
    out = torch.empty(B * W * T, HV * K, device=dev, dtype=bf)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    s = _lib.stream(dev)

    def run():
        _lib.call("kadllm_gdn_mixer_replay", proj.data_ptr(), ld, cs.data_ptr(), 4, cw.data_ptr(), rec.data_ptr(),
                  al.data_ptr(), dt.data_ptr(), nw.data_ptr(), 1e-6, out.data_ptr(), B, W, T, H, HV, K, K, None,
                  status.data_ptr(), s)

    ms = _time(run, reps)
    R = B * W * T
    return ms, "hbm", R * ld * 2 + R * HV * K * 2 + B * HV * K * K * 2 + B * C * 4 * 2


def case_mixer_cont(gen, reps, saved=False):
    """kadllm_gdn_mixer_continue at the second decode step of the benchmark: 32 requests x 256
    beams continuing from 256 parents (random parent indices); ``saved``: from the first
    step's records (the new tokens only), else replaying the parents' tokens too."""
    dev, bf = torch.device("cuda"), torch.bfloat16
    B, W, Wp, H, HV, K = 32, 256, 256, 16, 16, 128
    C = 2 * H * K + HV * K
    ld = C + HV * K + 2 * HV
    prev = (0.5 * torch.randn(B * Wp, ld, device=dev, generator=gen)).to(bf)
    proj = (0.5 * torch.randn(B * W, ld, device=dev, generator=gen)).to(bf)
    parent = torch.randint(0, Wp, (B, W), device=dev, generator=gen, dtype=torch.int32)
    cs = torch.randn(B, C, 4, device=dev, generator=gen).to(bf)
    cw = (0.3 * torch.randn(C, 4, device=dev, generator=gen)).to(bf)
    rec = (0.1 * torch.randn(B, HV, K, K, device=dev, generator=gen)).to(bf)
    al = torch.rand(HV, device=dev, generator=gen) * 2
    dt = torch.rand(HV, device=dev, generator=gen)
    nw = torch.ones(K, device=dev)
    out = torch.empty(B * W, HV * K, device=dev, dtype=bf)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    s = _lib.stream(dev)
    records = None
    if saved:  # the first step over the parents, writing their records
        records = torch.empty(_lib.lib().kadllm_gdn_mixer_record_bytes(B, Wp, HV, K), dtype=torch.uint8, device=dev)
        out1 = torch.empty(B * Wp, HV * K, device=dev, dtype=bf)
        _lib.call("kadllm_gdn_mixer_replay", prev.data_ptr(), ld, cs.data_ptr(), 4, cw.data_ptr(), rec.data_ptr(),
                  al.data_ptr(), dt.data_ptr(), nw.data_ptr(), 1e-6, out1.data_ptr(), B, Wp, 1, H, HV, K, K,
                  records.data_ptr(), status.data_ptr(), s)

    def run():
        _lib.call("kadllm_gdn_mixer_continue", prev.data_ptr(), parent.data_ptr(), Wp, proj.data_ptr(), ld,
                  cs.data_ptr(), 4, cw.data_ptr(), rec.data_ptr(), al.data_ptr(), dt.data_ptr(), nw.data_ptr(),
                  1e-6, out.data_ptr(), B, W, H, HV, K, K, _lib.ptr(records), status.data_ptr(), s)

    ms = _time(run, reps)
    R = B * W
    if saved:  # the new rows, the parents' q | k | v columns, gate a and records, the output, state and taps
        nbytes = R * ld * 2 + R * (C * 2 + HV * 2 + HV * 4 * K) + R * HV * K * 2 + B * HV * K * K * 2 + B * C * 8
        return ms, "hbm", nbytes
    return ms, "hbm", 2 * R * ld * 2 + R * HV * K * 2 + B * HV * K * K * 2 + B * C * 4 * 2


def case_replay(gen, reps, T=2):
    """ops.gated_delta (the reference's beam replay op) at the decode shape: 32 requests x
    256 beams, 16 heads of 128, BF16 q / k / v, fp32 gates and state."""
    from . import ops

    dev, bf = torch.device("cuda"), torch.bfloat16
    B, W, H, HV, K = 32, 256, 16, 16, 128
    BW = B * W
    q = torch.randn(BW, T, H, K, device=dev, generator=gen).to(bf)
    k = torch.randn(BW, T, H, K, device=dev, generator=gen).to(bf)
    v = torch.randn(BW, T, HV, K, device=dev, generator=gen).to(bf)
    g = -torch.rand(BW, T, HV, device=dev, generator=gen)
    beta = torch.rand(BW, T, HV, device=dev, generator=gen)
    s0 = 0.1 * torch.randn(B, HV, K, K, device=dev, generator=gen)
    ms = _time(lambda: ops.gated_delta(q, k, v, g, beta, s0, beam_width=W), reps)
    ops.check(dev)
    return ms, "hbm", BW * T * (2 * H + 2 * HV) * K * 2 + BW * T * HV * 4 * 2 + B * HV * K * K * 4


def case_qk_rope(gen, reps):
    """kadllm_qk_norm_rope at the prefill shape: 32 x 1024 rows of the attention projection
    (8 q heads with their gates, 2 k, 2 v heads of 256), rotary dims 64."""
    dev, bf = torch.device("cuda"), torch.bfloat16
    rows, L, Hq, HK, D, rot = 32 * 1024, 1024, 8, 2, 256, 64
    ld = Hq * 2 * D + 2 * HK * D
    P = torch.randn(rows, ld, device=dev, generator=gen).to(bf)
    qw = 0.1 * torch.randn(D, device=dev, generator=gen)
    kw = 0.1 * torch.randn(D, device=dev, generator=gen)
    t = torch.arange(L + 1, device=dev, dtype=torch.float32)[:, None] * (1e-4 ** (torch.arange(rot // 2, device=dev) / (rot // 2)))[None]
    cos = torch.cat([t.cos(), t.cos()], 1).to(bf).contiguous()
    sin = torch.cat([t.sin(), t.sin()], 1).to(bf).contiguous()
    q = torch.empty(rows, Hq * D, device=dev, dtype=bf)
    k = torch.empty(rows // L, L, HK, D, device=dev, dtype=bf)
    v = torch.empty_like(k)
    s = _lib.stream(dev)

    def run():
        _lib.call("kadllm_qk_norm_rope", P.data_ptr(), ld, Hq, HK, D, qw.data_ptr(), kw.data_ptr(), 1e-6,
                  cos.data_ptr(), sin.data_ptr(), rot, None, 0, L, q.data_ptr(), Hq * D, D, k.data_ptr(),
                  L * HK * D, HK * D, D, v.data_ptr(), L * HK * D, HK * D, D, rows, s)

    ms = _time(run, reps)
    return ms, "hbm", rows * (Hq + 2 * HK) * D * 2 * 2


def case_rmsnorm(gen, reps, rows=32 * 1024):
    """kadllm_add_rmsnorm as the step calls it after each fused residual update: read the
    hidden rows (1024 BF16), write their RMSNorm (1 + w); graph-timed (short launches)."""
    dev, bf, H = torch.device("cuda"), torch.bfloat16, 1024
    x = torch.randn(rows, H, device=dev, generator=gen).to(bf)
    w = 0.1 * torch.randn(H, device=dev, generator=gen)
    normed = torch.empty_like(x)

    def run():
        _lib.call("kadllm_add_rmsnorm", x.data_ptr(), None, 0, w.data_ptr(), 1e-6, normed.data_ptr(), rows, 1, 0, H,
                  _lib.stream(dev))

    ms = _time_graph(run, reps)
    return ms, "hbm", rows * H * 2 * 2


def case_select(gen, reps):
    from .grbeam import BeamSelector

    dev = torch.device("cuda")
    B, Wp, V, W = 32, 256, 248320, 256
    logits = (0.5 * torch.randn(B, Wp, V, device=dev, generator=gen)).to(torch.bfloat16)
    parent = -torch.rand(B, Wp, device=dev, generator=gen) * 4
    hist = torch.zeros(B, Wp, 1, dtype=torch.int64, device=dev)
    sel = BeamSelector(B, Wp, dev)
    ms = _time(lambda: sel.step(logits, parent, hist, W), reps)
    return ms, "hbm", B * Wp * V * 2


def case_gemm(gen, reps, M, N, K, epilogue=0):
    """kadllm_gemm at one of the step's projection shapes; the same product through
    torch.nn.functional.linear (cuBLAS) is timed beside it (plain product only)."""
    dev, bf = torch.device("cuda"), torch.bfloat16
    a = torch.randn(M, K, device=dev, generator=gen).to(bf)
    b = (0.05 * torch.randn(N, K, device=dev, generator=gen)).to(bf)
    n_out = N // 2 if epilogue == 1 else N
    out = torch.empty(M, n_out, device=dev, dtype=bf)
    resid = torch.randn(M, N, device=dev, generator=gen).to(bf) if epilogue == 2 else None
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def run():
        _lib.call("kadllm_gemm", a.data_ptr(), K, b.data_ptr(), K, out.data_ptr(), n_out, _lib.ptr(resid),
                  N if resid is not None else 0, M, N, K, n_out, epilogue, status.data_ptr(), _lib.stream(dev))

    ms = _time_graph(run, reps)
    if int(status.item()):
        raise RuntimeError("gemm reported a timed-out wait")
    ref = torch.empty(M, N, device=dev, dtype=bf)
    ref_ms = _time_graph(lambda: torch.nn.functional.linear(a, b, out=ref), reps)
    return ms, "tensor", 2.0 * M * N * K, {"shape": [M, N, K], "epilogue": epilogue, "cublas_ms": ref_ms,
                                            "cublas_tflops": 2.0 * M * N * K / (ref_ms / 1e3) / 1e12,
                                            "timing": "one CUDA graph of reps calls"}


CASES = {"prefill": case_prefill, "prefill8": lambda g, r: case_prefill(g, r, B=8), "attn_tiled": case_attn_tiled, "attn_split": case_attn_split, "conv": case_conv, "attn": case_attn, "mixer": case_mixer,
         "mixer2": lambda g, r: case_mixer(g, r, T=2), "select": case_select, "replay": case_replay,
         "mixer_cont": case_mixer_cont, "mixer_cont_saved": lambda g, r: case_mixer_cont(g, r, saved=True),
         "qk_rope": case_qk_rope,
         "rmsnorm": case_rmsnorm, "rmsnorm_decode": lambda g, r: case_rmsnorm(g, r, rows=8192),
         "attn_step": lambda g, r: case_attn_tiled(g, r, B=32, W=256, T=2, L=1024),
         "attn_causal": lambda g, r: case_attn_tiled(g, r, B=32, W=1, T=1, L=1024, causal=True),
         # the step's projections: prefill (32 x 1024 rows) and decode (32 x 256 beams, T = 1)
         "gemm_gdn_in": lambda g, r: case_gemm(g, r, 32768, 8224, 1024),
         "gemm_mlp_gu": lambda g, r: case_gemm(g, r, 32768, 7168, 1024, epilogue=1),
         "gemm_mlp_down": lambda g, r: case_gemm(g, r, 32768, 1024, 3584, epilogue=2),
         "gemm_out": lambda g, r: case_gemm(g, r, 8192, 1024, 2048, epilogue=2),
         "gemm_prefill_out": lambda g, r: case_gemm(g, r, 32768, 1024, 2048, epilogue=2),
         "gemm_decode_gu": lambda g, r: case_gemm(g, r, 8192, 7168, 1024, epilogue=1),
         "gemm_decode_down": lambda g, r: case_gemm(g, r, 8192, 1024, 3584, epilogue=2),
         "gemm_decode_in": lambda g, r: case_gemm(g, r, 8192, 8224, 1024),
         "gemm_lm_head": lambda g, r: case_gemm(g, r, 8192, 248320, 1024)}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--case", nargs="+", choices=sorted(CASES), required=True)
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    for case in args.case:
        gen = torch.Generator(device="cuda").manual_seed(0)
        res = CASES[case](gen, args.reps)
        ms, bound, work = res[:3]
        hbm, tflops, kind = _peaks()
        if bound == "tensor":
            achieved, peak, unit = work / (ms / 1e3) / 1e12, tflops, "TFLOP/s"
        else:
            achieved, peak, unit = work / (ms / 1e3) / 1e9, hbm, "GB/s"
        line = {"case": case, "ms": ms, "bound": bound, "work": work, "achieved": achieved,
                "unit": unit, "peak": peak, "frac": achieved / peak, "peak_kind": kind}
        if len(res) > 3:
            line.update(res[3])
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
