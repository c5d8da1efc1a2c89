"""Per-kernel timing and roofline accounting for the benchmark.

``KernelTimer`` brackets every C-ABI call with CUDA events on the launching
(current) stream; ``work_of`` gives the algorithmic work of one call from its
size arguments -- FLOPs for the tensor-core kernels, compulsory HBM bytes for
the streaming ones -- so achieved = work / event time can be compared with the
measured B200 peaks.
"""

from __future__ import annotations

import contextlib

import torch

from . import _lib


def work_of(name: str, args: tuple) -> tuple[str, float] | None:
    """(bound, algorithmic work) of one call: ("tensor", FLOPs) or ("hbm", bytes)."""
    if name == "kadllm_gdn_prefill_split":
        # compulsory HBM bytes (the binding roof: 86 GFLOP of tensor work take a
        # third of the time the bytes do): projection columns read once, output,
        # both prefix states
        B, L, H, HV, DK, DV = args[13:19]
        conv_dim = 2 * H * DK + HV * DV
        rows = B * L
        read = rows * (conv_dim + HV * DV + 2 * HV) * 2
        write = rows * HV * DV * 2 + B * HV * DK * DV * 2 + B * conv_dim * 4 * 2
        return "hbm", float(read + write)
    if name == "kadllm_attention_tiled":
        B, W, T, t0, H, HK, L, D = args[24:32]
        if args[33]:  # causal prefill
            return "tensor", float(4 * B * H * D * L * (L + 1) / 2)
        # query rows of steps t0 .. T-1, each against the prefix and its suffix keys s <= t
        return "tensor", float(sum(4 * B * W * H * D * (L + t + 1) for t in range(t0, T)))
    if name == "kadllm_causal_attention":
        B, L, H, HK, D = args[17:22]
        return "tensor", float(4 * B * H * D * L * (L + 1) / 2)
    if name == "kadllm_prefix_attention":
        B, W, T, H, HK, L, D = args[30:37]
        return "tensor", float(4 * B * W * T * H * D * L + 4 * B * W * H * D * T * (T + 1) / 2)
    if name == "kadllm_gemm":
        M, N, K = args[8:11]
        return "tensor", float(2 * M * N * K)
    if name == "kadllm_gdn_mixer_replay":
        B, W, T, H, HV, DK, DV = args[11:18]
        R = B * W * T
        conv_dim = 2 * H * DK + HV * DV
        read = R * (conv_dim + HV * DV + 2 * HV) * 2 + B * HV * DK * DV * 2 + B * conv_dim * 4 * 2
        records = R * HV * DV * 4 if args[18] is not None else 0  # the first step's deltas, fp32
        return "hbm", float(read + R * HV * DV * 2 + records)
    if name == "kadllm_gdn_mixer_continue":
        # the new rows (q | k | v | z | b | a columns), the request's state and conv taps, the
        # new rows' output, and either the parents' previous-step rows or, from records, the
        # parents' q | k | v | a columns and deltas
        B, W, H, HV, DK, DV = args[14:20]
        R = B * W
        conv_dim = 2 * H * DK + HV * DV
        new = R * (conv_dim + HV * DV + 2 * HV) * 2
        parents = R * (conv_dim + 2 * HV) * 2 + R * HV * DV * 4 if args[20] is not None else new
        read = new + parents + B * HV * DK * DV * 2 + B * conv_dim * 4 * 2
        return "hbm", float(read + R * HV * DV * 2)
    if name == "kadllm_beam_select":
        B, Wp, V, W, depth = args[11:16]
        esz = 4 if args[1] == 0 else 2
        return "hbm", float(B * Wp * V * esz)
    if name == "kadllm_silu_mul":
        inter, rows = args[2], args[4]
        return "hbm", float(rows * inter * 2 * 3)
    if name == "kadllm_add_rmsnorm":
        rows, H = args[6], args[9]
        return "hbm", float(rows * H * 2 * (4 if args[1] else 2))
    return None


def measured_traffic(name: str, args: tuple) -> float | None:
    """DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one call, from
    one ncu capture of the benchmark's shape of that call on a B200; None for
    shapes that were not captured."""
    if name == "kadllm_gdn_prefill_split" and tuple(args[13:19]) == (32, 1024, 16, 16, 128, 128):
        # captured at B = 8 (a quarter of the requests; traffic grows with them): tcgen05 prep
        # 101.8 + 97.3 MB, tcgen05 scan with the gated norm 185.5 + 16.4 MB; x 4
        return 1604.0e6
    if name == "kadllm_gdn_mixer_replay" and tuple(args[11:13]) == (32, 256) and tuple(args[14:18]) == (16, 16, 128, 128):
        if args[18] is not None:  # the first step writing its records: 168.0 + 66.1 MB
            return 234.1e6 if args[13] == 1 else None
        return {1: 181.0e6, 2: 353.6e6}.get(args[13])  # T = 1: 164.6 + 16.4 MB; T = 2: 306.0 + 47.6 MB
    if (name == "kadllm_gdn_mixer_continue" and args[2] == 256 and tuple(args[14:16]) == (32, 256)
            and tuple(args[16:20]) == (16, 16, 128, 128)):
        if args[20] is not None:  # from the first step's records: 300.7 + 26.6 MB
            return 327.3e6
        return 295.8e6  # 273.6 + 22.2 MB (random parents: children of one parent share its rows in L2)
    if name == "kadllm_attention_tiled" and (args[24], *args[28:32]) == (32, 8, 2, 1024, 256):
        if args[33]:  # causal prefill: 335.6 + 109.8 MB
            return 445.4e6
        return 285.4e6 if tuple(args[25:28]) == (256, 2, 0) else None  # decode T = 2: 235.0 + 50.4 MB
    if name == "kadllm_beam_select" and tuple(args[11:14]) == (32, 256, 248320):
        return 4100.4e6  # rowstats 4068.7 + 21.2 MB, collect 8.7 MB, threshold 1.3 MB, finalize 0.2 MB
    return None


class KernelTimer:
    def __init__(self):
        self.records: list[tuple[str, tuple, torch.cuda.Event, torch.cuda.Event]] = []

    @contextlib.contextmanager
    def install(self):
        original = _lib.call

        def timed_call(name, *args):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            original(name, *args)
            e.record()
            self.records.append((name, args, s, e))

        _lib.call = timed_call
        try:
            yield self
        finally:
            _lib.call = original

    def totals(self) -> dict[str, tuple[float, int]]:
        """name -> (total ms, calls); synchronise first."""
        out: dict[str, list] = {}
        for name, _, s, e in self.records:
            t = out.setdefault(name, [0.0, 0])
            t[0] += s.elapsed_time(e)
            t[1] += 1
        return {k: (v[0], v[1]) for k, v in out.items()}


def roofline_for(name: str, timer: KernelTimer, cfg, peaks: dict, peak_kind: str) -> dict:
    """Roofline of kernel `name` over the timed calls: achieved = work / duration."""
    work, ms, calls, bound = 0.0, 0.0, 0, None
    traffic: float | None = 0.0
    for n, args, s, e in timer.records:
        if n != name:
            continue
        w = work_of(n, args)
        if w is None:
            continue
        bound, amount = w
        work += amount
        ms += s.elapsed_time(e)
        calls += 1
        t = measured_traffic(n, args)
        traffic = None if traffic is None or t is None else traffic + t
    if not calls:
        return {"kernel": name, "bound": None, "achieved": None, "peak": None, "unit": None, "frac": None,
                "traffic": None}
    if bound == "tensor":  # timed inside a whole search (seconds of load): the sustained peak
        achieved = work / (ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        unit, per_launch = "TFLOP/s", work / calls / 1e12
    else:
        achieved = work / (ms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        unit, per_launch = "GB/s", work / calls
    return {"kernel": name, "bound": "tensor" if bound == "tensor" else "hbm", "achieved": achieved,
            "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": None if traffic is None else traffic / calls, "traffic_unit": "bytes per launch (ncu)",
            "launches": calls,
            "avg_launch_ms": ms / calls, "work_per_launch": per_launch,
            "peak_kind": f"{peak_kind} ({'bf16 sustained' if bound == 'tensor' else 'HBM copy'})"}
