"""GRBeam benchmark: requests/s on the Qwen3.5-0.8B-shaped hybrid (B200).

Workload (per GPU): random-init BF16 weights N(0, 0.02)
(seed 0), 32 requests of 1024 uniform-random prompt tokens per GPU, beam width
256, 3 output tokens (prefill + 2 decode steps + selection), full 248,320-token
vocabulary.  One step = one ``grbeam_search`` over one 32-request batch per
GPU -- by default the whole search captured once as a CUDA graph
(``kadllm_b200.grbeam.GraphedSearch``) and replayed each step, every kernel
of the search running each time (``--no-graph``: eager launches); with N GPUs
every rank runs its own batch (weak scaling: requests shard across GPUs with
replicated weights) with no collective inside the timed steps; the results are
all-gathered over NCCL once afterwards (``per_rank.with_gather_ms`` reports what
a per-step gather would cost).

``value``   requests/s with the prompts already resident in HBM;
``e2e``     the same through the public API from pinned host buffers, with the
            prompt upload and the token / score download inside the timed region.
Timing: CUDA events on the launching stream between barriers, max over ranks.
The working set (1.5 GB of weights, GBs of activations / logits) exceeds the
126 MB L2, so no explicit flush is needed between steps.

``--impl reference`` times the reference algorithm's CPU restatement (the
numpy oracle port of Kadllm's torch path) on all host cores, one whole request
per step (as many steps as fit a bounded CPU budget, reported as run); rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import tempfile
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, PROMPT, BEAM, DEPTH = 32, 1024, 256, 3
METRIC = "requests/s (Qwen3.5-0.8B, bs32, prefix 1024, beam 256, 3 tokens) at 1/2/4/8 B200"
WORKLOAD = "qwen3.5-0.8b-shaped hybrid, bf16 random N(0,0.02) seed 0, B=32/GPU, prefix 1024, beam 256, depth 3"


def algorithmic_flops(cfg, B=BATCH, L=PROMPT, W=BEAM, depth=DEPTH) -> float:
    """Dense FLOPs of the work one GRBeam call needs: linears 2 * params * rows,
    attention QK^T + PV, GDN state products, the LM head.  Needed work only: the
    last layer's output projection and MLP run on each request's last prompt
    position (the logits read nothing else), and each decode step replays its new
    token only (the earlier suffix tokens' per-layer work is the parent step's)."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    hq, d = cfg.num_attention_heads, cfg.head_dim
    hv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
    n = cfg.num_layers
    dec_rows = B * W * (depth - 1)  # one new token per beam per decode step
    flops = 0.0
    for i, kind in enumerate(cfg.layer_types):
        gdn = kind == "linear_attention"
        w_in = (cfg.gdn_in_dim if gdn else cfg.attn_in_dim) * H
        w_post = H * (cfg.value_dim if gdn else hq * d) + 3 * H * I
        tail_rows = B if i == n - 1 else B * L
        flops += 2 * w_in * B * L + 2 * w_post * tail_rows  # prefill
        flops += 2 * (w_in + w_post) * dec_rows              # decode
        if gdn:
            flops += B * hv * L * (6 * dk * dv + 4 * 64 * (dk + dv))  # chunked scan
            flops += dec_rows * hv * 2 * 2 * dk * dv                  # [q; k] x S0 per new token
        else:
            queries = B if i == n - 1 else None
            flops += 4 * B * hq * d * L * (L + 1) / 2 if queries is None else 4 * B * hq * d * L
            flops += sum(4 * B * W * hq * d * (L + t) for t in range(1, depth))  # one query row per beam
    flops += 2 * H * cfg.vocab_size * (B + dec_rows)
    return float(flops)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"kadllm_b200_clocks_gpu{gpu}_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.out.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        mhz, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        text = self.path.read_text()
        self.path.unlink(missing_ok=True)
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(mhz)}


def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------
# CPU legs (oracle port of the reference's torch path)
# ---------------------------------------------------------------------------
def host_threads() -> int:
    """Use every host core for the CPU legs, whatever OMP_NUM_THREADS the launcher
    set (torch.distributed.run sets 1): numpy's BLAS pool and torch's intra-op pool."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except ImportError:  # pragma: no cover - threadpoolctl is in the image
        pass
    import torch

    torch.set_num_threads(n)
    return n


def cpu_reference_request(weights_np, cfg, seed: int, prompt=PROMPT, n_layers=None) -> float:
    """Seconds for one whole request through the oracle (fp32): prefill of a
    ``prompt``-token prompt, two decode steps of ``BEAM`` beams and three
    selections over the full vocabulary, through all ``n_layers`` layers (default:
    the model's depth)."""
    import dataclasses

    from kadllm_b200.synthetic import random_prompts
    from oracle import grbeam_oracle as O

    n = cfg.num_layers if n_layers is None else n_layers
    sub = dataclasses.replace(cfg, layer_types=tuple(cfg.layer_types[:n]))
    ids = random_prompts(1, prompt, cfg.vocab_size, seed=seed)
    orc = O.HybridOracle(sub, weights_np, "fp32")
    t0 = time.perf_counter()
    O.grbeam_search(orc, ids, [BEAM] * DEPTH)
    return time.perf_counter() - t0


def numpy_weights_from(model_weights):
    """fp32 numpy copies of the benchmark weights (the oracle's input)."""
    return {k: v.float().cpu().numpy() for k, v in model_weights.items()}


CPU_BUDGET_S = 150.0  # the reference arm's timed samples stop once this much CPU time is spent


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the oracle port on the host cores, rank 0 only.  Each step
    is one whole request (24 layers, prefix 1024, beam 256, 3 tokens); the arm
    runs the requested steps or as many as fit ``CPU_BUDGET_S`` (at least one),
    and reports the steps it ran."""
    if rank != 0:
        return
    from kadllm_b200.config import QWEN35_08B
    from kadllm_b200.synthetic import numpy_weights

    cfg = QWEN35_08B
    threads = host_threads()
    weights = numpy_weights(cfg, seed=0, init="spec")
    warm = 0
    if args.warmup:  # one short warm-up: the embedding, final norm, LM head and selections only
        cpu_reference_request(weights, cfg, seed=999, n_layers=0)
        warm = 1
    times = []
    t_start = time.perf_counter()
    for i in range(max(1, args.steps)):
        times.append(cpu_reference_request(weights, cfg, seed=i))
        if time.perf_counter() - t_start + statistics.mean(times) > CPU_BUDGET_S:
            break
    per_req = statistics.mean(times)
    value = 1.0 / per_req
    sample = (f"{len(times)} whole request(s) (24 layers, prefix {PROMPT}, beam {BEAM}, {DEPTH} tokens, full "
              f"vocabulary) through the numpy oracle port (fp32), one per step, {threads} host threads; "
              f"{per_req:.1f} s per request (min {min(times):.1f}, max {max(times):.1f})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "requests/s", "n_gpus": world,
        "steps": len(times), "steps_requested": args.steps, "warmup": warm, "ms_per_step": per_req * 1000,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD + " (CPU: 1 request per step)", "global_batch": 1,
                   "seq_len": PROMPT, "beam": BEAM, "depth": DEPTH, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "requests/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "requests/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host_threads": threads,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------
def run_native(args, rank: int, world: int, local_rank: int) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from kadllm_b200 import _lib, grbeam_search
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.config import QWEN35_08B
    from kadllm_b200.grbeam import GraphedSearch
    from kadllm_b200.model import HybridModel
    from kadllm_b200.shard import all_ranks, gather_beams, max_over_ranks, rank_prompts
    from kadllm_b200.synthetic import torch_weights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = QWEN35_08B
    weights = torch_weights(cfg, seed=0, device=dev)
    engine = HybridModel(cfg, weights, device=dev)
    adapter = NativeGRBeamAdapter(engine)
    # per-GPU batch: 32 requests (weak scaling), or a fixed total split over the ranks (strong)
    if args.total_requests:
        if args.total_requests % world:
            raise SystemExit("--total-requests must divide evenly over the ranks")
        batch = args.total_requests // world
    else:
        batch = args.batch
    ids_host = torch.from_numpy(rank_prompts(rank, batch, PROMPT, cfg.vocab_size)).pin_memory()
    ids_dev = ids_host.to(dev)
    tok_host = torch.empty(batch, BEAM, DEPTH, dtype=torch.int64).pin_memory()
    sc_host = torch.empty(batch, BEAM, dtype=torch.float32).pin_memory()
    widths = [BEAM] * DEPTH

    def gather(res):  # the finished beams of every rank, in rank order (after the timed searches)
        return gather_beams(res.tokens, res.scores)

    # the search as one CUDA graph (static prompt buffer, every kernel replayed per step);
    # the eager path when capture is off or fails
    graphed = None
    launches_per_step = None
    with torch.inference_mode():
        n0 = _lib.launch_count
        grbeam_search(adapter, ids_dev, widths)  # eager reference search: this library's launches per step
        launches_per_step = _lib.launch_count - n0
        if not args.no_graph:
            try:
                graphed = GraphedSearch(adapter, batch, PROMPT, widths, dev)
            except Exception as exc:  # noqa: BLE001 - report and fall back to eager launches
                print(f"bench: CUDA graph capture failed ({type(exc).__name__}: {exc}); eager launches",
                      file=sys.stderr, flush=True)
                graphed = None

    # a step is one search of this rank's requests; the requests are independent, so no
    # collective runs between the barriers (each rank keeps its own beams)
    def step_device():
        return graphed(ids_dev) if graphed is not None else grbeam_search(adapter, ids_dev, widths)

    def step_e2e():
        ids = ids_host.to(dev, non_blocking=True)
        res = graphed(ids) if graphed is not None else grbeam_search(adapter, ids, widths)
        tok_host.copy_(res.tokens, non_blocking=True)
        sc_host.copy_(res.scores, non_blocking=True)
        return res

    per_rank = {}

    def timed(fn, steps, key=None):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches0 = _lib.launch_count
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        mine = start.elapsed_time(end)
        if key:
            per_rank[key] = [round(v / steps, 3) for v in all_ranks(mine, dev)]
        ms = max_over_ranks(mine, dev)
        return ms / steps, (launches_per_step * steps if graphed is not None else _lib.launch_count - launches0)

    def step_gather():  # the search plus the all-gather of every rank's beams (reported per rank)
        return gather(step_device())

    with torch.inference_mode():
        for _ in range(args.warmup):
            step_device()
        with ClockSampler(local_rank) as clocks:
            ms, launches = timed(step_device, args.steps, "step_ms")
        ms_e2e, _ = timed(step_e2e, args.steps)
        if world > 1:  # what a per-search gather of every rank's beams would add
            timed(step_gather, args.steps, "with_gather_ms")
        res = graphed(ids_dev) if graphed is not None else grbeam_search(adapter, ids_dev, widths)
        gather(res)  # the combined result (every rank takes part)
        if graphed is not None:
            graphed.check()
        valid = bool(res.valid.all().item())
        distinct = all(len({tuple(b) for b in req}) == BEAM for req in res.tokens.cpu().tolist())
        prof = profile_kernels(engine, adapter, ids_dev, widths, args) if rank == 0 else None

    if rank != 0:
        return
    flops = algorithmic_flops(cfg, B=batch)
    peaks, peak_kind = measured_peaks()
    value = world * batch / (ms / 1000)
    line = {
        "metric": METRIC, "value": value, "unit": "requests/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if args.total_requests else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random prompts, random-init weights)",
        "per_rank": per_rank,
        "config": {"workload": WORKLOAD if batch == 32 else WORKLOAD.replace("B=32/GPU", f"B={batch}/GPU"),
                   "model": "qwen3.5-0.8b-shaped", "global_batch": world * batch,
                   "seq_len": PROMPT, "beam": BEAM, "depth": DEPTH, "parallelism": f"dp{world} (request shards)",
                   "l2": "working set > 126 MB L2 (weights 1.5 GB, logits 4 GB per step); no flush"},
        "e2e": {"value": world * batch / (ms_e2e / 1000), "unit": "requests/s",
                "h2d_bytes_per_step": batch * PROMPT * 8, "d2h_bytes_per_step": batch * BEAM * (DEPTH * 8 + 4)},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "path_roofline": {"bound": "tensor", "algorithmic_tflop_per_step": flops / 1e12,
                          "achieved": flops / (ms / 1000) / 1e12,
                          "peak": peaks.get("bf16_tflops_sustained"), "unit": "TFLOP/s",
                          "frac": flops / (ms / 1000) / 1e12 / peaks.get("bf16_tflops_sustained"),
                          "peak_kind": f"{peak_kind} sustained bf16"},
        "checks": {"all_valid": valid, "distinct_beams": distinct},
        "launch": "cuda_graph" if graphed is not None else "eager",
    }
    if prof:
        line["roofline"] = prof["roofline"]
        line["kernel_ms"] = prof["kernel_ms"]
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(weights, cfg)
    print(json.dumps(line), flush=True)


SID_WIDTHS = (256, 256)
SID_LEVEL = 4096     # tokens per codebook level
SID_GROUPS = 256     # level-1 groups (16 level-2 tokens each)
SID_PREFIX = (512, 4096)


def run_sid(args, rank: int, world: int, local_rank: int) -> None:
    """Two-level conditional SID search: prefix lengths drawn
    uniformly from 512-4096 per request, SID-only head over 2 x 4096 codebook
    tokens, token 2 restricted to token 1's group, widths 256, 256."""
    import numpy as np
    import torch

    from kadllm_b200 import _lib
    from kadllm_b200.adapters import NativeGRBeamAdapter
    from kadllm_b200.config import QWEN35_08B
    from kadllm_b200.model import HybridModel
    from kadllm_b200.shard import max_over_ranks
    from kadllm_b200.sid import SidCodebook, SidHeadAdapter, sid_search
    from kadllm_b200.synthetic import torch_weights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = QWEN35_08B
    engine = HybridModel(cfg, torch_weights(cfg, seed=0, device=dev), device=dev)
    adapter = NativeGRBeamAdapter(engine)
    cb = SidCodebook.synthetic(cfg.vocab_size, SID_LEVEL, SID_LEVEL, SID_GROUPS, seed=0)
    head = SidHeadAdapter(adapter, cb)
    rng = np.random.default_rng(1000 + rank)
    lengths = rng.integers(SID_PREFIX[0], SID_PREFIX[1] + 1, args.sid_batch)
    host = [torch.from_numpy(rng.integers(0, cfg.vocab_size, int(n))).pin_memory() for n in lengths]
    dev_prompts = [p.to(dev) for p in host]
    tok_host = torch.empty(args.sid_batch, SID_WIDTHS[-1], 2, dtype=torch.int64).pin_memory()

    def step_device():
        return sid_search(adapter, dev_prompts, cb, SID_WIDTHS, head=head, streams=args.sid_streams)

    def step_e2e():
        res = sid_search(adapter, [p.to(dev, non_blocking=True) for p in host], cb, SID_WIDTHS, head=head,
                         streams=args.sid_streams)
        tok_host.copy_(res.tokens, non_blocking=True)
        return res

    def timed(fn, steps):
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches0 = _lib.launch_count
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return max_over_ranks(start.elapsed_time(end), dev) / steps, _lib.launch_count - launches0

    with torch.inference_mode():
        for _ in range(args.warmup):
            step_device()
        ms, launches = timed(step_device, args.steps)
        ms_e2e, _ = timed(step_e2e, args.steps)
        res = step_device()
        valid = bool(res.valid.all().item())
    if rank != 0:
        return
    line = {
        "metric": "requests/s (two-level conditional SID, Qwen3.5-0.8B, prefix 512-4096, beam 256)",
        "value": world * args.sid_batch / (ms / 1000), "unit": "requests/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random prompts and lengths, random-init weights, seeded codebooks)",
        "config": {"workload": "sid", "model": "qwen3.5-0.8b-shaped", "batch_per_gpu": args.sid_batch,
                   "prefix_lengths": [int(lengths.min()), int(lengths.max())], "widths": list(SID_WIDTHS),
                   "codebook": f"2 x {SID_LEVEL} tokens, {SID_GROUPS} groups", "head": "SID-only",
                   "streams": args.sid_streams},
        "e2e": {"value": world * args.sid_batch / (ms_e2e / 1000), "unit": "requests/s",
                "h2d_bytes_per_step": int(lengths.sum()) * 8, "d2h_bytes_per_step": args.sid_batch * SID_WIDTHS[-1] * 16},
        "gpu_launches": launches,
        "checks": {"all_valid": valid},
    }
    print(json.dumps(line), flush=True)


def hf_model(cfg, weights, device):
    """A Transformers ``Qwen3_5ForConditionalGeneration`` holding the benchmark's weights
    (BF16; a one-block stand-in vision tower, which GRBeam never runs) -- what the
    reference's runner loads with ``from_pretrained``."""
    import torch
    from transformers import Qwen3_5Config, Qwen3_5ForConditionalGeneration

    vision = dict(depth=1, hidden_size=64, intermediate_size=128, num_heads=2, out_hidden_size=cfg.hidden_size)
    hf_cfg = Qwen3_5Config(text_config=cfg.to_hf_kwargs(), vision_config=vision,
                           tie_word_embeddings=cfg.tie_word_embeddings)
    with torch.device("meta"):
        model = Qwen3_5ForConditionalGeneration(hf_cfg)
    model = model.to_empty(device=device).to(torch.bfloat16)
    text = model.model.language_model
    text.load_state_dict({k: v.to(torch.bfloat16) for k, v in weights.items() if k != "lm_head.weight"},
                         strict=False)
    if cfg.tie_word_embeddings:
        model.lm_head.weight = text.embed_tokens.weight
    return model.eval()


def run_dropin(args, rank: int, world: int, local_rank: int) -> None:
    """The reference runner's external-backend path, unchanged: ``benchmarks/grbeam.py
    --backend external --adapter-factory kadllm_b200.factory:make`` loads the model, calls
    the factory and times ``search(adapter, ids, [beam] * depth).tokens.tolist()`` by wall
    clock, eager launches, with its deterministic prompts ``10 + (i + 17 r) % 100``
    (benchmarks/grbeam.py:219-223,254-257,299,325-346)."""
    import torch

    from kadllm_b200 import _lib
    from kadllm_b200.config import QWEN35_08B
    from kadllm_b200.factory import make
    from kadllm_b200.synthetic import torch_weights

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = QWEN35_08B
    model = hf_model(cfg, torch_weights(cfg, seed=0, device=dev), dev)
    adapter, search = make(model)
    ids = torch.tensor([[10 + (i + r * 17) % 100 for i in range(PROMPT)] for r in range(BATCH)], device=dev)
    widths = [BEAM] * DEPTH

    def run():
        return search(adapter, ids, widths).tokens.tolist()

    with torch.inference_mode():
        for _ in range(args.warmup):
            tokens = run()
        times = []
        n0 = _lib.launch_count
        for _ in range(args.steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            tokens = run()
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
        launches = (_lib.launch_count - n0) // max(args.steps, 1)
    distinct = all(len({tuple(b) for b in req}) == BEAM for req in tokens)
    if rank != 0:
        return
    mean = statistics.mean(times)
    line = {
        "metric": METRIC + " -- drop-in runner path (eager, wall clock)", "value": world * BATCH / mean,
        "unit": "requests/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": mean * 1000, "median_ms": statistics.median(times) * 1000, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic weights; the reference runner's deterministic prompts",
        "config": {"workload": "dropin: factory.make(Qwen3_5ForConditionalGeneration) + search(...).tokens.tolist()",
                   "model": "qwen3.5-0.8b-shaped", "global_batch": world * BATCH, "seq_len": PROMPT,
                   "beam": BEAM, "depth": DEPTH},
        "library_launches_per_search": launches,
        "checks": {"distinct_beams": distinct},
    }
    print(json.dumps(line), flush=True)


def profile_kernels(engine, adapter, ids_dev, widths, args):
    """Per-entry-point device time over one extra search, CUDA events on the
    launching stream; the dominant kernel's roofline is derived from it."""
    import torch

    from kadllm_b200 import _lib, grbeam_search
    from kadllm_b200.roofline import KernelTimer, roofline_for

    timer = KernelTimer()
    with timer.install():
        grbeam_search(adapter, ids_dev, widths)
    torch.cuda.synchronize()
    totals = timer.totals()
    peaks, kind = measured_peaks()
    roof = roofline_for(args.roofline_kernel or max(totals, key=lambda k: totals[k][0]), timer, engine.cfg,
                        peaks, kind)
    return {"roofline": roof, "kernel_ms": {k: round(v[0], 3) for k, v in sorted(totals.items())}}


def cpu_baseline(weights, cfg) -> dict:
    """The oracle port on the host cores: one whole request (fp32, the benchmark's weights)."""
    threads = host_threads()
    dt = cpu_reference_request(numpy_weights_from(weights), cfg, seed=123)
    return {"value": 1.0 / dt, "unit": "requests/s", "cores": threads, "kind": "port",
            "sample": f"1 whole request (24 layers, prefix {PROMPT}, beam {BEAM}, {DEPTH} tokens, full vocabulary) "
                      f"through the numpy oracle port (fp32): {dt:.1f} s on {threads} host threads"}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--roofline-kernel", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="eager launches instead of one CUDA graph per search")
    ap.add_argument("--workload", choices=["grbeam", "sid", "dropin"], default="grbeam",
                    help="grbeam: the headline metric; sid: two-level conditional SID, prefixes 512-4096; "
                         "dropin: the reference runner's external-backend call, eager, wall clock")
    ap.add_argument("--sid-batch", type=int, default=32)
    ap.add_argument("--batch", type=int, default=BATCH, help="requests per GPU (weak scaling)")
    ap.add_argument("--total-requests", type=int, default=0,
                    help="a fixed number of requests split over the GPUs (strong scaling, e.g. 256)")
    ap.add_argument("--sid-streams", type=int, default=1)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist

    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        {"sid": run_sid, "dropin": run_dropin}.get(args.workload, run_native)(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
