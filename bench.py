"""Benchmark of the quantized matvec hot path (prints one JSON line on rank 0).

Workload (the headline metric): one decode step of a 32-layer stack of
Llama-3-8B-shaped projections at batch 1 — per layer q_proj/o_proj 4096x4096, k_proj/v_proj
1024x4096, gate/up 14336x4096 (Q4_K) and down 4096x14336 (Q6_K), 137,822,208 weight bytes per layer,
4.41 GB per step.  Per layer the step forms four inputs from the residual stream and the previous
outputs (RMS norm of h -> q/k/v, q's output -> o, RMS norm of h + o -> gate/up, SiLU(gate) * up -> down;
o_proj reads q_proj's output where attention would be) and runs the seven matvecs.  Default `--mode
calls`: the reference's call pattern (norm_q8 / Eingang / akt_q8 producers, then mmvq.mv_geteilt / mv)
with programmatic dependent launch, captured once in a CUDA graph as the reference's decoder does;
`--mode chain`: the same step as one persistent decode-chain launch.  Weights and activations are
seeded synthetic data with the config's distributions; every step reads 4.41 GB of distinct weights,
far more than L2 (126 MB), so no L2 flush is needed.  The batch-4 / batch-8 lines run the seven matvecs
per layer on fixed inputs (one Eingang per input).

value: weight GB/s of the whole job (all ranks; weak scaling: every GPU runs its own stack replica).
e2e: the same step with its first input copied from pinned host memory and its last output read back.
--impl reference: the reference's CPU path for the same workload on the host cores (a restatement in
oracle/: GGUF weights dequantised once to bf16, then torch F.linear, as the reference engine does on a
CPU device, ggufengine/models/common.py:516-527), one layer per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "weight GB/s and % of HBM peak for batch-1 quant matvec; decode tokens/s per layer stack"
LAYERS = 32
# (name, format, n_out, n_in, input slot)
LAYER = [("q", "Q4_K", 4096, 4096, 0), ("k", "Q4_K", 1024, 4096, 0), ("v", "Q4_K", 1024, 4096, 0),
         ("o", "Q4_K", 4096, 4096, 1), ("gate", "Q4_K", 14336, 4096, 2), ("up", "Q4_K", 14336, 4096, 2),
         ("down", "Q6_K", 4096, 14336, 3)]
INPUTS = [4096, 4096, 4096, 14336]          # activation widths of the four inputs of a layer
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_PEAKS["hbm_gbs"], "fallback"


class Clocks:
    """Samples nvidia-smi every 20 ms while running (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)                      # the sampler is running before the timed region starts
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def build_stack(device, seed0: int, n_layers: int = LAYERS):
    from nemicli_terminal_b200 import synth
    layers = []
    for l in range(n_layers):
        mats = []
        for j, (name, fmt, n_out, n_in, slot) in enumerate(LAYER):
            mats.append((name, fmt, n_out, n_in, slot, synth.blocks(fmt, n_out, n_in, seed=seed0 + 16 * l + j,
                                                                     device=device)))
        layers.append(mats)
    return layers


def layer_bytes() -> int:
    from nemicli_terminal_b200.formats import row_bytes
    return sum(n_out * row_bytes(fmt, n_in) for _, fmt, n_out, n_in, _ in LAYER)


def step_fn(stack, xs, batch):
    """The seven matvecs of each layer on fixed inputs through the public API (mmvq.mv_geteilt: one
    launch per group of matrices that shares an input, q/k/v, o, gate/up, down): returns the outputs
    (list).  Batches above 1 quantise once per input (Eingang)."""
    from nemicli_terminal_b200 import mmvq
    outs = []
    for l, mats in enumerate(stack):
        for slot in range(4):
            group = [m for m in mats if m[4] == slot]
            fmt, n_in = group[0][1], group[0][3]
            # one launch per group (q/k/v, gate/up share it); more tokens: one Eingang per input
            x = xs[l][slot] if batch == 1 else mmvq.Eingang(xs[l][slot])
            outs += mmvq.mv_geteilt(fmt, [(m[5], m[2]) for m in group], x, n_in)
    return outs


def build_chain(stack, device, seed: int = 0):
    """The stack as one decode chain: per layer RMSNORM -> q,k,v | o (reads q's output: attention
    stand-in) | RMSNORM(h + o) -> gate,up | SILU_MUL -> down, the residual stream carried across layers."""
    from nemicli_terminal_b200 import chain, synth
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h0 = synth.activations(1, 4096, seed=seed + 11, device=device)[0].contiguous()
    stages, h, r, outs = [], h0, None, []
    for i, mats in enumerate(stack):
        m = {name: (fmt, raw, n_out, n_in) for name, fmt, n_out, n_in, slot, raw in mats}
        wa = (torch.rand(4096, generator=g, device=device) + 0.5).contiguous()
        wf = (torch.rand(4096, generator=g, device=device) + 0.5).contiguous()
        st, h_mid, y_down = chain.layer_stages(m["q"], m["k"], m["v"], m["o"], m["gate"], m["up"], m["down"],
                                               h_in=h, resid_in=r, attn_norm=wa, ffn_norm=wf, first=i == 0)
        stages += st
        outs += [y for s_ in st for y in s_.ys]
        h, r = h_mid, y_down
    return chain.Chain(stages), h0, r, outs


def build_calls(stack, device, seed: int = 0):
    """The chain's step (same weights, norms and residual stream as build_chain with the same seed) as
    per-call launches with their true dependencies, the reference's one-token step pattern: per layer
    RMS norm -> q,k,v (mmvq.mv_norm) | o on q's output | RMS norm of h + o -> gate,up | SiLU(gate) * up
    -> down.  The RMS norms are norm_q8 launches; q's quantised output (o's input) and SiLU(gate) * up
    quantised (down's input) are formed by the q/k/v and gate/up launches themselves (mmvq.NextInput),
    so a layer is six launches.  With PDL every launch starts while the previous one finishes and each
    matvec streams its weights early.
    Returns (step function -> outputs, h0, the list the last down output is written to)."""
    from nemicli_terminal_b200 import mmvq, synth
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    h0 = synth.activations(1, 4096, seed=seed + 11, device=device)[0].contiguous()
    norms, nexts = [], []
    for _ in stack:
        wa = (torch.rand(4096, generator=g, device=device) + 0.5).contiguous()
        wf = (torch.rand(4096, generator=g, device=device) + 0.5).contiguous()
        norms.append((wa, wf))
        # o's input (q's outputs quantised) and down's (SiLU(gate) * up) formed by the launches before them
        nexts.append((mmvq.NextInput(4096, "quant", device), mmvq.NextInput(14336, "silu_mul", device)))
    last = [None]

    def step():
        h, r, outs = h0, None, []
        for mats, (wa, wf), (n_o, n_d) in zip(stack, norms, nexts):
            m = {name: (fmt, raw, n_out, n_in) for name, fmt, n_out, n_in, slot, raw in mats}
            (q, k, v), h = mmvq.mv_norm("Q4_K", [(m[x][1], m[x][2]) for x in ("q", "k", "v")], h, wa, 1e-5, rest=r,
                                        next_input=n_o, src=(0,))
            o = mmvq.mv("Q4_K", m["o"][1], n_o.eingang, 4096, 4096)
            (gt, up), h = mmvq.mv_norm("Q4_K", [(m[x][1], m[x][2]) for x in ("gate", "up")], h, wf, 1e-5, rest=o,
                                        next_input=n_d, src=(0, 1))
            d = mmvq.mv("Q6_K", m["down"][1], n_d.eingang, 4096, 14336)
            outs += [q, k, v, o, gt, up, d]
            r = d
        last[0] = r
        return outs

    step.norms = norms
    return step, h0, last


def calls_launches_per_layer(pdl: bool) -> int:
    """Kernels per layer of build_calls' step: norm, q,k,v (forming o's input) | o | norm, gate,up
    (forming down's input) | down, with or without PDL."""
    return 6


def capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            out = fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    torch.cuda.synchronize()
    return g, out


def time_graph(g, steps: int, warmup: int, dist=None):
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    return a.elapsed_time(b) / 1e3


def max_over_ranks(v: float, dist, device) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_engine_layer(seed0: int, threads: int):
    """The reference's CPU route for one layer: weights dequantised once to bf16 (restated in oracle/)."""
    from nemicli_terminal_b200 import synth
    from oracle import oracle as O
    mats = []
    for j, (name, fmt, n_out, n_in, slot) in enumerate(LAYER):
        raw = synth.blocks(fmt, n_out, n_in, seed=seed0 + j)
        w = torch.from_numpy(O.dequant(fmt, raw.numpy(), n_out * n_in)).view(n_out, n_in).to(torch.bfloat16)
        mats.append((w, slot))
    xs = [torch.randn(1, n, dtype=torch.bfloat16) for n in INPUTS]
    return mats, xs


def cpu_time_layer(mats, xs, reps: int) -> float:
    import torch.nn.functional as F
    t0 = time.perf_counter()
    for _ in range(reps):
        for w, slot in mats:
            F.linear(xs[slot], w)
    return (time.perf_counter() - t0) / reps


def cpu_baseline(budget_s: float = 12.0):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    mats, xs = cpu_engine_layer(7, threads)
    cpu_time_layer(mats, xs, 1)                    # warm
    per = cpu_time_layer(mats, xs, 1)
    reps = max(1, int(budget_s / max(per, 1e-3)))
    per = cpu_time_layer(mats, xs, reps)
    gbs = layer_bytes() / per / 1e9
    return {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"one Llama-3-8B layer (7 projections, {layer_bytes()} GGUF bytes) x {reps} reps, "
                      "bf16 F.linear on weights dequantised once (reference CPU route restated in oracle/)",
            "tok_s_32_layers": 1.0 / (per * LAYERS)}


def sharded_suite(world: int, rank: int, dist, device, steps: int, warmup: int) -> dict:
    """BASELINE configs 3 and 4 sharded over this job's ranks, measured in the same process as the headline:
    the 128256x4096 vocabulary projection (Q8_0 and Q6_K, 1 and 8 tokens) row-sharded with an all-gather of
    the logits, and the 128-expert MoE FFN (batch 1, 4, 16) expert-sharded with all-to-all exchanges.  Per
    case: the time with the collective and without it (compute only), the load imbalance, and parity
    against the unsharded computation on this rank (max over ranks of max|diff| / max|ref|).  Every rank
    holds the same weights (same seeds) and the same vocab input; MoE tokens and routings are per rank.
    Times are CUDA events over graph replays, max over ranks; distinct shard copies rotate so that each
    replay reads more than twice L2."""
    from nemicli_terminal_b200 import moe, mmvq, shard, synth
    from nemicli_terminal_b200.formats import TYPE_ID, row_bytes
    from nemicli_terminal_b200.layers import PackedExperts
    peak, _ = peaks()
    l2 = torch.cuda.get_device_properties(device).L2_cache_size

    def rel(y, ref):
        r = float((y.double() - ref.double()).abs().max() / ref.double().abs().max().clamp_min(1e-30))
        return max_over_ranks(r, dist, device)

    out = {"vocab": {}, "moe": {}}
    for fmt in ("Q8_0", "Q6_K"):
        full = synth.blocks(fmt, VOCAB_ROWS, VOCAB_IN, seed=500, device=device)
        lo, hi = shard.shard_range(VOCAB_ROWS, world, rank)
        loc = shard.slice_rows(fmt, full, VOCAB_ROWS, VOCAB_IN, lo, hi)
        copies = max(1, -(-2 * l2 // loc.numel()))
        lins = [shard.RowShardedLinear(fmt, loc if c == 0 else loc.clone(), VOCAB_ROWS, VOCAB_IN)
                for c in range(copies)]
        total = VOCAB_ROWS * row_bytes(fmt, VOCAB_IN)
        for T in (1, 8):
            x = synth.activations(T, VOCAB_IN, seed=501 + T, device=device)
            x = x[0].contiguous() if T == 1 else x.contiguous()
            par = rel(lins[0](x), mmvq.mv(fmt, full, x, VOCAB_ROWS, VOCAB_IN))
            g_loc, _ = capture(lambda: [l.local(x) for l in lins])
            g_full, _ = capture(lambda: [l(x) for l in lins])
            t_full = max_over_ranks(time_graph(g_full, steps, warmup, dist) / (steps * copies), dist, device)
            t_loc = max_over_ranks(time_graph(g_loc, steps, warmup, dist) / (steps * copies), dist, device)
            del g_loc, g_full
            out["vocab"][f"{fmt} {T}tok"] = {
                "us": t_full * 1e6, "gbs": total / t_full / 1e9, "compute_only_us": t_loc * 1e6,
                "compute_only_hbm_frac_per_gpu": loc.numel() / t_loc / 1e9 / peak,
                "gather_us": (t_full - t_loc) * 1e6, "parity_max_rel": par, "parity": "ok" if par == 0.0 else
                ("ok" if par < 1e-6 else "FAIL")}
        del lins, full, loc
    torch.cuda.empty_cache()
    shapes = ((MOE_FF, MOE_DIM), (MOE_FF, MOE_DIM), (MOE_DIM, MOE_FF))
    per_expert = sum(o * row_bytes("Q4_K", i) for o, i in shapes)
    blobs = [synth.blocks("Q4_K", MOE_EXPERTS * o, i, seed=700 + s_, device=device).view(MOE_EXPERTS, -1)
             for s_, (o, i) in enumerate(shapes)]
    elo, ehi = shard.shard_range(MOE_EXPERTS, world, rank)
    full_ex = [PackedExperts(b, TYPE_ID["Q4_K"], MOE_EXPERTS, o, i, torch.float32) for b, (o, i) in zip(blobs, shapes)]
    loc_ex = [PackedExperts(b[elo:ehi].reshape(-1), TYPE_ID["Q4_K"], ehi - elo, o, i, torch.float32)
              for b, (o, i) in zip(blobs, shapes)]
    layer = shard.ExpertShardedMoE(*loc_ex, MOE_EXPERTS, MOE_DIM)
    ref_layer = moe.MoeFFN(*full_ex)
    for B in (1, 4, 16):
        n_rot = 8
        xs = [synth.activations(B, MOE_DIM, seed=710 + r + 97 * rank, device=device) for r in range(n_rot)]
        routes = [moe.route(synth.router_logits(B, MOE_EXPERTS, seed=720 + r + 97 * rank, device=device), MOE_K)
                  for r in range(n_rot)]
        par = max(rel(layer(x, ix, w), ref_layer(x, ix, w)) for x, (ix, w) in zip(xs[:2], routes[:2]))
        recvs = [layer.dispatch(x, ix)[0] for x, (ix, _) in zip(xs, routes)]
        g_full, _ = capture(lambda: [layer(x, ix, w) for x, (ix, w) in zip(xs, routes)])
        g_cmp, _ = capture(lambda: [layer.compute(r) for r in recvs])
        t_full = max_over_ranks(time_graph(g_full, steps, warmup, dist) / (steps * n_rot), dist, device)
        t_cmp = max_over_ranks(time_graph(g_cmp, steps, warmup, dist) / (steps * n_rot), dist, device)
        del g_full, g_cmp
        single = {}
        if world == 1:
            # the unsharded layer: the grouped kernels (3 launches) and the per-(token, slot) expert matvecs
            per_slot = moe.MoeFFN(*full_ex, act=lambda t: torch.nn.functional.silu(t))
            grouped = lambda x, ix, w: moe.grouped_ffn(*full_ex, x, ix, w)          # noqa: E731
            for name, fn in (("grouped_us", grouped), ("per_slot_us", per_slot)):
                g1, _ = capture(lambda: [fn(x, ix, w) for x, (ix, w) in zip(xs, routes)])
                single[name] = time_graph(g1, steps, warmup, dist) / (steps * n_rot) * 1e6
                del g1
        # load: pairs each owner receives (all ranks' routings), and the experts this rank's owner touches
        sent = torch.stack([torch.bincount(shard.owner_of(ix.reshape(-1), MOE_EXPERTS, world), minlength=world)
                            for ix, _ in routes]).sum(0).to(device)
        if dist is not None:
            dist.all_reduce(sent)
        per_rank = sent.tolist()
        mean = sum(per_rank) / world
        touched = torch.zeros(MOE_EXPERTS, dtype=torch.int64, device=device)
        for ix, _ in routes:
            touched.index_fill_(0, ix.reshape(-1), 1)
        uniq = float(touched.sum()) / n_rot                 # upper bound per routing: this rank's own tokens
        out["moe"][f"batch {B}"] = {
            "us_per_call": t_full * 1e6, "compute_only_us": t_cmp * 1e6, "exchange_us": (t_full - t_cmp) * 1e6,
            "pairs_per_owner": per_rank, "imbalance_max_over_mean": max(per_rank) / mean if mean else 1.0,
            "parity_max_rel": par, "parity": "ok" if par < 1e-5 else "FAIL",
            "touched_expert_gbs_rank0_tokens": uniq * per_expert / t_full / 1e9, **single}
        if single:
            out["moe"][f"batch {B}"]["grouped_touched_gbs"] = uniq * per_expert / (single["grouped_us"] * 1e-6) / 1e9
    del blobs, full_ex, loc_ex, layer, ref_layer
    torch.cuda.empty_cache()
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    mats, xs = cpu_engine_layer(7, threads)
    for _ in range(args.warmup):
        cpu_time_layer(mats, xs, 1)
    t = cpu_time_layer(mats, xs, args.steps)
    gbs = layer_bytes() / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config2: Llama-3-8B layer projections (Q4_K + Q6_K down), batch 1; "
                                   "one layer per step (bounded CPU sample of the 32-layer stack)",
                       "batch": 1, "layers_per_step": 1},
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "one layer per step, bf16 F.linear on weights dequantised once"},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "tok_s_32_layers": 1.0 / (t * LAYERS)}
    print(json.dumps(line), flush=True)


def run_ours(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from nemicli_terminal_b200 import build as nbuild
    nbuild.build()
    from nemicli_terminal_b200 import mmvq, synth

    mmvq.pdl(not args.no_pdl)            # weights are static: the next matvec may stream them early
    peak, peak_kind = peaks()
    stack = build_stack(device, seed0=100000 * rank, n_layers=args.layers)
    lb = layer_bytes()
    step_bytes = lb * args.layers
    results = {}
    mode_used = args.mode
    if args.mode == "chain":
        ch, h0_dev, last_out, chain_outs = build_chain(stack, device, seed=100000 * rank)
        g1, _ = capture(lambda: ch.run())
        with Clocks(local) as clk:
            t = time_graph(g1, args.steps, max(3, args.warmup), dist)
        clocks = clk.summary()
        t = max_over_ranks(t, dist, device)
        results[1] = {"s_per_step": t / args.steps, "steps": args.steps}
    if args.mode == "calls":
        calls_step, h0_dev, calls_last = build_calls(stack, device, seed=100000 * rank)
        g1, _ = capture(calls_step)
        last_out = calls_last[0]
        with Clocks(local) as clk:
            t = time_graph(g1, args.steps, max(3, args.warmup), dist)
        clocks = clk.summary()
        t = max_over_ranks(t, dist, device)
        results[1] = {"s_per_step": t / args.steps, "steps": args.steps}
    for batch in ([1] + [b for b in args.batches if b != 1]):
        if batch == 1:
            continue
        xs = [[synth.activations(batch, n, seed=7919 * l + s + batch, device=device) for s, n in enumerate(INPUTS)]
              for l in range(args.layers)]
        g, outs = capture(lambda: step_fn(stack, xs, batch))
        steps = max(5, args.steps // 2)
        t = time_graph(g, steps, max(3, args.warmup), dist)
        t = max_over_ranks(t, dist, device)
        results[batch] = {"s_per_step": t / steps, "steps": steps}
        del g
    t1 = results[1]["s_per_step"]
    value = world * step_bytes / t1 / 1e9

    if args.mode == "chain":
        # the whole step is one kernel (the chain): its launch time is the step time
        kernel_name = f"chain_kernel (Q4_K 4096 + Q6_K 14336 configs), {len(ch.stages)} stages"
        tk, kbytes = t1, step_bytes
    else:
        # dominant kernel alone: the gate_proj launches (Q4_K 14336x4096, 33.0 MB each) of the stack
        gate_raw = [mats[4][5] for mats in stack]
        e_gate = mmvq.Eingang(synth.activations(1, 4096, seed=17, device=device)[0].contiguous())
        gk, _ = capture(lambda: [mmvq.mv("Q4_K", r, e_gate, 14336, 4096) for r in gate_raw])
        reps = 20
        tk = time_graph(gk, reps, 3) / (reps * len(gate_raw))
        kbytes = 14336 * (4096 // 256) * 144
        kernel_name = ("mv_tma_kernel<Q4_K> gate_proj 14336x4096, quantised input, back to back over the "
                       f"{len(gate_raw)} layers' matrices" + (" with PDL" if not args.no_pdl else ""))
    achieved = kbytes / tk / 1e9
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.txt")
    if os.path.exists(tf):
        for line in open(tf):
            if line.startswith(f"{args.mode}_dram_bytes_per_launch="):
                traffic = int(line.split("=")[1])

    # e2e: the step's inputs from pinned host memory to the device, the step, its results back
    h_in = [[h0_dev.cpu().pin_memory()]]
    dev_in = [[h0_dev]]
    res_dev = [last_out]
    h_out = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in res_dev]
    h2d = sum(x.numel() * x.element_size() for row in h_in for x in row)
    d2h = sum(o.numel() * o.element_size() for o in res_dev)
    e_steps = max(3, args.steps // 2)

    def e2e_step():
        for row_h, row_d in zip(h_in, dev_in):
            for hh, d in zip(row_h, row_d):
                d.copy_(hh, non_blocking=True)
        g1.replay()
        for hh, d in zip(h_out, res_dev):
            hh.copy_(d, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e_steps):
        e2e_step()
    b.record()
    torch.cuda.synchronize()
    te = max_over_ranks(a.elapsed_time(b) / 1e3 / e_steps, dist, device)

    sharded = None if args.no_sharded else sharded_suite(world, rank, dist, device, max(5, args.steps // 10),
                                                          max(3, args.warmup))
    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu) else None
    launches_per_step = 1 if args.mode == "chain" else args.layers * calls_launches_per_layer(not args.no_pdl)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t1 * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded, config-2 distributions)",
            "config": {"workload": "config2: decode step of a 32-layer Llama-3-8B projection stack "
                                   "(q,k,v,o,gate,up Q4_K; down Q6_K), batch 1; RMS norms with the residual "
                                   "adds and the SiLU gate between the matvecs, o_proj reads q_proj's output in "
                                   "place of attention" + ("; one decode-chain launch per step" if args.mode == "chain"
                                                           else "; per-call launches (norm_q8, then the matvecs; o's and "
                                                                "down's inputs formed by the launches before them), PDL"),
                       "layers": args.layers, "batch": 1, "weight_bytes_per_step": step_bytes,
                       "l2": "inputs larger than L2 (4.41 GB distinct weights per step), no flush",
                       "parallelism": (f"value: replicas x{world} of the config-2 stack (one per GPU, no "
                                       "collective); configs 3 and 4 sharded over the GPUs in `sharded`")
                                      if world > 1 else "single GPU",
                       "graph": "whole step captured once in a CUDA graph",
                       "mode": args.mode,
                       "pdl": not args.no_pdl},
            "tok_s": world / t1, "hbm_frac_per_gpu": value / world / peak,
            "batches": {str(b): {"gbs": world * step_bytes / r["s_per_step"] / 1e9,
                                 "tok_s": world * b / r["s_per_step"], "ms_per_step": r["s_per_step"] * 1e3}
                        for b, r in results.items()},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "kernel": kernel_name,
                         "algorithmic_bytes_per_launch": kbytes, "peak_kind": f"{peak_kind} hbm_gbs",
                         "launch_us": tk * 1e6},
            "cpu_baseline": cpu,
            "e2e": {"value": world * step_bytes / te / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": te * 1e3},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "sharded": sharded,
        }
        print(json.dumps(line), flush=True)
    del g1
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


VOCAB_ROWS, VOCAB_IN = 128256, 4096
# single-matrix workloads: config 1 (Q4_0) and config 5 (ternary / 2-bit codebook formats)
MATRIX_WORKLOADS = {
    "cfg1": [("Q4_0", 4096, 4096)],
    "cfg5": [("TQ2_0", 14336, 4096), ("TQ2_0", 4096, 14336), ("IQ2_XXS", 14336, 4096), ("IQ2_XXS", 4096, 14336)],
}
MOE_EXPERTS, MOE_DIM, MOE_FF, MOE_K = 128, 2048, 768, 8


def _init_rank():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from nemicli_terminal_b200 import build as nbuild
    nbuild.build()
    return world, rank, local, device, dist


def run_matrices(args):
    """Configs 1 and 5: batch-1 matvecs of single matrices (mmvq.mv with the in-kernel quantisation),
    each in a CUDA graph over enough distinct copies to read more than twice L2 per replay.  N > 1:
    independent replicas (weak scaling)."""
    world, rank, local, device, dist = _init_rank()
    from nemicli_terminal_b200 import mmvq, synth
    from nemicli_terminal_b200.formats import row_bytes
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    peak, peak_kind = peaks()
    mmvq.pdl(not args.no_pdl)            # static weights: each call may stream them while the previous ends
    per = {}
    tot_bytes, tot_s = 0, 0.0
    for fmt, n_out, n_in in MATRIX_WORKLOADS[args.workload]:
        mb = n_out * row_bytes(fmt, n_in)
        copies = max(1, -(-2 * l2 // mb))
        mats = [synth.blocks(fmt, n_out, n_in, seed=900 + 31 * rank + c, device=device) for c in range(copies)]
        x = synth.activations(1, n_in, seed=901, device=device)[0].contiguous()
        g, _ = capture(lambda: [mmvq.mv(fmt, m, x, n_out, n_in) for m in mats])
        t = time_graph(g, args.steps, max(3, args.warmup), dist) / (args.steps * copies)
        t = max_over_ranks(t, dist, device)
        per[f"{fmt} {n_out}x{n_in}"] = {"gbs": mb / t / 1e9, "us": t * 1e6, "bytes": mb, "copies": copies,
                                        "hbm_frac": mb / t / 1e9 / peak}
        tot_bytes += mb
        tot_s += t
        del g
    if rank == 0:
        line = {"metric": f"weight GB/s of batch-1 quant matvec ({args.workload})",
                "value": world * tot_bytes / tot_s / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": tot_s * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8", "data": f"synthetic (seeded, {args.workload} distributions)",
                "config": {"workload": args.workload + ": " + ", ".join(per), "batch": 1,
                           "l2": "distinct copies of each matrix totalling > 2x L2 per replay",
                           "pdl": not args.no_pdl},
                "matrices": per, "peak": peak, "peak_kind": peak_kind}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


TILE_MATRICES = [("Q4_K", 14336, 4096), ("Q4_K", 4096, 4096), ("Q6_K", 4096, 14336)]
TILE_TOKENS = (17, 32, 64, 112)


def run_tiles(args):
    """The tensor-core tile path (mmvq.mm -> qmv_mm_tc) at config-2 matrix shapes for 17..112 tokens (the
    reference's MMQ range), beside the int8 kernels (mmvq.mv) on the same inputs; CUDA graphs over
    distinct copies reading more than twice L2 per replay.  Parity of every case against oracle C is in
    tests/test_gpu_tc.py.  N > 1: independent replicas."""
    world, rank, local, device, dist = _init_rank()
    from nemicli_terminal_b200 import mmvq, synth
    from nemicli_terminal_b200.formats import row_bytes
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    peak, peak_kind = peaks()
    out = {}
    tot_flop, tot_s = 0.0, 0.0
    for fmt, n_out, n_in in TILE_MATRICES:
        mb = n_out * row_bytes(fmt, n_in)
        copies = max(1, -(-2 * l2 // mb))
        mats = [synth.blocks(fmt, n_out, n_in, seed=950 + c, device=device) for c in range(copies)]
        for M in TILE_TOKENS:
            x = synth.activations(M, n_in, seed=951 + M, device=device)
            row = {}
            for name, fn in (("tile", mmvq.mm_tc), ("int8", mmvq.mv)):
                g, _ = capture(lambda: [fn(fmt, m, x, n_out, n_in) for m in mats])
                t = max_over_ranks(time_graph(g, args.steps, max(3, args.warmup), dist) / (args.steps * copies),
                                   dist, device)
                del g
                row[name + "_us"] = t * 1e6
                if name == "tile":
                    row["tile_tflops"] = 2.0 * M * n_out * n_in / t / 1e12
                    row["tile_weight_gbs"] = mb / t / 1e9
                    tot_flop += 2.0 * M * n_out * n_in
                    tot_s += t
            row["speedup_vs_int8"] = row["int8_us"] / row["tile_us"]
            out[f"{fmt} {n_out}x{n_in} {M}tok"] = row
    if rank == 0:
        line = {"metric": "TFLOP/s of the tensor-core tile path (17..112 tokens, config-2 shapes)",
                "value": world * tot_flop / tot_s / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": tot_s * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded, config-2 distributions)",
                "config": {"workload": "tiles: " + ", ".join(f"{f} {o}x{i}" for f, o, i in TILE_MATRICES),
                           "tokens": list(TILE_TOKENS), "l2": "distinct copies > 2x L2 per replay"},
                "cases": out, "peak": peak, "peak_kind": peak_kind}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_moe(args):
    """Config 4: MoE FFN of 128 Q4_K experts (gate/up 768x2048, down 2048x768), top-8 routing, batch
    1 / 4 / 16, captured in a CUDA graph over 16 rotating routings.  One GPU: moe.MoeFFN.  N GPUs:
    shard.ExpertShardedMoE (experts split, fixed-capacity all-to-all exchanges; each rank has its own
    tokens).  Bytes per call = distinct experts touched x 2,654,208 (per rank)."""
    world, rank, local, device, dist = _init_rank()
    from nemicli_terminal_b200 import mmvq, moe, shard, synth
    from nemicli_terminal_b200.formats import TYPE_ID, row_bytes
    mmvq.pdl(not args.no_pdl)            # static experts; each kernel reads the routing after the previous ends
    from nemicli_terminal_b200.layers import PackedExperts
    lo, hi = shard.shard_range(MOE_EXPERTS, world, rank)
    ne = hi - lo
    shapes = ((MOE_FF, MOE_DIM), (MOE_FF, MOE_DIM), (MOE_DIM, MOE_FF))
    ex = [PackedExperts(synth.blocks("Q4_K", ne * o, i, seed=700 + 7 * rank + s_, device=device), TYPE_ID["Q4_K"],
                        ne, o, i, torch.float32) for s_, (o, i) in enumerate(shapes)]
    per_expert = sum(o * row_bytes("Q4_K", i) for o, i in shapes)
    results = {}
    for B in (1, 4, 16):
        n_rot = 16
        xs = [synth.activations(B, MOE_DIM, seed=710 + r + 97 * rank, device=device) for r in range(n_rot)]
        routes = [moe.route(synth.router_logits(B, MOE_EXPERTS, seed=720 + r + 97 * rank, device=device), MOE_K)
                  for r in range(n_rot)]
        uniq = sum(int(torch.unique(ix).numel()) for ix, _ in routes) / n_rot
        layer = moe.MoeFFN(*ex) if world == 1 else shard.ExpertShardedMoE(*ex, MOE_EXPERTS, MOE_DIM)
        g, _ = capture(lambda: [layer(x, ix, w) for x, (ix, w) in zip(xs, routes)])
        t = time_graph(g, args.steps, max(3, args.warmup), dist) / (args.steps * n_rot)
        del g
        t = max_over_ranks(t, dist, device)
        results[str(B)] = {"us_per_call": t * 1e6, "unique_experts": uniq, "gbs": uniq * per_expert / t / 1e9 * world}
    if rank == 0:
        line = {"metric": "MoE FFN expert weight GB/s (config 4, top-8 of 128 Q4_K experts)",
                "value": results["1"]["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": results["1"]["us_per_call"] / 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded, config-4 distributions)",
                "config": {"workload": "config4: 128 experts x {gate, up 768x2048, down 2048x768} Q4_K, top-8, "
                                       + ("one GPU, graph-captured" if world == 1 else f"expert-sharded over {world} GPUs, "
                                          "own tokens per rank, fixed-capacity all-to-all exchanges, graph-captured"),
                           "bytes_per_expert": per_expert, "rotating_routings": 16, "pdl": not args.no_pdl},
                "batches": results}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_vocab(args):
    """Config 3: the vocabulary projection (128256 x 4096, Q8_0 or Q6_K) row-sharded over the N ranks
    (shard.RowShardedLinear: local matvec + one NCCL all-gather of the fp32 logits), batch --tokens (the
    config names 1 and 8; 2..8 tokens run the tensor-core few-token kernels).  Each rank
    rotates over enough copies of its shard to read more than twice its L2 between repeats.  value:
    whole-matrix weight bytes per second of the sharded call (strong scaling: the matrix is fixed)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from nemicli_terminal_b200 import build as nbuild
    nbuild.build()
    from nemicli_terminal_b200 import shard, synth
    from nemicli_terminal_b200.formats import row_bytes
    fmt = args.vocab_format
    lo, hi = shard.shard_range(VOCAB_ROWS, world, rank)
    local_bytes = (hi - lo) * row_bytes(fmt, VOCAB_IN)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    copies = max(1, -(-2 * l2 // local_bytes))
    lins = [shard.RowShardedLinear(fmt, synth.blocks(fmt, hi - lo, VOCAB_IN, seed=500 + 17 * rank + c, device=device),
                                   VOCAB_ROWS, VOCAB_IN) for c in range(copies)]
    T = args.tokens
    x = synth.activations(T, VOCAB_IN, seed=501, device=device)
    x = x[0].contiguous() if T == 1 else x.contiguous()
    g_local, _ = capture(lambda: [lin.local(x) for lin in lins])
    g_full, outs = capture(lambda: [lin(x) for lin in lins])
    with Clocks(local) as clk:
        t_full = time_graph(g_full, args.steps, max(3, args.warmup), dist) / (args.steps * copies)
    clocks = clk.summary()
    t_local = time_graph(g_local, args.steps, max(3, args.warmup), dist) / (args.steps * copies)
    t_full = max_over_ranks(t_full, dist, device)
    t_local = max_over_ranks(t_local, dist, device)
    total = VOCAB_ROWS * row_bytes(fmt, VOCAB_IN)
    peak, peak_kind = peaks()
    if rank == 0:
        line = {"metric": "vocab projection weight GB/s (row-sharded, all-gathered logits)",
                "value": total / t_full / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_full * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded, config-3 distributions)",
                "config": {"workload": f"config3: {VOCAB_ROWS}x{VOCAB_IN} {fmt} vocabulary projection, batch {T}, "
                                       f"rows split over {world} GPU(s), NCCL all-gather of fp32 logits",
                           "weight_bytes": total, "shard_bytes": local_bytes, "copies_rotated": copies,
                           "l2": "each rank rotates over copies of its shard totalling > 2x L2"},
                "compute_only": {"value": total / t_local / 1e9, "unit": "GB/s", "us": t_local * 1e6,
                                 "hbm_frac_per_gpu": local_bytes / t_local / 1e9 / peak},
                "gather_us": (t_full - t_local) * 1e6, "peak": peak, "peak_kind": peak_kind,
                "gpu_launches": copies * args.steps * ((1 if T == 1 else 2) + (0 if world == 1 else 1)),
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    del g_local, g_full
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batches", type=int, nargs="*", default=[1, 4, 8])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-pdl", action="store_true", help="plain stream order between the matvec launches")
    ap.add_argument("--no-sharded", action="store_true", help="skip configs 3 and 4 (row / expert sharded)")
    ap.add_argument("--mode", choices=["chain", "calls"], default="calls",
                    help="calls: the step as per-call launches with PDL (the reference's call pattern, faster "
                         "here); chain: the step as one decode-chain launch")
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers in the stack (profiling runs use fewer)")
    ap.add_argument("--workload", choices=["stack", "vocab", "moe", "cfg1", "cfg5", "tiles"], default="stack",
                    help="stack: config 2 (the headline); vocab: config 3 row-sharded over the GPUs; "
                         "moe: config 4; cfg1 / cfg5: the single-matrix configs; tiles: the tensor-core tile "
                         "path for 17..112 tokens")
    ap.add_argument("--vocab-format", choices=["Q8_0", "Q6_K"], default="Q8_0")
    ap.add_argument("--tokens", type=int, default=1, help="vocab workload: tokens per call (config 3: 1 and 8)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "vocab":
        run_vocab(args)
    elif args.workload == "moe":
        run_moe(args)
    elif args.workload == "tiles":
        run_tiles(args)
    elif args.workload in MATRIX_WORKLOADS:
        run_matrices(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
