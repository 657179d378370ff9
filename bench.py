#!/usr/bin/env python3
"""Benchmark of the B200 sparse-decode hot path (attention-lab's score -> top-k -> attend, plus the cache append).

Workload (default `c3`, the configuration the headline metric is quoted on: 32K context): a Qwen3-8B-shape decode
step of the hot path over every layer: 36 layers, B = 32 requests per GPU, G = 8 KV groups, h = 4 query heads per
group, d = 128, r = 32, legal length L = 32768, rho = 1/32 (k = 1024, S = 1092), bf16 K/V and bf16 index keys (the
reference's default index layout), random synthetic data (no checkpoint or dataset is involved in this path).
One step = for every layer: the K/V append of the new token, then the fused sparse step (z column, u, candidate
scores, top-k, F merge, gather-free attention). Every layer has its own cache, so nothing stays in L2 between layers
(each fused launch reads 679 MB).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c3|c2|c4|c1]

Under torchrun every rank runs the same per-GPU workload on its own requests (request sharding, no collective on
the data path: weak scaling); the timed region is bracketed by barriers and synchronisations, its device time is the
max over ranks, and rank 0 prints one JSON line. `--impl reference` times the CPU restatement of the reference's
path (oracle/oracle.py) on the host cores and prints the reference arm's line. Two other measurements print their
own line: `--context-split` (C4, one sequence split over the torchrun ranks) and `--prefill` (C5, the batched
prefill scorer over one 8192-token chunk).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: (layers, B, G, h, L, rho, description)
    "c3": (36, 32, 8, 4, 32768, 1 / 32, "C3: Qwen3-8B-shape hot path, 36 layers, B=32 per GPU, L=32768, rho=1/32"),
    "c2": (28, 1, 8, 2, 8193, 1 / 32, "C2: Qwen3-0.6B-shape hot path, 28 layers, B=1, L=8193, rho=1/32"),
    "c4": (1, 1, 8, 4, 131072, 1 / 32, "C4: one Qwen3-8B-shape layer, B=1, L=131072, rho=1/32"),
    "c1": (1, 1, 8, 2, 2048, 1 / 32, "C1: one Qwen3-0.6B-shape layer, B=1, L=2048, rho=1/32"),
}
D, R = 128, 32


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c3")
    ap.add_argument("--index-dtype", choices=["bf16", "f32"], default="bf16")
    ap.add_argument("--cluster", type=int, default=0, help="CTAs per (batch, group); 0 = automatic")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-baselines", action="store_true", help="skip the same-box dense / torch reference timings")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU work budget of the CPU baseline sample")
    ap.add_argument("--batch", type=int, default=0, help="override the workload's requests per GPU (profiling cases)")
    ap.add_argument("--layers", type=int, default=0, help="override the workload's layer count (profiling cases)")
    ap.add_argument("--context-split", action="store_true",
                    help="C4 measurement: one sequence split over the torchrun ranks (attention_lab_b200.context_split)")
    ap.add_argument("--no-graph", action="store_true", help="context split: launch every step from the host")
    ap.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                    help="context split: move keys and partials over peer memory (default) or NCCL all-gathers")
    ap.add_argument("--model", choices=["c2", "c3"], default=None,
                    help="end-to-end decode of a random-init Qwen3 through attention_lab_b200.runner: c2 (0.6B, 8192-token "
                         "prompt, 256 greedy steps) or c3 (8B shape, 32K context per request); sparse vs dense")
    ap.add_argument("--model-steps", type=int, default=0, help="decode steps of --model (0 = the config's)")
    ap.add_argument("--model-graph", action="store_true",
                    help="--model: also time one decode step captured as a CUDA graph and replayed at a fixed context")
    ap.add_argument("--prefill", action="store_true",
                    help="C5 measurement: the batched prefill scorer over one 8192-token chunk (8 heads, k=256)")
    return ap.parse_args()


def workload(args):
    layers, B, G, h, L, rho, desc = WORKLOADS[args.workload]
    if args.batch or args.layers:
        layers, B = args.layers or layers, args.batch or B
        desc += f" [profiling override: B={B}, layers={layers}]"
    return layers, B, G, h, L, rho, desc


def ledger(B, G, h, L, rho, layers, zb, eb):
    """Algorithmic bytes from the reference's ledger terms (scripts/roofline.py:61-74, scan_scope=candidates),
    per (layer, request): score = G*r*M*zb, attend = S*G*d*2*eb."""
    from attention_lab_b200.selection import fixed_budget, selection_layout
    lay = selection_layout(L)
    k = lay.clamp_k(fixed_budget(L, rho))
    M, S = lay.candidate_count, lay.fixed_count + k
    score = G * R * M * zb
    attend = S * G * D * 2 * eb
    return {"k": k, "S": S, "M": M, "lo": lay.candidate_lo, "hi": lay.candidate_hi, "F": lay.fixed_count,
            "score_bytes": score, "attend_bytes": attend, "d_s1_per_layer_request": score + attend,
            "per_launch": B * (score + attend), "dense_kv_per_layer_request": 2 * G * L * D * eb}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region (every 20 ms)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    return 6650.0, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


# ------------------------------------------------------------------------------------------------ CPU side
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


class CpuReferencePath:
    """The reference's hot path on the host cores: oracle/torch_ref.py, the reference's own torch operators
    (decode.py:145-163 and the K/V copies of qwen_wrap.py:90-106) in its dtypes (bf16 K/V, the index dtype for z),
    over the workload's B requests at legal length L. Host memory holds one layer's caches ([B,G,L,d] K and V, [B,G,r,L]
    index), which every layer of the step reuses with its own indexer weights and step inputs. Caches are filled from
    one N(0,1) block (each request and tensor at its own offset), so building them costs a copy, not a random draw."""

    def __init__(self, B, G, h, L, rho, layers, zb):
        import torch
        from attention_lab_b200.selection import build_step_plan, fixed_budget
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.torch, self.B, self.G, self.h, self.L, self.layers = torch, B, G, h, L, layers
        bf = torch.bfloat16
        idt = bf if zb == 2 else torch.float32
        gen = torch.Generator().manual_seed(0)
        block = torch.randn(1 << 24, generator=gen).to(bf)
        n_blk = block.numel()

        def filled(shape, dtype, scale, salt):
            t = torch.empty(shape, dtype=dtype)
            flat = t.view(-1)
            step = 7919 * (salt + 1)
            for i, a in enumerate(range(0, flat.numel(), n_blk)):
                n = min(n_blk, flat.numel() - a)
                off = (i * step) % (n_blk - n + 1) if n < n_blk else 0
                flat[a:a + n].copy_(block[off:off + n])
            if scale != 1.0:
                t.mul_(scale)
            return t
        C = L
        self.K = filled((B, G, C, D), bf, 1.0, 1)
        self.V = filled((B, G, C, D), bf, 1.0, 2)
        self.Z = filled((B, G, R, C), idt, 0.23, 3)
        self.WQ = [(torch.randn(G, h * D, R, generator=gen) * (0.02 / math.sqrt(R))).to(idt) for _ in range(layers)]
        self.WK = [(torch.randn(G, R, D, generator=gen) * 0.02).to(idt) for _ in range(layers)]
        self.Q = [torch.randn(B, G, h, 1, D, generator=gen).to(bf) for _ in range(layers)]
        self.QP = [torch.randn(B, G, h, 1, D, generator=gen).to(idt) for _ in range(layers)]
        self.KPN = [torch.randn(B, G, 1, D, generator=gen).to(idt) for _ in range(layers)]
        self.KN = [torch.randn(B, G, 1, D, generator=gen).to(bf) for _ in range(layers)]
        self.plan = build_step_plan(B, G, C, L, fixed_budget(L, rho), "cpu")

    def layer(self, l):
        from oracle import torch_ref as tr
        p = self.plan
        with self.torch.inference_mode():
            tr.append_kv(self.K, self.V, self.L - 1, self.KN[l], self.KN[l])
            out, _ = tr.sparse_decode_step_kernel(self.Q[l], self.QP[l], self.K, self.V, self.Z, self.WQ[l], self.WK[l],
                                                  p.fixed_rows, p.off_lo, p.lo, p.hi, p.k, p.selected_count,
                                                  k_pre_new=self.KPN[l], write_col=p.write_col, scale=1 / math.sqrt(D))
        return out

    def step(self):
        for l in range(self.layers):
            self.layer(l)

    def describe(self):
        return (f"oracle/torch_ref.py: the reference's torch operators (matmul, topk, cat, index_select, SDPA, copy_) "
                f"in bf16, B={self.B} requests x {self.layers} layers at L={self.L} per step, "
                f"{self.threads} torch threads on {cpu_model()}")


def cpu_sample(args, B, G, h, L, rho, layers, budget_s):
    """The cpu_baseline of the GPU arm: layers of the step through CpuReferencePath until ~budget_s has passed
    (at least one), tokens/s = B / (layers x mean layer time). Returns the cpu_baseline object."""
    ref = CpuReferencePath(B, G, h, L, rho, layers, 2 if args.index_dtype == "bf16" else 4)
    ref.layer(0)                                                  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        ref.layer(n % layers)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    per_layer = (time.perf_counter() - t0) / n
    return {"value": B / (per_layer * layers), "unit": "tokens/s", "cores": ref.threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{n} layer(s) of the step ({ref.describe()}); tokens/s = B / (layers x mean layer time)"}


def run_reference_arm(args):
    """The reference arm: W warm-up and K timed FULL steps (every layer, every request) of the reference's path on
    the host cores (CpuReferencePath), timed with the wall clock; rank 0 only (other ranks exit at once)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    layers, B, G, h, L, rho, desc = workload(args)
    zb = 2 if args.index_dtype == "bf16" else 4
    ref = CpuReferencePath(B, G, h, L, rho, layers, zb)
    for _ in range(args.warmup):
        ref.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.step()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = B / (ms / 1e3)
    sample = f"{args.steps} full step(s) after {args.warmup} warm-up step(s): {ref.describe()}"
    line = {"impl": "reference", "metric": metric_name(args.workload), "value": round(value, 3), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_of(args, desc, B, G, h, L, rho, layers),
            "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": ref.threads, "kind": "port",
                             "cpu_model": cpu_model(), "sample": sample},
            "timed_s": round(sum(times), 2),
            "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def metric_name(workload):
    return "decode tokens/s of the sparse score+top-k+attend hot path (all layers, append included)"


def config_of(args, desc, B, G, h, L, rho, layers):
    return {"workload": desc, "layers": layers, "batch_per_gpu": B, "global_batch": B * args.gpus, "seq_len": L,
            "kv_groups": G, "heads_per_group": h, "head_dim": D, "index_width": R, "rho": rho,
            "kv_dtype": "bf16", "index_dtype": args.index_dtype, "parallelism": f"request-sharded x{args.gpus}",
            "l2": "inputs larger than L2: every layer has its own cache and one fused launch reads >= 126 MB"
                  if args.workload in ("c3", "c4") else "per-layer caches (working set per launch below L2)"}


# ------------------------------------------------------------------------------------------------ GPU side
def run_context_split(args):
    """One layer of C4 (B=1, L=131072, rho=1/32) with its positions split over the torchrun ranks: every timed step is
    the whole protocol (local top-k, key exchange, threshold, partial attend, partial exchange, merge; the exchanges
    over peer memory, or NCCL all-gathers with --exchange nccl). Device
    time per step with CUDA events, max over ranks; prints one JSON line (rank 0)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from attention_lab_b200 import context_split as csplit
    from attention_lab_b200.selection import fixed_budget
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _, B, G, h, L, rho, desc = WORKLOADS["c4"]
    k0 = fixed_budget(L, rho)
    plan = csplit.plan_shard(L, k0, rank, world, L)
    cs_ = plan.shard_capacity
    gen = torch.Generator(device=dev).manual_seed(99 + rank)

    def rnd(*shape, scale=1.0):
        t = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        return t.normal_(0.0, scale, generator=gen)
    K, V, Z = rnd(B, G, cs_, D), rnd(B, G, cs_, D), rnd(B, G, R, cs_, scale=0.23)
    WQ, WK = rnd(G, h * D, R, scale=0.02 / math.sqrt(R)), rnd(G, R, D, scale=0.02)
    Q, QP, KPN = rnd(B, G, h, 1, D), rnd(B, G, h, 1, D), rnd(B, G, 1, D)
    xchg = csplit.PeerExchange(B, G, plan.k, h, device=dev) if args.exchange == "peer" else None

    def step():    # every rank passes the newest key; the shard that owns position L - 1 writes its z column
        return csplit.context_split_decode_step(Q, QP, K, V, Z, WQ, WK, plan, k_pre_new=KPN, exchange=xchg)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = None
    if not args.no_graph:          # the whole protocol (kernels and both all-gathers) as one CUDA graph
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
    run = graph.replay if graph is not None else step
    run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    lg = ledger(B, G, h, L, rho, 1, 2, 2)
    peak, _ = measured_peak()
    if rank == 0:
        print(json.dumps({"metric": "C4 context-split layer latency (whole protocol, max over ranks)",
                          "value": round(ms * 1e3, 2), "unit": "us", "n_gpus": world, "steps": args.steps,
                          "warmup": max(3, args.warmup), "higher_is_better": False, "scaling": "strong",
                          "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": desc + f", split over {world} rank(s)", "k": lg["k"], "S": lg["S"],
                                     "shard_capacity": cs_, "cuda_graph": graph is not None,
                                     "exchange": ("peer memory (NVLink loads, epoch flags)" if xchg is not None
                                                  else "NCCL all-gathers") if world > 1 else "none (one rank)"},
                          "ledger_bytes": lg["d_s1_per_layer_request"],
                          "achieved_gbs_aggregate": round(lg["d_s1_per_layer_request"] / (ms * 1e-3) / 1e9, 1),
                          "peak_gbs_per_gpu": peak}))
    del graph, run                 # a graph holding NCCL work is released before the process group
    if xchg is not None:
        xchg.close()
    if world > 1:
        dist.destroy_process_group()


def run_model(args):
    """End-to-end greedy decode of a random-init Qwen3 through attention_lab_b200.runner (the reference wrapper's
    interface on this library's kernels), sparse (rho = 1/32, index selector) against dense decode over the same
    caches, both with this library's dense kernel and with torch SDPA (the reference's A path, sdpa_fold).

    c2: Qwen3-0.6B, B = 1, an 8192-token prompt of uniform ids prefilled in 2048-token chunks (this builds the index
        table), then 256 greedy steps (legal lengths 8193 .. 8448, k0 = 256).
    c3: Qwen3-8B shape, 32K context per request, as many requests as the GPU holds next to the weights (at most 32).
        The caches are filled with synthetic N(0,1) K/V and N(0, 0.23^2) index keys (a 32 x 32K-token prefill through
        an 8B model is not part of the decode measurement), then greedy steps at legal lengths up to 32768.
    Timing: CUDA events around the decode loop (device time; every step is a full model forward from token ids to
    next-token logits and the greedy argmax, with the runner's host work in the loop); tokens/s = B x steps / time."""
    import torch
    from attention_lab_b200 import runner as rn
    from attention_lab_b200.selection import fixed_budget
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    big = args.model == "c3"
    cfg = rn.qwen3_config("8b" if big else "0.6b")
    model = rn.random_qwen3(cfg, device=dev, dtype=torch.bfloat16, seed=0)
    idt = torch.bfloat16 if args.index_dtype == "bf16" else torch.float32
    n_params = sum(p.numel() for p in model.parameters())
    holder = rn.wrap_model(model)
    G, d, layers, V = cfg.num_key_value_heads, cfg.head_dim, cfg.num_hidden_layers, cfg.vocab_size
    if big:
        ctx, steps = 32768, args.model_steps or 16
        cap = ctx
        per_req = layers * (2 * G * cap * d * 2 + G * 32 * cap * (2 if idt == torch.bfloat16 else 4))
        free = torch.cuda.mem_get_info(dev)[0]
        B = int(max(1, min(32, (free - (6 << 30)) // per_req)))
    else:
        ctx, steps, B = 8192, args.model_steps or 256, 1
        cap = ctx + steps
    st = rn.make_state(model, cap, "sparse", batch=B, index_dtype=idt)
    cache = st.cache
    gen = torch.Generator(device=dev).manual_seed(5)
    with torch.inference_mode():
        if big:
            start = ctx - steps
            for l in range(layers):
                cache.k[l].normal_(0.0, 1.0, generator=gen)
                cache.v[l].normal_(0.0, 1.0, generator=gen)
                cache.z[l].normal_(0.0, 0.23, generator=gen)
            cache.valid_length = start
        else:
            prompt = torch.randint(0, 151643, (B, ctx), generator=gen, device=dev)
            rn.LabRunner(model, holder, st).prefill(prompt, 2048)
            start = ctx
    dense = rn.LabCache.__new__(rn.LabCache)             # the same K/V buffers, without the index table
    dense.__dict__.update(cache.__dict__)
    dense.z, dense.index_dim = None, None
    dense.writes, dense.last_write = list(cache.writes), list(cache.last_write)
    first = torch.randint(0, 151643, (B, 1), generator=gen, device=dev)

    def decode(state, n):
        run = rn.LabRunner(model, holder, state)
        state.cache.rollback(start)
        if state.mode == "sparse":
            state.begin_request(1 / 32)
        tok = first
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        e0.record()
        for _ in range(n):
            tok = run.step(tok).argmax(dim=-1)
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n, (time.perf_counter() - t0) * 1e3 / n

    def graphed(state, n):
        """One decode step at legal length start + 1 (model forward, the read, greedy argmax written back into the
        step's input) captured as a CUDA graph, replayed n times: every replay is a whole decode step at that
        context (slot `start` is rewritten each time), with no host work between steps."""
        run = rn.LabRunner(model, holder, state)
        tok = first.clone()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                state.cache.rollback(start)
                if state.mode == "sparse":
                    state.begin_request(1 / 32)
                tok.copy_(run.step(tok).argmax(dim=-1))
        torch.cuda.current_stream(dev).wait_stream(side)
        state.cache.rollback(start)
        if state.mode == "sparse":
            state.begin_request(1 / 32)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            tok.copy_(run.step(tok).argmax(dim=-1))
        state.cache.rollback(start)
        graph.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            graph.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        del graph
        return e0.elapsed_time(e1) / n

    res = {}
    with torch.inference_mode():
        for name, state in (("sparse", st), ("dense_kernel", rn.LabState(dense, None, mode="full")),
                            ("dense_sdpa", rn.LabState(dense, None, mode="full", decode_backend="sdpa_fold"))):
            decode(state, min(3, steps))                  # warm-up
            ms, wall = decode(state, steps)
            res[name] = {"tokens_per_s": round(B / (ms / 1e3), 2), "ms_per_step": round(ms, 3),
                         "wall_ms_per_step": round(wall, 3)}
            if args.model_graph:
                gms = graphed(state, max(steps, 10))
                res[name]["graph_tokens_per_s"] = round(B / (gms / 1e3), 2)
                res[name]["graph_ms_per_step"] = round(gms, 3)
    k0 = fixed_budget(start + 1, 1 / 32)
    line = {"metric": f"end-to-end decode tokens/s, random-init Qwen3-{'8B shape' if big else '0.6B'} ({args.model.upper()})",
            "value": res["sparse"]["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": steps,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": (f"{args.model.upper()}: {layers} layers, hidden {cfg.hidden_size}, "
                                    f"{cfg.num_attention_heads}/{G} heads, d {d}, vocab {V}, B {B}, context up to "
                                    f"{start + steps}, rho 1/32 (k0 {k0}), index {args.index_dtype}"),
                       "batch": B, "parameters": n_params, "cache_capacity": cap,
                       "caches": "synthetic fill" if big else "prefilled from an 8192-token prompt (chunks of 2048)",
                       "cuda_graph": False},
            "modes": res,
            "speedup_vs_dense_sdpa": round(res["sparse"]["tokens_per_s"] / res["dense_sdpa"]["tokens_per_s"], 3),
            "speedup_vs_dense_kernel": round(res["sparse"]["tokens_per_s"] / res["dense_kernel"]["tokens_per_s"], 3)}
    if args.model_graph:
        g = {k: v["graph_tokens_per_s"] for k, v in res.items()}
        line["graph"] = {"what": f"one decode step at legal length {start + 1} captured as a CUDA graph and replayed "
                                 "(no host work between steps)",
                         "sparse_tokens_per_s": g["sparse"],
                         "speedup_vs_dense_sdpa": round(g["sparse"] / g["dense_sdpa"], 3),
                         "speedup_vs_dense_kernel": round(g["sparse"] / g["dense_kernel"], 3)}
    print(json.dumps(line), flush=True)
    return 0


def cpu_prefill_sample(H, T, k, budget_s):
    """The whole C5 chunk (H heads x T rows) through oracle.cpu_prefill_rows (float32 numpy), blocks of 256 rows in
    parallel over the host cores (one BLAS thread each); repeated until ~budget_s. Returns query rows/s."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from threadpoolctl import threadpool_limits
    from oracle import oracle as orc
    rng = np.random.default_rng(0)
    u = rng.standard_normal((H, T, R), dtype=np.float32)
    zT = rng.standard_normal((H, R, T), dtype=np.float32)
    blocks = [(h, t0) for t0 in range(T - 256, -1, -256) for h in range(H)]      # longest rows first
    workers = max(1, min(64, os.cpu_count() or 1))

    def one(b):
        h, t0 = b
        return orc.cpu_prefill_rows(u[h], zT[h], 0, t0, t0 + 256, k)
    with threadpool_limits(1), ThreadPoolExecutor(workers) as ex:
        passes, t0 = 0, time.perf_counter()
        while True:
            list(ex.map(one, blocks))
            passes += 1
            if time.perf_counter() - t0 >= budget_s:
                break
        wall = time.perf_counter() - t0
    return {"value": round(H * T * passes / wall, 1), "unit": "rows/s", "cores": workers, "kind": "port",
            "sample": f"the whole chunk ({H} heads x {T} rows, float32 matmul + argpartition per row), {passes} "
                      f"pass(es) in {wall:.1f} s over {workers} threads"}


def run_prefill(args):
    """Config C5: the batched prefill scorer (al_prefill_score_topk) over one chunk of T = 8192 query rows against
    C = 8192 cached keys, 8 KV heads, r = 32, bf16 ~N(0,1) inputs, causal candidates, top-256 per row. One launch per
    step; the L2 is flushed (a 256 MiB write) before every timed launch, outside the events. Under torchrun every rank
    runs its own chunk (replicas, no collective). Prints one JSON line (rank 0)."""
    import torch
    import torch.distributed as dist
    from attention_lab_b200 import ops
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    H, T, C, k = 8, 8192, 8192, 256
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    u = torch.randn(H, T, R, generator=gen, device=dev).to(torch.bfloat16)
    zT = torch.randn(H, R, C, generator=gen, device=dev).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        ops.prefill_score_topk(u, zT, k)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for e0, e1 in ev:
            flush.fill_(1)
            e0.record(stream)
            ops.prefill_score_topk(u, zT, k)
            e1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # end to end through the operator: pinned host inputs in, indices back to the host, every step
    hu, hz = u.cpu().pin_memory(), zT.cpu().pin_memory()
    hidx = torch.empty((H, T, k), dtype=torch.int32).pin_memory()
    du, dz = torch.empty_like(u), torch.empty_like(zT)

    def e2e_step():
        du.copy_(hu, non_blocking=True)
        dz.copy_(hz, non_blocking=True)
        hidx.copy_(ops.prefill_score_topk(du, dz, k), non_blocking=True)
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    m = [max(0, min(C, p + 1 - 64) - min(4, p + 1)) for p in range(T)]
    flops = 2.0 * H * R * sum(m)                          # candidate columns only
    nbytes = u.numel() * 2 + zT.numel() * 2 + H * T * k * 4
    hbm, _ = measured_peak()
    peaks = ROOT / "MEASURED_PEAKS.json"
    tflops_peak = float(json.loads(peaks.read_text())["bf16_tflops"]) if peaks.exists() else 1590.0
    achieved = nbytes / (ms * 1e-3) / 1e9
    line = {"metric": "C5 prefill scorer query rows per second (8 heads x 8192 rows, top-256 each)",
            "value": round(world * H * T / (ms * 1e-3), 1), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C5: batched prefill scorer, u [8,8192,32] x zT [8,32,8192] bf16 N(0,1), causal, "
                                   "per-row top-256 (int32 positions out)",
                       "l2": "flushed before every timed launch (256 MiB write)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": None, "algorithmic_bytes": nbytes,
                         "tensor": {"flops": flops, "achieved_tflops": round(flops / (ms * 1e-3) / 1e12, 2),
                                    "peak_tflops": tflops_peak,
                                    "frac": round(flops / (ms * 1e-3) / 1e12 / tflops_peak, 5)}},
            "e2e": {"value": round(world * H * T / (e2e_ms * 1e-3), 1), "unit": "rows/s",
                    "h2d_bytes_per_step": u.numel() * 2 + zT.numel() * 2, "d2h_bytes_per_step": H * T * k * 4},
            "gpu_launches": args.steps, "clocks": clocks.summary()}
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_prefill_sample(H, T, k, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.context_split:
        return run_context_split(args)
    if args.prefill:
        return run_prefill(args)
    if args.model:
        return run_model(args)
    import torch
    import torch.distributed as dist
    import attention_lab_b200 as al
    from attention_lab_b200 import _lib
    from attention_lab_b200.selection import build_step_plan

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    layers, B, G, h, L, rho, desc = workload(args)
    zb = 2 if args.index_dtype == "bf16" else 4
    idt = torch.bfloat16 if zb == 2 else torch.float32
    kvt = torch.bfloat16
    lg = ledger(B, G, h, L, rho, layers, zb, 2)
    C = L                                    # the step re-decodes position L-1: append + z column are idempotent
    plan = build_step_plan(B, G, C, L, lg["k"], dev)
    assert (plan.k, plan.selected_count) == (lg["k"], lg["S"])
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    def rnd(*shape, dtype, scale=1.0):
        t = torch.empty(shape, dtype=dtype, device=dev)
        t.normal_(0.0, scale, generator=gen)
        return t

    # per-layer caches, weights and step inputs, resident before timing
    Ks = [rnd(B, G, C, D, dtype=kvt) for _ in range(layers)]
    Vs = [rnd(B, G, C, D, dtype=kvt) for _ in range(layers)]
    Zs = [rnd(B, G, R, C, dtype=idt, scale=0.23) for _ in range(layers)]
    WQ = [rnd(G, h * D, R, dtype=idt, scale=0.02 / math.sqrt(R)) for _ in range(layers)]
    WK = [rnd(G, R, D, dtype=idt, scale=0.02) for _ in range(layers)]
    Q = [rnd(B, G, h, 1, D, dtype=kvt) for _ in range(layers)]
    QP = [rnd(B, G, h, 1, D, dtype=idt) for _ in range(layers)]
    KPN = [rnd(B, G, 1, D, dtype=idt) for _ in range(layers)]
    KN = [rnd(B, G, 1, D, dtype=kvt) for _ in range(layers)]
    VN = [rnd(B, G, 1, D, dtype=kvt) for _ in range(layers)]
    OUT = [torch.empty(B, G, h, 1, D, dtype=kvt, device=dev) for _ in range(layers)]
    lib = _lib.load()
    idx_code = _lib.AL_BF16 if zb == 2 else _lib.AL_F32
    kv_strides = (_lib.strides(KN[0], 4), _lib.strides(VN[0], 4))
    scale = 1 / math.sqrt(D)

    def append_args(l, stream):
        return (Ks[l].data_ptr(), Vs[l].data_ptr(), _lib.AL_BF16, KN[l].data_ptr(), kv_strides[0], VN[l].data_ptr(),
                kv_strides[1], _lib.AL_BF16, None, 0, None, None, None, None, None, B, G, C, D, R, L - 1, 1, stream)

    def step_args(l, stream):
        return (Q[l].data_ptr(), Q[l].stride(0), Q[l].stride(1), Q[l].stride(2),
                QP[l].data_ptr(), QP[l].stride(0), QP[l].stride(1), QP[l].stride(2),
                Ks[l].data_ptr(), Vs[l].data_ptr(), _lib.AL_BF16, Zs[l].data_ptr(), WQ[l].data_ptr(),
                WK[l].data_ptr(), idx_code, KPN[l].data_ptr(), KPN[l].stride(0), KPN[l].stride(1),
                plan.fixed_rows.data_ptr(), plan.off_lo.data_ptr(), B, G, h, D, R, C, plan.lo, plan.hi, plan.k,
                plan.selected_count, plan.fixed_count, plan.write_col, scale, 0, OUT[l].data_ptr(), None, None,
                args.cluster, stream)

    stream = torch.cuda.Stream(device=dev)
    sh = stream.cuda_stream
    A_ARGS = [append_args(l, sh) for l in range(layers)]
    S_ARGS = [step_args(l, sh) for l in range(layers)]

    def step_raw():
        for l in range(layers):
            _lib.check(lib.al_append_kvz(*A_ARGS[l]))
            _lib.check(lib.al_sparse_decode_step(*S_ARGS[l]))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- correctness guard before timing: one step, kernel error word clear
    with torch.cuda.stream(stream):
        step_raw()
    torch.cuda.synchronize(dev)
    assert _lib.device_status() == 0

    # ---- capture one step (2 launches per layer) as a CUDA graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_raw()
    torch.cuda.synchronize(dev)

    # ---- device-timed value: K graph replays after W warm-ups
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    t_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    value = world * B / (t_ms / 1e3)

    # ---- roofline of the dominant kernel: the `layers` fused launches of one step captured alone as a CUDA graph and
    #      replayed (launch_ms = graph time / layers, no per-launch event overhead); each launch also timed on its own
    #      with events as a cross-check; the appends timed alone
    fgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(fgraph, stream=stream):
        for l in range(layers):
            _lib.check(lib.al_sparse_decode_step(*S_ARGS[l]))
    n_roof = max(3, min(args.steps, 10))
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(layers)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(layers)]
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        fgraph.replay()
        g0.record(stream)
        for i in range(n_roof):
            fgraph.replay()
        g1.record(stream)
        for l in range(layers):
            starts[l].record(stream)
            _lib.check(lib.al_sparse_decode_step(*S_ARGS[l]))
            ends[l].record(stream)
        a0.record(stream)
        for i in range(n_roof):
            for l in range(layers):
                _lib.check(lib.al_append_kvz(*A_ARGS[l]))
        a1.record(stream)
    torch.cuda.synchronize(dev)
    fused_ms = max_over_ranks(g0.elapsed_time(g1) / (n_roof * layers))
    event_ms = statistics.mean(starts[l].elapsed_time(ends[l]) for l in range(layers))
    append_ms = a0.elapsed_time(a1) / (n_roof * layers)
    del fgraph
    peak, peak_src = measured_peak()
    achieved = lg["per_launch"] / (fused_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None,
                "kernel": "sparse_step_kernel (fused z column + u + scan + radix top-k + gather-free attend)",
                "bytes_per_launch": lg["per_launch"], "launch_ms": round(fused_ms, 5),
                "launch_timing": f"CUDA graph of the {layers} fused launches of a step, {n_roof} replays, time / launches",
                "launch_ms_events": round(event_ms, 5), "peak_source": peak_src,
                "bytes_rule": "B x (G*r*M*zb + S*G*d*2*eb) per launch (scripts/roofline.py:61-74 terms)"}
    traffic_file = ROOT / "profiles" / f"traffic_{args.workload}_{args.index_dtype}.json"
    if traffic_file.exists():
        try:
            roofline["traffic"] = json.loads(traffic_file.read_text()).get("dram_bytes_per_launch")
        except ValueError:
            pass

    # ---- e2e through the public API with host buffers: H2D of every layer's step inputs, the drop-in operators,
    #      D2H of every layer's attention output. The copies run on two side streams so that layer l's inputs land
    #      while earlier layers compute and each output leaves as soon as it is written; inputs are double-buffered
    #      across steps. The timed region ends after the last D2H copy.
    e2e = None
    if not args.no_e2e:
        host_in = [[t.cpu().pin_memory() for t in (Q[l], QP[l], KPN[l], KN[l], VN[l])] for l in range(layers)]
        host_out = [torch.empty(OUT[0].shape, dtype=kvt).pin_memory() for _ in range(layers)]
        dev_in = [[[torch.empty_like(t) for t in (Q[l], QP[l], KPN[l], KN[l], VN[l])] for l in range(layers)]
                  for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for row in host_in for t in row)
        d2h = sum(t.numel() * t.element_size() for t in host_out)
        h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in = [[torch.cuda.Event() for _ in range(layers)] for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(layers)]
        done = [torch.cuda.Event(), torch.cuda.Event()]
        state = {"i": 0}

        def e2e_step():
            j = state["i"] % 2
            first = state["i"] < 2
            state["i"] += 1
            with torch.cuda.stream(h2d_s):
                if not first:
                    h2d_s.wait_event(done[j])            # the step that last used these buffers has consumed them
                for l in range(layers):
                    for dst, src in zip(dev_in[j][l], host_in[l]):
                        dst.copy_(src, non_blocking=True)
                    ev_in[j][l].record(h2d_s)
            for l in range(layers):
                stream.wait_event(ev_in[j][l])
                q, qp, kpn, kn, vn = dev_in[j][l]
                al.append_kvz(Ks[l], Vs[l], None, L - 1, kn, vn)
                out = al.sparse_decode_step_kernel(q, qp, Ks[l], Vs[l], Zs[l], WQ[l], WK[l], plan.fixed_rows,
                                                   plan.off_lo, plan.lo, plan.hi, plan.k, plan.selected_count,
                                                   k_pre_new=kpn, write_col=plan.write_col, scale=scale,
                                                   cluster=args.cluster)
                ev_out[l].record(stream)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_out[l])
                    host_out[l].copy_(out, non_blocking=True)
                    out.record_stream(d2h_s)
            done[j].record(stream)

        n_e2e = max(3, min(args.steps, 30))
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                e2e_step()
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(n_e2e):
                e2e_step()
            stream.wait_stream(d2h_s)                    # the last outputs are on the host
            f1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1)) / n_e2e
        e2e = {"value": world * B / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4), "steps": n_e2e,
               "path": "attention_lab_b200.append_kvz + sparse_decode_step_kernel per layer, pinned host I/O on two "
                       "copy streams overlapping the compute"}

    # ---- same-box baselines (rank 0 reports its own): dense decode over the same caches
    baselines = None
    if not args.no_baselines and rank == 0:
        baselines = same_box_baselines(torch, al, Ks, Vs, Q, L, layers, B, stream, scale,
                                       sparse_inputs=(Zs, WQ, WK, QP, KPN, plan))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(args, B, G, h, L, rho, layers, args.cpu_seconds)

    if rank == 0:
        line = {"metric": metric_name(args.workload), "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": config_of(args, desc, B, G, h, L, rho, layers),
                "score_attend_us_per_layer": round(fused_ms * 1e3, 2), "append_us_per_layer": round(append_ms * 1e3, 2),
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": 2 * layers * args.steps,
                "clocks": clocks.summary(), "same_box": baselines}
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def same_box_baselines(torch, al, Ks, Vs, Q, L, layers, B, stream, scale, sparse_inputs=None):
    """Same-box baselines over the same caches: dense decode with torch SDPA, the h heads folded into the query axis
    (the reference's full_attention(backend="sdpa_fold"), full.py:31-34), this library's own dense kernel, and the
    reference's own sparse path run by torch on the GPU -- the operators of decode.py:145-163 (z column copy, u matmul,
    candidate matmul, torch.topk, cat with F, two index_selects, SDPA; decode.py:86-93,131-142, indexer.py:15-29)."""
    import torch.nn.functional as F
    out = {}

    def timed(fn, n=5):
        with torch.cuda.stream(stream):
            for _ in range(2):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n):
                fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def sdpa_fold():
        for l in range(layers):
            q = Q[l]
            b, g, h, _, d = q.shape
            F.scaled_dot_product_attention(q.view(b, g, h, d), Ks[l], Vs[l], scale=scale)

    def ours_dense():
        for l in range(layers):
            al.dense_decode_step(Q[l], Ks[l], Vs[l], L, scale=scale)

    try:
        ms = timed(sdpa_fold)
        out["torch_sdpa_fold_dense"] = {"tokens_per_s": round(B / (ms / 1e3), 2), "ms_per_step": round(ms, 3)}
    except RuntimeError as e:
        out["torch_sdpa_fold_dense"] = {"error": str(e)[:200]}
    ms = timed(ours_dense)
    out["ours_dense"] = {"tokens_per_s": round(B / (ms / 1e3), 2), "ms_per_step": round(ms, 3)}
    if sparse_inputs is not None:
        Zs, WQ, WK, QP, KPN, plan = sparse_inputs

        def torch_reference_sparse():
            for l in range(layers):
                q, zT = Q[l], Zs[l]
                b, g, h, _, d = q.shape
                wc = plan.write_col
                zT[..., wc:wc + 1].copy_(torch.matmul(WK[l].unsqueeze(0), KPN[l].transpose(-1, -2)))
                u = torch.matmul(QP[l].permute(0, 1, 3, 2, 4).reshape(b, g, 1, h * d), WQ[l].unsqueeze(0))
                top = torch.topk(torch.matmul(u, zT[..., plan.lo:plan.hi]), plan.k, dim=-1).indices.view(b, g, plan.k)
                rows = torch.cat([plan.fixed_rows, top + plan.off_lo], dim=-1).view(-1)
                S = plan.selected_count
                k_sub = Ks[l].view(-1, d).index_select(0, rows).view(b, g, S, d)
                v_sub = Vs[l].view(-1, d).index_select(0, rows).view(b, g, S, d)
                F.scaled_dot_product_attention(q.reshape(b, g, h, d), k_sub, v_sub, scale=scale)
        try:
            ms = timed(torch_reference_sparse)
            out["torch_reference_sparse_path"] = {"tokens_per_s": round(B / (ms / 1e3), 2), "ms_per_step": round(ms, 3)}
        except RuntimeError as e:
            out["torch_reference_sparse_path"] = {"error": str(e)[:200]}
    return out


if __name__ == "__main__":
    sys.exit(main())
