"""Decode-step benchmark: tokens/s and HBM GB/s of RoPE + KV-cache write +
paged attention over a ragged batch (Qwen2.5-3B-shaped: 64 sequences with
context U[128, 4096], 16 query / 2 KV heads, head_dim 128, block_size 16,
40k-block pool, bf16, RoPE theta 1e6), on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode step of one attention layer, for every sequence of the
batch: RoPE, the KV-cache write of the new token and paged attention, one
launch. Steps rotate over independent layers (own KV pool, tables, inputs), so
consecutive steps never find their KV in L2. With N GPUs (torchrun, one
process per GPU) the global batch is 64*N sequences drawn from the same
distribution and assigned to GPUs by LPT on context length; each GPU owns its
pool and metadata and no collective touches the data path (weak scaling).

Printed (rank 0, one JSON line): value = whole-job tokens/s from CUDA events
over the timed region (max over ranks), e2e = the same through the public op
API with inputs copied from pinned host memory every step and the output
read back, roofline of the attention kernel, the CPU oracle timed on this
host, clocks sampled during the timed region.

``--impl reference`` times the reference algorithm on the host cores (the
CPU oracle: the reference has no CPU kernels of its own for this path) on
bounded samples of the same workload, rank 0 only.
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

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "tinyllama.py_b200"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "decode-attention tokens/sec and HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
UNIT = "tokens/s"
WORKLOAD = "qwen2.5-3b decode step: 64 seqs/GPU, ctx U[128,4096], 16q/2kv heads, hd128, bs16, bf16"
LAYERS = 4           # default number of rotating independent KV pools
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU-baseline sample budget (rank 0, N=1)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-group", type=int, default=4,
                    help="e2e: consecutive steps whose inputs share one host-to-device copy "
                         "(rounded to a multiple of --layers; 4 measured best of 4, 8, 12)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="rotating independent KV pools per GPU (profiling runs use 1)")
    ap.add_argument("--workload", choices=["qwen3b", "long_tail", "ragged"], default="qwen3b",
                    help="qwen3b: the decode step (default); long_tail: 256 long-tailed "
                         "sequences LPT-split over the GPUs, ~150 GB pool each (strong "
                         "scaling); ragged: decode + prompt chunks with prefill attention, "
                         "1 GPU")
    ap.add_argument("--pool-gb", type=float, default=150.0,
                    help="long_tail: KV pool per GPU in GB")
    ap.add_argument("--sweep", action="store_true",
                    help="shape sweep (block size x batch x context x dtype x heads): one JSON "
                         "line per point with the attention kernel's rate and the CPU oracle's")
    ap.add_argument("--sweep-cpu-seconds", type=float, default=1.0,
                    help="CPU oracle budget per sweep point")
    return ap.parse_args()


# ------------------------------------------------------------------ setup
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def global_lengths(n_gpus: int, seed: int):
    from paged_decode import workloads as W

    return W.qwen3b_decode(seed, batch=64 * n_gpus).seq_lens


def lpt_balance(world: int, seed: int) -> float:
    """Largest GPU's context tokens over the mean: the ideal-bound factor of
    the weak-scaling split (1.0 = perfectly balanced)."""
    from paged_decode import partition as P

    lens = global_lengths(world, seed)
    loads = P.shard_loads(lens, P.lpt_assign(lens, world))
    return round(max(loads) / (sum(loads) / world), 4)


def rank_spec(rank: int, world: int, seed: int, layer: int):
    from paged_decode import partition as P
    from paged_decode import workloads as W

    lens = global_lengths(world, seed)
    shard = P.lpt_assign(lens, world)[rank]
    base = W.qwen3b_decode(seed)
    return W.DecodeSpec(base.name, [lens[i] for i in shard], base.num_heads, base.num_kv_heads,
                        base.head_dim, base.block_size, base.dtype, num_blocks=base.num_blocks,
                        rope_theta=base.rope_theta, max_position=base.max_position,
                        seed=seed * 1000 + rank * 10 + layer)


# --------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = devices
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        if visible:
            ids = [v.strip() for v in visible.split(",") if v.strip()]
            sel = ",".join(ids[d] for d in self.devices if d < len(ids))
        else:
            sel = ",".join(map(str, self.devices))
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", sel],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def prime(self, busy, timeout_s: float = 3.0) -> int:
        """Keep the GPU busy with `busy()` (untimed) until the sampler's first
        line arrives, so that short timed regions still get samples under load.
        Returns how many times `busy` ran."""
        n, t0 = 0, time.perf_counter()
        while self.proc is not None and not self.lines and time.perf_counter() - t0 < timeout_s:
            busy()
            n += 1
        return n

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- ours
def measured_hbm_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    """Dense bf16 tensor peak (TFLOP/s) measured on this pool, burst figure."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except (ValueError, KeyError):
            pass
    return 1590.0, "fallback"


def profiled_traffic(key: str):
    """DRAM bytes per attention launch from the committed ncu summary, if any."""
    p = REPO / "profiles" / "roofline_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(key + "="):
            try:
                return float(line.split("=", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def run_ours(args, rank, world, local):
    import torch.distributed as dist

    from cscr import attention as A
    from paged_decode import roofline as R
    from paged_decode import workloads as W

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    nl = args.layers
    layers = [W.make_batch(rank_spec(rank, world, args.seed, l), device=dev) for l in range(nl)]
    spec0 = layers[0].spec
    S, H, KVH, D = len(spec0.seq_lens), spec0.num_heads, spec0.num_kv_heads, spec0.head_dim
    stream = torch.cuda.Stream(dev)

    def step(b):
        # One launch per step: RoPE of the new tokens, their KV-cache write
        # and paged attention (the decode batch's new token of sequence s is
        # at position seq_lens[s] - 1). Layers run back to back; the previous
        # launch writes no metadata this one reads before its dependency wait.
        return A.paged_attention_with_rope(b.query, b.key.view(S, KVH * D), b.value,
                                           b.key_cache, b.value_cache, b.block_tables,
                                           b.seq_lens, b.cos_sin_cache, b.scale,
                                           overlap_prologue=True)

    def attn_only(b):
        return A.paged_attention(b.query, b.key_cache, b.value_cache, b.block_tables,
                                 b.seq_lens, b.scale)

    with torch.cuda.stream(stream):
        for b in layers:  # warm: workspace, attributes, tensor maps
            step(b)
            attn_only(b)
        stream.synchronize()
        g_step, g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=stream):
            for b in layers:
                step(b)
        with torch.cuda.graph(g_attn, stream=stream):
            for b in layers:
                attn_only(b)

    # Exactly K timed steps: K // nl replays of the nl-layer graph, then the
    # remaining K % nl steps launched directly; exactly W warm-up steps.
    steps = max(1, args.steps)
    reps, rest = divmod(steps, nl)
    warm = max(0, args.warmup)

    def timed(graph, fn, n_reps, n_rest):
        with torch.cuda.stream(stream):
            for i in range(warm):
                fn(layers[i % nl])
        stream.synchronize()
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(n_reps):
                graph.replay()
            for i in range(n_rest):
                fn(layers[i])
            e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        own = e0.elapsed_time(e1)
        ms = own
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms, own

    devices = list(range(world)) if world > 1 else [local]
    # clocks: sampled from before the warm-up to the end of the e2e leg
    sampler = ClockSampler(devices) if rank == 0 else None
    primed = 0
    if sampler:
        sampler.__enter__()

        def busy():
            with torch.cuda.stream(stream):
                for _ in range(50):
                    g_step.replay()
            stream.synchronize()

        primed = sampler.prime(busy) * 50 * nl
    step_ms, own_step_ms = timed(g_step, step, reps, rest)
    attn_ms, _ = timed(g_attn, attn_only, reps, rest)

    # spread: 20 samples of the step, each over a slice of the replays
    nsamp = 20
    per = max(1, max(reps, 1) // nsamp)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(nsamp + 1)]
    with torch.cuda.stream(stream):
        evs[0].record(stream)
        for i in range(nsamp):
            for _ in range(per):
                g_step.replay()
            evs[i + 1].record(stream)
    torch.cuda.synchronize(dev)
    samp = torch.tensor([evs[i].elapsed_time(evs[i + 1]) * 1e3 / (per * nl) for i in range(nsamp)],
                        dtype=torch.float64)
    if world > 1:
        samp = samp.to(dev)
        dist.all_reduce(samp, op=dist.ReduceOp.MAX)
        samp = samp.cpu()
    q10, q50, q90 = (float(torch.quantile(samp, q)) for q in (0.1, 0.5, 0.9))

    # ---- end to end through the public ops, host buffers each step
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, layers, step, stream, dev, world, barrier, rank)
        e2e["eager"] = run_e2e_eager(args, layers, dev, world, barrier)
    if sampler:
        sampler.__exit__(None, None, None)

    tokens_per_step = 64 * world
    value = tokens_per_step * steps / (step_ms / 1e3)
    lens_all = [b.seq_lens.cpu().numpy() for b in layers]
    attn_bytes = statistics.fmean(
        R.attention_bytes(l, spec0.block_size, H, KVH, D, 2) for l in lens_all)
    rope_bytes = R.rope_bytes(S, H, KVH, D, D, 2) + R.cache_write_bytes(S, KVH, D, 2)
    # every rank's own step time and bytes: what limits the N-GPU curve
    mine = torch.tensor([own_step_ms * 1e3 / steps, attn_bytes + rope_bytes,
                         float(sum(int(l.sum()) for l in lens_all) / nl)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
    else:
        gathered = [mine]
    per_rank = [{"rank": r, "us_per_step": round(float(g[0]), 3),
                 "bytes_per_step": int(g[1]), "context_tokens": int(g[2]),
                 "gbs": round(float(g[1]) / (float(g[0]) * 1e-6) / 1e9, 1)}
                for r, g in enumerate(x.cpu() for x in gathered)]
    t_attn_us = attn_ms * 1e3 / steps
    t_step_us = step_ms * 1e3 / steps
    # the step is one launch of the fused kernel: its bytes over its time
    achieved = (attn_bytes + rope_bytes) / (t_step_us * 1e-6) / 1e9
    peak, peak_kind = measured_hbm_peak()
    traffic = profiled_traffic("qwen3b_decode_attention_bytes_per_launch")

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": round(step_ms / steps, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v and KV pool, seeded lengths)",
        "config": {"workload": WORKLOAD, "global_batch": tokens_per_step, "seq_len": "U[128,4096]",
                   "parallelism": f"sequence-sharded x{world} (LPT), no collective",
                   "lpt_max_load_over_mean": lpt_balance(world, args.seed),
                   "l2": f"{nl} rotating independent KV pools per GPU "
                         f"(~{nl * attn_bytes / 1e6:.0f} MB of KV per rotation > 126 MB L2)",
                   "timed_region": "CUDA-graph replay of the decode step: RoPE + KV-cache write "
                                   "+ paged attention in one launch per layer",
                   "clock_priming_steps": primed},
        "hbm_gbs_step": round((attn_bytes + rope_bytes) / (t_step_us * 1e-6) / 1e9, 1),
        "hbm_frac_of_8tbs_step": round((attn_bytes + rope_bytes) / (t_step_us * 1e-6) / 1e9
                                       / NOMINAL_HBM_GBS, 4),
        "roofline": {"kernel": "paged_attention_tc_kernel (fused RoPE + cache write)",
                     "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                     "algorithmic_bytes_per_launch": int(attn_bytes + rope_bytes),
                     "launch_us": round(t_step_us, 3),
                     "traffic": traffic},
        "attention_only": {"launch_us": round(t_attn_us, 3),
                           "achieved_gbs": round(attn_bytes / (t_attn_us * 1e-6) / 1e9, 1),
                           "note": "paged_attention alone (query already rotated), graph of "
                                   "back-to-back launches without programmatic overlap"},
        "step_us_p10_p50_p90": [round(q10, 3), round(q50, 3), round(q90, 3)],
        "gpu_launches": steps * world,
        "gpu_launches_per_rank": steps,
        "per_rank": per_rank,
        "clocks": sampler.summary() if sampler else None,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if world == 1:
        line["cpu_baseline"] = cpu_baseline(layers[0], args.cpu_seconds)
    return line


def pack_layout(S, H, KVH, D, maxB):
    """Byte offsets of one step's inputs in a single host/device buffer."""
    segs = [("query", S * H * D * 2), ("key", S * KVH * D * 2), ("value", S * KVH * D * 2),
            ("tables", S * maxB * 4), ("lens", S * 4)]
    off, out = 0, {}
    for name, n in segs:
        out[name] = (off, n)
        off += (n + 255) // 256 * 256
    return out, off


def run_e2e(args, layers, step_fn, stream, dev, world, barrier, rank):
    """Same steps through the op API with pinned-host inputs and a host read-back."""
    import torch.distributed as dist

    from cscr import attention as A

    spec0 = layers[0].spec
    S, H, KVH, D = len(spec0.seq_lens), spec0.num_heads, spec0.num_kv_heads, spec0.head_dim
    maxB = max(b.block_tables.shape[1] for b in layers)
    layout, total = pack_layout(S, H, KVH, D, maxB)
    nl = len(layers)
    # A group of gs consecutive steps (a multiple of nl: step j of a group
    # runs layer j % nl): its inputs back to back in one pinned host buffer,
    # and two device staging banks of the same size.
    gs = nl * max(1, getattr(args, "e2e_group", 4) // nl)
    host = torch.zeros(gs * total, dtype=torch.uint8).pin_memory()
    for j in range(gs):
        b = layers[j % nl]
        h = host[j * total:(j + 1) * total]

        def put(name, t):
            o, n = layout[name]
            h[o:o + n].copy_(t.contiguous().view(torch.uint8).view(-1).cpu())

        bt = torch.zeros(S, maxB, dtype=torch.int32)
        bt[:, : b.block_tables.shape[1]] = b.block_tables.cpu()
        put("query", b.query); put("key", b.key); put("value", b.value)
        put("tables", bt); put("lens", b.seq_lens)
    banks = torch.empty(2, gs * total, dtype=torch.uint8, device=dev)

    def views_of(bank, r):
        d = banks[bank, r * total:(r + 1) * total]

        def view(name, dtype, shape):
            o, n = layout[name]
            return d[o:o + n].view(dtype).view(*shape)

        return dict(query=view("query", torch.bfloat16, (S, H, D)),
                    key=view("key", torch.bfloat16, (S, KVH * D)),
                    value=view("value", torch.bfloat16, (S, KVH, D)),
                    tables=view("tables", torch.int32, (S, maxB)),
                    lens=view("lens", torch.int32, (S,)))

    views = [[views_of(k, j) for j in range(gs)] for k in range(2)]
    # A decode pass as a serving engine runs it: the public-API calls of a
    # 36-layer model's pass (Qwen2.5-3B has 36 layers) captured once into a
    # CUDA graph. The steps go in groups of gs consecutive steps: one pinned
    # host-to-device copy brings a group's inputs into a staging bank (two
    # banks, so a group's copy overlaps the previous group's compute), the
    # group's steps run back to back with programmatic overlap (each kernel
    # reads only its context lengths and block tables - which the copy, a full
    # dependency, wrote - before it waits for the kernel ahead of it), and
    # the group's outputs are read back on their own stream while the next
    # group computes. Every step's inputs and output cross PCIe every replay.
    groups = -(-36 // gs)
    per_graph = groups * gs
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    outs = [torch.empty(S, H, D, dtype=torch.bfloat16).pin_memory() for _ in range(per_graph)]

    def steps_block():
        fork = torch.cuda.Event()
        fork.record(stream)
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        done = []
        for gi in range(groups):
            bank = gi % 2
            ready = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                if gi >= 2:
                    s_in.wait_event(done[gi - 2])  # the bank's previous readers finished
                banks[bank].copy_(host, non_blocking=True)
                ready.record(s_in)
            stream.wait_event(ready)
            produced = []
            for j in range(gs):
                b, v = layers[j % nl], views[bank][j]
                produced.append(A.paged_attention_with_rope(
                    v["query"], v["key"], v["value"], b.key_cache, b.value_cache, v["tables"],
                    v["lens"], b.cos_sin_cache, b.scale, overlap_prologue=True))
            ev = torch.cuda.Event()
            ev.record(stream)
            done.append(ev)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                for j, out in enumerate(produced):
                    outs[gi * gs + j].copy_(out, non_blocking=True)
        join_in, join_out = torch.cuda.Event(), torch.cuda.Event()
        join_in.record(s_in)
        join_out.record(s_out)
        stream.wait_event(join_in)
        stream.wait_event(join_out)

    reps = max(1, (args.steps // 4) // per_graph)
    steps = reps * per_graph
    with torch.cuda.stream(stream):
        banks[0].copy_(host)
        banks[1].copy_(host)
        steps_block()  # warm: workspaces, tensor maps
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            steps_block()
        for _ in range(max(args.warmup, 1)):
            g.replay()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    del g
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return {"value": round(S * world * steps / (ms / 1e3), 1), "unit": UNIT,
            "h2d_bytes_per_step": int(total), "d2h_bytes_per_step": int(S * H * D * 2),
            "steps": steps,
            "path": "cscr.attention.paged_attention_with_rope (RoPE + cache write + attention, "
                    "overlap_prologue=True), per step its inputs host-to-device from pinned memory "
                    f"(one copy per group of {gs} consecutive steps, double-buffered) and its "
                    f"output device-to-host, copies on their own streams; {per_graph} steps "
                    "(a 36-layer decode pass, rounded up to whole groups) per CUDA-graph replay"}


def run_e2e_eager(args, layers, dev, world, barrier):
    """The same steps through the public op, launched one by one from Python
    (no CUDA graph): per step one pinned host-to-device copy of that step's
    inputs, the op, and a device-to-host copy of its output, all on one
    stream. Includes the per-call host cost (argument checks, ctypes) that a
    caller who does not capture graphs pays."""
    import torch.distributed as dist

    from cscr import attention as A

    spec0 = layers[0].spec
    S, H, KVH, D = len(spec0.seq_lens), spec0.num_heads, spec0.num_kv_heads, spec0.head_dim
    maxB = max(b.block_tables.shape[1] for b in layers)
    layout, total = pack_layout(S, H, KVH, D, maxB)
    nl = len(layers)
    hosts = []
    for b in layers:
        h = torch.zeros(total, dtype=torch.uint8).pin_memory()

        def put(name, t):
            o, n = layout[name]
            h[o:o + n].copy_(t.contiguous().view(torch.uint8).view(-1).cpu())

        bt = torch.zeros(S, maxB, dtype=torch.int32)
        bt[:, : b.block_tables.shape[1]] = b.block_tables.cpu()
        put("query", b.query); put("key", b.key); put("value", b.value)
        put("tables", bt); put("lens", b.seq_lens)
        hosts.append(h)
    d = torch.empty(total, dtype=torch.uint8, device=dev)

    def view(name, dtype, shape):
        o, n = layout[name]
        return d[o:o + n].view(dtype).view(*shape)

    q, k = view("query", torch.bfloat16, (S, H, D)), view("key", torch.bfloat16, (S, KVH * D))
    v, t = view("value", torch.bfloat16, (S, KVH, D)), view("tables", torch.int32, (S, maxB))
    lens = view("lens", torch.int32, (S,))
    out_h = torch.empty(S, H, D, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.current_stream(dev)

    def one(i):
        b = layers[i % nl]
        d.copy_(hosts[i % nl], non_blocking=True)
        out = A.paged_attention_with_rope(q, k, v, b.key_cache, b.value_cache, t, lens,
                                          b.cos_sin_cache, b.scale)
        out_h.copy_(out, non_blocking=True)

    n = max(1, min(args.steps, 2000))
    for i in range(max(args.warmup, 1)):
        one(i)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        one(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = tt.item()
    return {"value": round(S * world * n / (ms / 1e3), 1), "unit": UNIT, "steps": n,
            "h2d_bytes_per_step": int(total), "d2h_bytes_per_step": int(S * H * D * 2),
            "us_per_step": round(ms * 1e3 / n, 2),
            "path": "cscr.attention.paged_attention_with_rope called from Python once per step, "
                    "no CUDA graph; per step one pinned H2D copy of its inputs and a D2H copy "
                    "of its output on the same stream"}


# -------------------------------------------------- long-tail (config 4)
LONG_TAIL = ("long-tail decode step: 256 seqs in all, ctx clip(32*(1+pareto(1.2)), 32, 32768), "
             "16q/2kv heads, hd128, bs32, bf16, ~150 GB pool per GPU")


def _timed_graph(graph, stream, dev, reps, warm, world, barrier):
    """Device time of `reps` replays after `warm` untimed ones: (max over
    ranks, this rank's own)."""
    import torch.distributed as dist

    with torch.cuda.stream(stream):
        for _ in range(warm):
            graph.replay()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    own = e0.elapsed_time(e1)
    ms = own
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms, own


def run_long_tail(args, rank, world, local):
    """Config 4: one global batch of 256 long-tailed sequences, LPT-split over
    the GPUs (strong scaling), each GPU with a ~150 GB block pool; per step the
    fused decode step of every sequence (RoPE + cache write + attention).
    Steps rotate over 4 disjoint block sets of the pool (> 126 MB of KV per
    rotation), so no step finds its KV in L2."""
    import torch.distributed as dist

    from cscr import attention as A
    from paged_decode import partition as Pn
    from paged_decode import pool as Pool
    from paged_decode import roofline as R
    from paged_decode import workloads as W

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    lens = W.long_tail_lengths(args.seed, batch=256)
    shards = Pn.lpt_assign(lens, world)
    mine = [lens[i] for i in shards[rank]]
    H, KVH, D, bs = 16, 2, 128, 32
    budget = int(args.pool_gb * 1e9)
    NB = Pool.blocks_for_budget(budget, 1, KVH, D, bs, torch.bfloat16)
    (kc, vc), = Pool.allocate_kv_cache(1, NB, KVH, D, bs, torch.bfloat16, device=dev)
    nl = args.layers
    layers = [W.make_batch(W.DecodeSpec("long_tail", mine, H, KVH, D, bs, "bfloat16",
                                        num_blocks=NB, max_position=32768,
                                        seed=args.seed * 1000 + rank * 10 + l),
                           device=dev, caches=(kc, vc)) for l in range(nl)]
    S = len(mine)
    stream = torch.cuda.Stream(dev)

    def step(b):
        return A.paged_attention_with_rope(b.query, b.key.view(S, KVH * D), b.value,
                                           b.key_cache, b.value_cache, b.block_tables,
                                           b.seq_lens, b.cos_sin_cache, b.scale,
                                           overlap_prologue=True)

    with torch.cuda.stream(stream):
        for b in layers:
            step(b)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for b in layers:
                step(b)
    reps = max(1, args.steps // nl)
    steps = reps * nl
    ms, own = _timed_graph(g, stream, dev, reps, max(1, math.ceil(args.warmup / nl)), world,
                           barrier)
    per_step_bytes = statistics.fmean(
        R.attention_bytes(b.seq_lens.cpu().numpy(), bs, H, KVH, D, 2) for b in layers) + \
        R.rope_bytes(S, H, KVH, D, D, 2) + R.cache_write_bytes(S, KVH, D, 2)
    mine_t = torch.tensor([own * 1e3 / steps, per_step_bytes, float(sum(mine)), float(S)],
                          dtype=torch.float64, device=dev)
    if world > 1:
        gathered = [torch.empty_like(mine_t) for _ in range(world)]
        dist.all_gather(gathered, mine_t)
    else:
        gathered = [mine_t]
    del g
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    per_rank = [{"rank": r, "seqs": int(x[3]), "context_tokens": int(x[2]),
                 "us_per_step": round(float(x[0]), 3), "bytes_per_step": int(x[1]),
                 "gbs": round(float(x[1]) / (float(x[0]) * 1e-6) / 1e9, 1)}
                for r, x in enumerate(t.cpu() for t in gathered)]
    peak, peak_kind = measured_hbm_peak()
    total_bytes = sum(pr["bytes_per_step"] for pr in per_rank)
    t_step = ms * 1e3 / steps
    bound_tokens = Pn.makespan_bound(lens, world)
    return {
        "metric": METRIC, "value": round(256 * steps / (ms / 1e3), 1), "unit": UNIT,
        "n_gpus": world, "steps": steps, "warmup": max(1, math.ceil(args.warmup / nl)) * nl,
        "ms_per_step": round(ms / steps, 6), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v and KV blocks, seeded Pareto lengths)",
        "config": {"workload": LONG_TAIL, "global_batch": 256, "seq_len": "Pareto(1.2) x 32, "
                   "clipped to [32, 32768]", "parallelism": f"sequence-sharded x{world} (LPT), "
                   "no collective", "pool_blocks_per_gpu": NB,
                   "pool_gb_per_gpu": round(2 * NB * KVH * bs * D * 2 / 1e9, 1),
                   "l2": f"{nl} disjoint block sets of the pool rotate"},
        "per_rank": per_rank,
        "bound": {"max_context": int(max(lens)), "sum_context": int(sum(lens)),
                  "makespan_bound_tokens": bound_tokens,
                  "max_rank_tokens": max(pr["context_tokens"] for pr in per_rank),
                  "efficiency_tokens": round(sum(lens) / world / max(
                      pr["context_tokens"] for pr in per_rank), 4),
                  "efficiency_bytes": round(total_bytes / world / max(
                      pr["bytes_per_step"] for pr in per_rank), 4)},
        "hbm_gbs_per_gpu_mean": round(total_bytes / world / (t_step * 1e-6) / 1e9, 1),
        "frac_of_measured_peak_per_gpu": round(total_bytes / world / (t_step * 1e-6) / 1e9
                                               / peak, 4),
        "peak_kind": peak_kind,
        "gpu_launches": steps * world,
    }


# ------------------------------------------------ ragged step (config 3)
RAGGED = ("continuous-batching step: 252 decode seqs (ctx lognormal median 1024, sigma 1, "
          "clip [16, 8192]) + 4 prompt chunks U[256, 2048], 16q/2kv heads, hd128, bs16, fp16")


def run_ragged(args, local):
    """Config 3 on one GPU: per step RoPE + cache write of every packed token
    (~4.9k), decode attention of the 252 decode sequences and causal prefill
    attention of the 4 prompt chunks; positions and slots built on the device
    from the block tables. Kernels timed alone and as the whole step."""
    from cscr import attention as A
    from cscr import pos_encoding as PE
    from paged_decode import roofline as R
    from paged_decode import workloads as W

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    nl = args.layers
    layers = [W.make_batch(W.ragged_batch(args.seed + 7 * l), device=dev) for l in range(nl)]
    H, KVH, D = 16, 2, 128
    stream = torch.cuda.Stream(dev)
    prep = []
    for b in layers:
        T = b.query.shape[0]
        npt = b.num_prompt_tokens
        lens = b.spec.prefill_lens
        starts = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        tables = torch.stack([b.token_block_tables[int(starts[c])] for c in range(len(lens))])
        prep.append(dict(T=T, npt=npt, tables=tables.contiguous(), maxq=int(max(lens)),
                         qs=torch.from_numpy(starts).to(dev),
                         ctx=torch.tensor(lens, dtype=torch.int32, device=dev),
                         out=torch.empty(T, H, D, dtype=torch.float16, device=dev)))

    def rope(b, x):
        return PE.rotary_embedding_neox_with_cache(b.positions, b.query.view(x["T"], -1),
                                                   b.key.view(x["T"], -1), b.value,
                                                   b.key_cache, b.value_cache, b.slot_mapping,
                                                   D, b.cos_sin_cache)

    def decode(b, x, q):
        return A.paged_attention(q[x["npt"]:], b.key_cache, b.value_cache, b.block_tables,
                                 b.seq_lens, b.scale)

    def prefill(b, x, q):
        return A.paged_prefill_attention(q[:x["npt"]], b.key_cache, b.value_cache, x["tables"],
                                         x["qs"], x["ctx"], b.scale, max_query_len=x["maxq"],
                                         out=x["out"][:x["npt"]])

    qrot = [rope(b, x).view(x["T"], H, D) for b, x in zip(layers, prep)]  # warm + inputs
    legs = {
        "rope_cache_write": lambda i: rope(layers[i], prep[i]),
        "decode_attention": lambda i: decode(layers[i], prep[i], qrot[i]),
        "prefill_attention": lambda i: prefill(layers[i], prep[i], qrot[i]),
        "step": lambda i: (lambda q: (decode(layers[i], prep[i], q),
                                      prefill(layers[i], prep[i], q)))(
            rope(layers[i], prep[i]).view(prep[i]["T"], H, D)),
    }
    times = {}
    reps = max(1, args.steps // nl)
    for name, fn in legs.items():
        with torch.cuda.stream(stream):
            for i in range(nl):
                fn(i)
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(nl):
                    fn(i)
        ms, _ = _timed_graph(g, stream, dev, reps, 3, 1, lambda: None)
        times[name] = ms * 1e3 / (reps * nl)
        del g
    lens_dec = [b.seq_lens.cpu().numpy() for b in layers]
    dec_bytes = statistics.fmean(R.attention_bytes(l, 16, H, KVH, D, 2) for l in lens_dec)
    T_mean = statistics.fmean(x["T"] for x in prep)
    rope_b = R.rope_bytes(T_mean, H, KVH, D, D, 2) + R.cache_write_bytes(T_mean, KVH, D, 2)
    pre_flops = statistics.fmean(
        sum(4 * H * D * n * (n + 1) / 2 for n in b.spec.prefill_lens) for b in layers)
    peak, peak_kind = measured_hbm_peak()
    tflops_peak = measured_tensor_peak()
    n_dec = len(lens_dec[0])
    return {
        "metric": METRIC, "value": round(n_dec / (times["step"] * 1e-6), 1), "unit": UNIT,
        "n_gpus": 1, "steps": reps * nl, "warmup": 3 * nl, "ms_per_step": round(
            times["step"] / 1e3, 6), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) q/k/v and KV pool, seeded lengths)",
        "config": {"workload": RAGGED, "decode_seqs": n_dec, "packed_tokens": round(T_mean),
                   "l2": f"{nl} rotating independent pools",
                   "value_is": "decode tokens per second of the whole step (RoPE + cache "
                               "write of all tokens, decode and prefill attention)"},
        "us": {k: round(v, 3) for k, v in times.items()},
        "roofline": {
            "rope_cache_write": {"bound": "hbm", "bytes": int(rope_b), "achieved": round(
                rope_b / (times["rope_cache_write"] * 1e-6) / 1e9, 1), "unit": "GB/s",
                "frac": round(rope_b / (times["rope_cache_write"] * 1e-6) / 1e9 / peak, 4)},
            "decode_attention": {"bound": "hbm", "bytes": int(dec_bytes), "achieved": round(
                dec_bytes / (times["decode_attention"] * 1e-6) / 1e9, 1), "unit": "GB/s",
                "frac": round(dec_bytes / (times["decode_attention"] * 1e-6) / 1e9 / peak, 4)},
            "prefill_attention": {"bound": "tensor", "flops": int(pre_flops), "achieved": round(
                pre_flops / (times["prefill_attention"] * 1e-6) / 1e12, 1), "unit": "TFLOP/s",
                "frac": round(pre_flops / (times["prefill_attention"] * 1e-6) / 1e12
                              / tflops_peak[0], 4), "peak": tflops_peak[0],
                "peak_kind": tflops_peak[1]},
            "hbm_peak": peak, "hbm_peak_kind": peak_kind},
        "gpu_launches": 3 * reps * nl,
    }


# ------------------------------------------------------------ CPU side
def oracle_inputs(batch):
    """Host copies of one layer's decode step, pool cut to the blocks it uses."""
    from paged_decode import workloads as W

    kc, vc, tables, lens = W.compact_for_oracle(batch)
    S = batch.num_decode
    pos = batch.positions.cpu().numpy()
    # the new token's slot, renumbered into the compacted pool
    bs = batch.spec.block_size
    slots = np.array([tables[s, pos[s] // bs] * bs + pos[s] % bs for s in range(S)], np.int64)
    return dict(q=W.to_numpy(batch.query.view(S, -1)), k=W.to_numpy(batch.key.view(S, -1)),
                v=W.to_numpy(batch.value), pos=pos, slots=slots, tables=tables, lens=lens,
                kc=kc, vc=vc, cs=W.to_numpy(batch.cos_sin_cache), scale=batch.scale,
                H=batch.spec.num_heads, D=batch.spec.head_dim)


def oracle_step(inp, seqs, threads):
    """The reference algorithm for a subset of sequences: RoPE, KV write, attention."""
    from oracle import decode_oracle as O

    idx = np.asarray(seqs)
    q_rot, k_rot = O.rotary_embedding_neox(inp["pos"][idx], inp["q"][idx], inp["k"][idx],
                                           inp["D"], inp["cs"], "bfloat16")
    O.reshape_and_cache(k_rot, inp["v"][idx], inp["kc"], inp["vc"], inp["slots"][idx])
    return O.paged_attention_threads(q_rot.reshape(len(idx), inp["H"], inp["D"]), inp["kc"],
                                     inp["vc"], inp["tables"][idx], inp["lens"][idx],
                                     inp["scale"], "bfloat16", threads)


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(batch, seconds):
    cores = os.cpu_count() or 1
    inp = oracle_inputs(batch)
    S = len(inp["lens"])
    chunk = min(S, cores)
    done, t0, i = 0, time.perf_counter(), 0
    while True:
        seqs = [(i * chunk + j) % S for j in range(chunk)]
        oracle_step(inp, seqs, cores)
        done += chunk
        i += 1
        el = time.perf_counter() - t0
        if el >= seconds and done >= S:
            break
    return {"value": round(done / el, 2), "unit": UNIT, "cores": cores, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"CPU oracle (numpy, {cores} threads) over {done} sequences of the same "
                      f"workload in chunks of {chunk}, {el:.1f} s"}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from paged_decode import workloads as W

    batch = W.make_batch(rank_spec(0, 1, args.seed, 0), device="cpu")
    inp = oracle_inputs(batch)
    cores = os.cpu_count() or 1
    S = len(inp["lens"])
    chunk = min(S, cores)
    for i in range(args.warmup):
        oracle_step(inp, [(i * chunk + j) % S for j in range(chunk)], cores)
    t0 = time.perf_counter()
    for i in range(args.steps):
        oracle_step(inp, [(i * chunk + j) % S for j in range(chunk)], cores)
    el = time.perf_counter() - t0
    value = chunk * args.steps / el
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v and KV pool, seeded lengths)",
        "config": {"workload": WORKLOAD, "global_batch": 64,
                   "sample_per_step": f"{chunk} of the 64 sequences (rotating)"},
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"each step: RoPE + cache write + attention of {chunk} "
                                   f"sequences, CPU oracle (numpy, {cores} threads)"},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_sweep(args, rank, world, local):
    """Attention over each sweep shape: 1..N GPUs, LPT-sharded batch, one line per point."""
    import torch.distributed as dist

    from cscr import attention as A
    from paged_decode import partition as Pn
    from paged_decode import roofline as R
    from paged_decode import workloads as W

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))
    peak, peak_kind = measured_hbm_peak()
    for spec in W.sweep_points():
        # batch of the point per GPU (weak scaling), LPT split of the global batch
        glob = spec.seq_lens * world
        mine = [glob[i] for i in Pn.lpt_assign(glob, world)[rank]]
        local_spec = W.DecodeSpec(spec.name, mine, spec.num_heads, spec.num_kv_heads,
                                  spec.head_dim, spec.block_size, spec.dtype,
                                  seed=spec.seed + rank)
        # enough independent pools that one pass over them exceeds twice the
        # 126 MB L2, so every launch reads its KV from HBM
        e = 2 if spec.dtype != "float32" else 4
        per_layer = R.attention_bytes(mine, spec.block_size, spec.num_heads, spec.num_kv_heads,
                                      spec.head_dim, e)
        nl = int(min(64, max(2, math.ceil(300e6 / max(per_layer, 1)))))
        layers = [W.make_batch(W.DecodeSpec(**{**local_spec.__dict__, "seed": local_spec.seed + 7 * l}),
                               device=dev) for l in range(nl)]
        stream = torch.cuda.Stream(dev)

        def attn():
            for b in layers:
                A.paged_attention(b.query, b.key_cache, b.value_cache, b.block_tables,
                                  b.seq_lens, b.scale)

        with torch.cuda.stream(stream):
            attn()
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                attn()
            for _ in range(3):
                g.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        reps = max(5, 200 // nl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / (reps * len(layers))
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        byt = per_layer
        line = {"point": spec.name, "pools": nl, "n_gpus": world, "tokens_per_s": round(len(glob) / (ms / 1e3), 1),
                "us_per_launch": round(ms * 1e3, 2),
                "hbm_gbs_per_gpu": round(byt / (ms / 1e3) / 1e9, 1),
                "frac_of_measured_peak": round(byt / (ms / 1e3) / 1e9 / peak, 4),
                "peak_kind": peak_kind}
        if rank == 0 and world == 1 and args.sweep_cpu_seconds > 0:
            line["cpu_oracle_tokens_per_s"] = sweep_cpu(layers[0], args.sweep_cpu_seconds)
        if rank == 0:
            print(json.dumps(line), flush=True)
        del layers, g
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()


def sweep_cpu(batch, seconds):
    """Reference attention (CPU oracle, all host threads) on a bounded sample."""
    from oracle import decode_oracle as O
    from paged_decode import workloads as W

    S = batch.num_decode
    take = list(range(min(S, os.cpu_count() or 1)))
    sub = W.DecodeBatch(**{**batch.__dict__})
    sub.block_tables = batch.block_tables[take]
    sub.seq_lens = batch.seq_lens[take]
    kc, vc, tables, lens = W.compact_for_oracle(sub)
    q = W.to_numpy(batch.query[take])
    done, t0 = 0, time.perf_counter()
    while True:
        O.paged_attention_threads(q, kc, vc, tables, lens, batch.scale, batch.spec.dtype)
        done += len(take)
        if time.perf_counter() - t0 >= seconds:
            break
    return round(done / (time.perf_counter() - t0), 2)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.sweep:
        run_sweep(args, rank, world, local)
        return
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(json.dumps({"error": "launch with torchrun for --gpus > 1"}))
        sys.exit(2)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    elif args.workload == "long_tail":
        line = run_long_tail(args, rank, world, local)
    elif args.workload == "ragged":
        line = run_ragged(args, local) if rank == 0 else None
    else:
        line = run_ours(args, rank, world, local)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
