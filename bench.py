"""Benchmark of the B200 attention forward (headline: causal GQA prefill, C2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload ("C2"): causal GQA prefill,
B=4, Hq=32, Hkv=8 (G=4), S=4096, D=128, BSHD layout, bf16 in / fp32 accumulate,
Q/K/V ~ N(0,1) from seed 42 (synthetic; no dataset).  A step is one forward
over that batch.  Metric: TFLOP/s with the FA/SDPA causal count
4*B*Hq*S^2*D/2 = 5.498e11 FLOP per step.

Timing: W untimed warm-up steps, then K timed steps between a barrier +
synchronize on both sides.  Before every step a 256 MiB buffer is written to
flush L2; each step is bracketed by CUDA events on the launching stream (the
flush is outside the event pair).  ``value`` = FLOPs of all ranks / max over
ranks of the summed step times.  ``e2e`` repeats the step through the public
API with pinned host buffers: H2D of Q, K, V, the forward, D2H of O and LSE.

Multi-GPU (torchrun, one rank per GPU, NCCL): the work shards by
(batch x KV-head group) with no collective on the data path; every rank runs
its own B=4 shard (weak scaling, global batch 4N).

``--impl reference`` times the reference's own CPU path for this workload
(torch SDPA with enable_gqa, base/baseline_gqa_causal.py:61-65, restated in
oracle/attention_oracle.py:sdpa_cpu) on the host cores, one bounded sample
per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

C2 = dict(B=4, Hq=32, Hkv=8, S=4096, D=128)
METRIC = "GQA fwd TFLOP/s/GPU & % BF16 tensor peak; split-KV decode HBM GB/s & % peak"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def causal_flops(B, Hq, S, D):
    return 4.0 * B * Hq * S * S * D / 2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM traffic recorded from an ncu capture in profiles/<name>."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        mhz, maxmhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm, mx, pw = float(r[0]), float(r[1]), float(r[2])
            except (ValueError, IndexError):
                continue
            maxmhz = mx
            if pw > 200:  # under load
                mhz.append(sm)
            for n, v in zip(names, r[4:8]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": maxmhz,
                "reasons": sorted(reasons), "samples_under_load": len(mhz)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def c2_config(world):
    """The workload description both arms report (the C2 configuration)."""
    B, Hq, Hkv, S, D = (C2[k] for k in ("B", "Hq", "Hkv", "S", "D"))
    return {"workload": "C2 causal GQA prefill (Llama-3-8B attention shape)", "entry": "bw_gqa_causal_fwd",
            "batch_total": B * world, "batch_per_gpu": B, "seq_len": S, "heads_q": Hq, "heads_kv": Hkv,
            "head_dim": D, "layout": "BSHD",
            "parallelism": f"shard by batch x KV-group, {world} rank(s), no collective",
            "l2": "256 MiB buffer written before every step, outside the event pair",
            "flops_per_step": causal_flops(B, Hq, S, D) * world, "flop_count": "4*B*Hq*S^2*D/2"}


# ---------------------------------------------------------------- CPU path
def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def median_rate(work, times):
    """work / median(seconds): the statistic both arms and every CPU leg use."""
    return work / statistics.median(times)


class CpuReference:
    """The reference's CPU path (torch SDPA, enable_gqa, causal) on one (b, KV-group)
    slice of C2: G=4 query heads x S=4096 x D=128, bf16, all host cores."""

    def __init__(self):
        from oracle.attention_oracle import sdpa_cpu
        self.fn = sdpa_cpu
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        G, S, D = C2["Hq"] // C2["Hkv"], C2["S"], C2["D"]
        g = torch.Generator().manual_seed(42)
        self.q = torch.randn(1, G, S, D, generator=g).bfloat16()
        self.k = torch.randn(1, 1, S, D, generator=g).bfloat16()
        self.v = torch.randn(1, 1, S, D, generator=g).bfloat16()
        self.scale = 1 / math.sqrt(D)
        self.flops = causal_flops(1, G, S, D)
        self.sample = f"1 (b, KV-group) slice of C2 = {G} heads x S={S} x D={D} bf16 causal per step"

    def step(self):
        """Seconds for one sample."""
        t0 = time.perf_counter()
        self.fn(self.q, self.k, self.v, self.scale, causal=True)
        return time.perf_counter() - t0

    def measure(self, warmup=3, budget_s=10.0, max_reps=200, min_reps=5):
        for _ in range(warmup):
            self.step()
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < min_reps or (time.perf_counter() < t_end and len(times) < max_reps):
            times.append(self.step())
        return self.summary(times)

    def summary(self, times):
        return {"value": median_rate(self.flops, times) / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                "kind": "port", "stat": f"median of {len(times)} samples after warm-up", "cpu_model": cpu_model(),
                "sample": self.sample}


def cpu_legs(budget_s=4.0):
    """The other configurations' CPU path (the reference's torch SDPA calls) on
    bounded samples, reported in each configuration's own unit:

    * C4 decode: the per-sequence SDPA loop (Sq = 1, enable_gqa) over the first
      4 of the 64 seeded sequences, as K/V bytes read per second (GB/s);
    * C3 MHA D=128: one (b, h) slice of the non-causal B=8 H=16 S=2048 call;
    * C5 long context: one KV group (8 query heads) at S=16384, causal,
      EXTRAPOLATED to S=131072 by the S^2 work ratio (the full slice would take
      minutes per sample)."""
    from oracle.attention_oracle import sdpa_cpu
    torch.set_num_threads(os.cpu_count() or 1)

    def timed(fn):
        fn()
        times, t_end = [], time.perf_counter() + budget_s
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        return times

    legs = {}
    lens = torch.randint(1024, 32769, (64,), generator=torch.Generator().manual_seed(42))[:4].tolist()
    g = torch.Generator().manual_seed(42)
    Hq, Hkv, D = 64, 8, 128
    q = torch.randn(4, Hq, 1, D, generator=g).bfloat16()
    kv = [(torch.randn(1, Hkv, L, D, generator=g).bfloat16(), torch.randn(1, Hkv, L, D, generator=g).bfloat16())
          for L in lens]
    t = timed(lambda: [sdpa_cpu(q[b:b + 1], k, v, 1 / math.sqrt(D)) for b, (k, v) in enumerate(kv)])
    nbytes = sum(2 * L * Hkv * D * 2 for L in lens)
    legs["C4_decode"] = {"value": median_rate(nbytes, t) / 1e9, "unit": "GB/s",
                         "sample": f"per-sequence SDPA loop over 4 of the 64 C4 sequences (L = {lens})",
                         "stat": f"median of {len(t)}"}
    S = 2048
    q3 = torch.randn(1, 1, S, D, generator=g).bfloat16()
    k3 = torch.randn(1, 1, S, D, generator=g).bfloat16()
    v3 = torch.randn(1, 1, S, D, generator=g).bfloat16()
    t = timed(lambda: sdpa_cpu(q3, k3, v3, 1 / math.sqrt(D)))
    legs["C3_mha_D128"] = {"value": median_rate(4.0 * S * S * D, t) / 1e12, "unit": "TFLOP/s",
                           "sample": "one (b, h) slice of C3 D=128 (S=2048, non-causal)", "stat": f"median of {len(t)}"}
    S5 = 16384
    q5 = torch.randn(1, 8, S5, D, generator=g).bfloat16()
    k5 = torch.randn(1, 1, S5, D, generator=g).bfloat16()
    v5 = torch.randn(1, 1, S5, D, generator=g).bfloat16()
    t = timed(lambda: sdpa_cpu(q5, k5, v5, 1 / math.sqrt(D), causal=True))
    rate = median_rate(causal_flops(1, 8, S5, D), t)
    full_s = causal_flops(1, 64, 131072, D) / rate
    legs["C5_long_context"] = {"value": rate / 1e12, "unit": "TFLOP/s", "extrapolated": True,
                               "ms_full_config_extrapolated": full_s * 1e3,
                               "sample": "one KV group (8 query heads) causal at S=16384; full C5 time extrapolated "
                                         "by the S^2 work ratio", "stat": f"median of {len(t)}"}
    return legs


def run_reference(args, world, rank):
    if rank != 0:
        return
    ref = CpuReference()
    for _ in range(args.warmup):
        ref.step()
    t = [ref.step() for _ in range(args.steps)]
    cpu = ref.summary(t)
    value = cpu["value"]
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(t),
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1), seed 42", "scaling": "weak",
            "config": dict(c2_config(world), cpu_sample=ref.sample),
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU path
def c2_inputs(rank, device):
    B, Hq, Hkv, S, D = (C2[k] for k in ("B", "Hq", "Hkv", "S", "D"))
    g = torch.Generator(device=device).manual_seed(42 + rank)
    q = torch.randn(B, S, Hq, D, generator=g, device=device).bfloat16()
    k = torch.randn(B, S, Hkv, D, generator=g, device=device).bfloat16()
    v = torch.randn(B, S, Hkv, D, generator=g, device=device).bfloat16()
    return q, k, v


def time_steps(fn, steps, warmup, flush, world):
    """Per-step CUDA-event times (ms) of `fn` on the current stream, L2 flushed before each."""
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        flush()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def bench_decode(flush, steps, warmup, len_div=1):
    """C4: split-KV decode B=64, Hq=64, Hkv=8, D=128, L_b ~ U[1024, 32768] (seed 42).
    len_div > 1 divides every length (small case for profiler captures)."""
    import blackwell_b200 as bw
    B, Hq, Hkv, D = 64, 64, 8, 128
    lens = torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(42)) // len_div
    total = int(lens.sum())
    offs = torch.cumsum(lens, 0) - lens
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    lens_d, offs_d = lens.int().cuda(), offs.long().cuda()
    ws = torch.empty(bw.attention.decode_workspace_size(B, Hq, Hkv, D, total), dtype=torch.uint8, device="cuda")
    o = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, dtype=torch.float32, device="cuda")
    fn = lambda: bw.gqa_decode(q, k, v, lens_d, offs_d, workspace=ws, out=o, lse=lse)
    ms = time_steps(fn, steps, warmup, flush, 1)
    assert bw.stream_status() == 0
    nbytes = 2 * total * Hkv * D * 2 + 2 * B * Hq * D * 2 + B * Hq * 4
    t = statistics.median(ms)
    del k, v
    return {"workload": "C4 split-KV decode B=64 Hq=64 Hkv=8 D=128 L~U[1024,32768] seed 42 (+LSE-combine)",
            "sum_L": total, "ms": t, "GB/s": nbytes / t / 1e6, "algorithmic_bytes": nbytes, "launches_per_step": 2}


def bench_decode_paged(flush, steps, warmup, page_size=64):
    """C4 over a paged KV cache: the same lengths, K/V in pages of `page_size`
    tokens placed in a random physical order (seed 42)."""
    import blackwell_b200 as bw
    B, Hq, Hkv, D = 64, 64, 8, 128
    lens = torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(42))
    pages = (lens + page_size - 1) // page_size
    num_pages = int(pages.sum())
    max_pages = int(pages.max())
    perm = torch.randperm(num_pages, generator=torch.Generator().manual_seed(42)).int()
    bt = torch.full((B, max_pages), -1, dtype=torch.int32)
    start = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[start:start + pages[b]]
        start += int(pages[b])
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    kc = torch.randn(num_pages, page_size, Hkv, D, generator=g, device="cuda").bfloat16()
    vc = torch.randn(num_pages, page_size, Hkv, D, generator=g, device="cuda").bfloat16()
    bt_d, lens_d = bt.cuda(), lens.int().cuda()
    o = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, dtype=torch.float32, device="cuda")
    bound = min(num_pages * page_size, B * max_pages * page_size)
    ws = torch.empty(bw.attention.decode_workspace_size(B, Hq, Hkv, D, bound), dtype=torch.uint8, device="cuda")
    fn = lambda: bw.attention.gqa_decode_paged(q, kc, vc, bt_d, lens_d, workspace=ws, out=o, lse=lse)
    ms = time_steps(fn, steps, warmup, flush, 1)
    assert bw.stream_status() == 0
    total = int(lens.sum())
    nbytes = 2 * total * Hkv * D * 2 + 2 * B * Hq * D * 2 + B * Hq * 4
    t = statistics.median(ms)
    del kc, vc
    return {"workload": f"C4 over a paged KV cache, page_size {page_size}, pages in random order",
            "ms": t, "GB/s": nbytes / t / 1e6}


def bench_decode_sp(world, rank, steps, warmup, flush):
    """C4 decode with every sequence's keys split over the ranks (sequence
    parallel): per step each rank runs bw_gqa_decode_partial on its 1/N of every
    sequence, ONE all-gather of the packed (O, LSE) partials over NCCL, and
    bw_lse_combine_packed.  The three phases are timed separately with CUDA
    events on the launching stream; each figure is the max over ranks of the
    per-rank median."""
    import blackwell_b200 as bw
    from blackwell_b200.distributed import split_sequences
    B, Hq, Hkv, D = 64, 64, 8, 128
    lens = torch.randint(1024, 32769, (B,), generator=torch.Generator().manual_seed(42))
    loc, _ = split_sequences(lens.numpy(), world, rank)
    loc_t = torch.from_numpy(loc)
    total = int(loc_t.sum())
    offs = (torch.cumsum(loc_t.long(), 0) - loc_t.long())
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    g.manual_seed(1000 + rank)
    k = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(total, Hkv, D, generator=g, device="cuda").bfloat16()
    lens_d, offs_d = loc_t.int().cuda(), offs.cuda()
    ws = torch.empty(bw.attention.decode_workspace_size(B, Hq, Hkv, D, total), dtype=torch.uint8, device="cuda")
    P = bw.attention.packed_split_floats(B, Hq, D)
    n_o = B * Hq * D
    buf = torch.empty(P, dtype=torch.float32, device="cuda")
    gathered = torch.empty(world, P, dtype=torch.float32, device="cuda")
    o = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, dtype=torch.float32, device="cuda")
    if world > 1:
        import torch.distributed as dist
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]

    def step(e=None):
        if e: e[0].record()
        bw.attention.gqa_decode_partial(q, k, v, lens_d, offs_d, workspace=ws, out=buf[:n_o].view(B, Hq, D),
                                        lse=buf[n_o:n_o + B * Hq].view(B, Hq))
        if e: e[1].record()
        if world > 1:
            dist.all_gather_into_tensor(gathered, buf)
        else:
            gathered[0].copy_(buf)
        if e: e[2].record()
        bw.attention.lse_combine_packed(gathered, B, Hq, D, out=o, lse=lse)
        if e: e[3].record()

    for _ in range(warmup):
        flush()
        step()
    torch.cuda.synchronize()
    barrier(world)
    for e in ev:
        flush()
        step(e)
    torch.cuda.synchronize()
    barrier(world)
    assert bw.stream_status() == 0
    med = lambda a, b: statistics.median(e[a].elapsed_time(e[b]) for e in ev)
    r = {ph: max_over_ranks(med(a, b), world) for ph, (a, b) in
         {"ms_decode_partial": (0, 1), "ms_allgather": (1, 2), "ms_combine": (2, 3), "ms": (0, 3)}.items()}
    full_total = int(lens.sum())
    nbytes = 2 * full_total * Hkv * D * 2 + 2 * B * Hq * D * 2 + B * Hq * 4
    r.update({"workload": "C4 decode, every sequence's keys split over the ranks (sequence parallel), "
                          "one NCCL all-gather of packed (O, LSE) partials + LSE-combine",
              "ranks": world, "bytes_allgathered_per_rank": P * 4, "GB/s_total": nbytes / r["ms"] / 1e6,
              "GB/s_per_gpu": nbytes / r["ms"] / 1e6 / world})
    del k, v
    return r


def bench_prefill(shape, causal, layout, flush, steps, warmup):
    import blackwell_b200 as bw
    B, Hq, Hkv, S, D = shape
    g = torch.Generator(device="cuda").manual_seed(42)
    if layout == "bshd":
        q = torch.randn(B, S, Hq, D, generator=g, device="cuda").bfloat16().transpose(1, 2)
        k = torch.randn(B, S, Hkv, D, generator=g, device="cuda").bfloat16().transpose(1, 2)
        v = torch.randn(B, S, Hkv, D, generator=g, device="cuda").bfloat16().transpose(1, 2)
    else:
        q = torch.randn(B, Hq, S, D, generator=g, device="cuda").bfloat16()
        k = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
        v = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
    o = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device="cuda")
    fn = lambda: bw.gqa_split_fwd(q, k, v, 1 / math.sqrt(D), causal=causal, out=o, lse=lse)
    ms = time_steps(fn, steps, warmup, flush, 1)
    assert bw.stream_status() == 0
    flops = causal_flops(B, Hq, S, D) if causal else 4.0 * B * Hq * S * S * D
    t = statistics.median(ms)
    return {"ms": t, "TFLOP/s": flops / t / 1e9}


def bench_fused(shape, flush, steps, warmup):
    """The reference's fused op (QK-norm + RoPE + causal GQA) at a prefill shape:
    the Q and K prologues as streaming passes into a workspace, then the
    attention kernel (bw_gqa_fused_fwd)."""
    import blackwell_b200 as bw
    B, Hq, Hkv, S, D = shape
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, Hq, S, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, Hkv, S, D, generator=g, device="cuda").bfloat16()
    half = D // 2
    inv = 10000.0 ** (-torch.arange(half, dtype=torch.float64, device="cuda") * 2.0 / D)
    ang = torch.arange(S, dtype=torch.float64, device="cuda")[:, None] * inv[None]
    cache = torch.cat([ang.cos(), ang.sin()], 1).float().contiguous()
    qg = 1 + 0.1 * torch.randn(D, generator=g, device="cuda")
    kg = 1 + 0.1 * torch.randn(D, generator=g, device="cuda")
    fn = lambda: bw.gqa_fused_fwd(q, k, v, cache, qg, kg, causal=True)
    ms = time_steps(fn, steps, warmup, flush, 1)
    assert bw.stream_status() == 0
    t = statistics.median(ms)
    return {"ms": t, "TFLOP/s": causal_flops(B, Hq, S, D) / t / 1e9}


def bench_norm_rope(flush, steps, warmup):
    """QK-norm + RoPE (NeoX) of the C2 query tensor [4, 32, 4096, 128] bf16, gamma
    present: one streaming pass, 2 x 128 MiB of traffic."""
    import blackwell_b200 as bw
    B, H, S, D = 4, 32, 4096, 128
    g = torch.Generator(device="cuda").manual_seed(42)
    q = torch.randn(B, H, S, D, generator=g, device="cuda").bfloat16()
    half = D // 2
    inv = 10000.0 ** (-torch.arange(half, dtype=torch.float64, device="cuda") * 2.0 / D)
    ang = torch.arange(S, dtype=torch.float64, device="cuda")[:, None] * inv[None]
    cache = torch.cat([ang.cos(), ang.sin()], 1).float().contiguous()
    gamma = 1 + 0.1 * torch.randn(D, generator=g, device="cuda")
    out = torch.empty_like(q)
    ms = time_steps(lambda: bw.qk_norm_rope(q, cache, gamma, out=out), steps, warmup, flush, 1)
    assert bw.stream_status() == 0
    t = statistics.median(ms)
    return {"ms": t, "GB/s": 2 * q.numel() * 2 / t / 1e6}


def bench_c5(world, rank, steps, warmup):
    """C5: causal GQA B=1, Hq=64, Hkv=8, S=131072, D=128, one or more KV-head groups
    per rank (8 groups sharded over the ranks, no exchange).  Each rank holds only
    its groups' Q/K/V (BHSD).  Time = max over ranks of the CUDA-event time."""
    import blackwell_b200 as bw
    from blackwell_b200.distributed import unit_range
    Hq, Hkv, S, D = 64, 8, 131072, 128
    G = Hq // Hkv
    g0, g1 = unit_range(Hkv, world, rank)
    ng = g1 - g0
    if ng == 0:
        ms = 0.0
    else:
        gen = torch.Generator(device="cuda").manual_seed(42 + rank)
        q = torch.randn(1, ng * G, S, D, generator=gen, device="cuda").bfloat16()
        k = torch.randn(1, ng, S, D, generator=gen, device="cuda").bfloat16()
        v = torch.randn(1, ng, S, D, generator=gen, device="cuda").bfloat16()
        o = torch.empty_like(q)
        lse = torch.empty(1, ng * G, S, dtype=torch.float32, device="cuda")
        fn = lambda: bw.gqa_causal_fwd(q, k, v, out=o, lse=lse)
        ms = statistics.median(time_steps(fn, steps, warmup, lambda: None, world))
        assert bw.stream_status() == 0
        del q, k, v, o
        torch.cuda.empty_cache()
    if ng == 0:
        time_steps(lambda: None, steps, warmup, lambda: None, world)
    ms_max = max_over_ranks(ms, world)
    flops = causal_flops(1, Hq, S, D)
    return {"workload": "C5 causal GQA B=1 Hq=64 Hkv=8 S=131072 D=128, KV groups sharded over ranks",
            "groups_per_rank": [unit_range(Hkv, world, r)[1] - unit_range(Hkv, world, r)[0] for r in range(world)],
            "ms": ms_max, "TFLOP/s_total": flops / ms_max / 1e9, "TFLOP/s_per_gpu": flops / ms_max / 1e9 / world,
            "l2": "inputs (>= 320 MiB per rank) exceed L2; no flush"}


def run_ours(args, world, rank, local):
    import blackwell_b200 as bw
    from blackwell_b200 import _ffi
    _ffi.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, peak_kind = load_peaks()
    flush_buf = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    flush = lambda: flush_buf.zero_()

    B, Hq, Hkv, S, D = (C2[k] for k in ("B", "Hq", "Hkv", "S", "D"))
    q, k, v = c2_inputs(rank, dev)
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    o = torch.empty(B, S, Hq, D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, Hq, S, dtype=torch.float32, device=dev)
    scale = 1 / math.sqrt(D)
    step = lambda: bw.gqa_causal_fwd(qt, kt, vt, scale, out=o.transpose(1, 2), lse=lse)

    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, args.warmup, flush, world)
    rc = bw.stream_status()
    if rc != 0:
        raise RuntimeError(f"device error {rc}")
    total_ms = sum(ms)
    total_ms_max = max_over_ranks(total_ms, world)
    flops = causal_flops(B, Hq, S, D)
    value = flops * args.steps * world / (total_ms_max * 1e-3) / 1e12
    per_launch_ms = total_ms / args.steps
    achieved = flops / (per_launch_ms * 1e-3) / 1e12

    # ---- end to end through the public API with pinned host buffers
    e2e_steps = 3 if args.profile else max(3, min(args.steps, 20))
    hq_, hk_, hv_ = (x.cpu().pin_memory() for x in (q, k, v))
    ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
    hl = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()
    ws = torch.empty(bw.host_workspace_size(B, Hq, Hkv, S, D), dtype=torch.uint8, device=dev)

    def e2e_step():
        # public host-buffer C-ABI call (bw_attn_fwd_host): copy-in, kernel and
        # copy-out pipelined in sequence chunks (PCIe in / out and the kernel overlap)
        bw.attention_from_host(hq_.transpose(1, 2), hk_.transpose(1, 2), hv_.transpose(1, 2), ho.transpose(1, 2),
                               hl, scale=scale, causal=True, chunks=args.e2e_chunks, workspace=ws)

    ms_e2e = time_steps(e2e_step, e2e_steps, 2, lambda: None, world)
    e2e_ms_max = max_over_ranks(sum(ms_e2e), world)
    e2e_value = flops * e2e_steps * world / (e2e_ms_max * 1e-3) / 1e12
    h2d = sum(x.numel() * x.element_size() for x in (hq_, hk_, hv_))
    d2h = ho.numel() * ho.element_size() + hl.numel() * hl.element_size()

    secondary = {}
    if rank == 0 and world == 1 and not (args.no_secondary or args.profile):
        del hq_, hk_, hv_, ws
        torch.cuda.empty_cache()
        sec_steps = max(20, min(args.steps // 10, 50))
        secondary["C3_mha_D64"] = bench_prefill((8, 16, 16, 2048, 64), False, "bhsd", flush, sec_steps, 3)
        secondary["C3_mha_D128"] = bench_prefill((8, 16, 16, 2048, 128), False, "bhsd", flush, sec_steps, 3)
        ref_shape = bench_prefill((8, 12, 4, 4096, 64), True, "bhsd", flush, sec_steps, 3)
        ref_shape["reference_V46_B300_ms"] = 0.5863
        secondary["reference_shape_causal_B8_Hq12_Hkv4_S4096_D64"] = ref_shape
        secondary["fused_norm_rope_causal_C2_bhsd"] = bench_fused((4, 32, 8, 4096, 128), flush, sec_steps, 3)
        for key in ("C3_mha_D64", "C3_mha_D128", "reference_shape_causal_B8_Hq12_Hkv4_S4096_D64",
                    "fused_norm_rope_causal_C2_bhsd"):
            secondary[key]["frac_of_peak"] = secondary[key]["TFLOP/s"] / peaks["bf16_tflops"]
        dec = bench_decode(flush, sec_steps, 3)
        dec["frac_of_hbm_peak"] = dec["GB/s"] / peaks["hbm_gbs"]
        secondary["C4_decode"] = dec
        for ps in (16, 64):
            dp = bench_decode_paged(flush, sec_steps, 3, page_size=ps)
            dp["frac_of_hbm_peak"] = dp["GB/s"] / peaks["hbm_gbs"]
            secondary[f"C4_decode_paged_{ps}"] = dp

    if not (args.no_secondary or args.profile):
        c5 = bench_c5(world, rank, 3, 3)
        sp = bench_decode_sp(world, rank, 20, 3, flush)
        if rank == 0:
            # a quarter-second launch is a sustained load: its fraction is quoted
            # against the sustained peak (the burst one beside it)
            sus = peaks.get("bf16_tflops_sustained")
            c5["frac_of_sustained_peak_per_gpu"] = c5["TFLOP/s_per_gpu"] / sus if sus else None
            c5["frac_of_burst_peak_per_gpu"] = c5["TFLOP/s_per_gpu"] / peaks["bf16_tflops"]
            secondary["C5_long_context"] = c5
            sp["frac_of_hbm_peak_per_gpu"] = sp["GB/s_per_gpu"] / peaks["hbm_gbs"]
            secondary["C4_decode_sequence_parallel"] = sp

    cpu = None
    if rank == 0 and world == 1 and not args.profile:
        cpu = CpuReference().measure(warmup=3, budget_s=10.0)
        cpu["legs"] = cpu_legs()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_launch_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seed 42 (+rank)",
            "config": c2_config(world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops"], "peak_kind": f"{peak_kind} bf16 burst",
                         "traffic": profile_traffic("fmha_fwd_c2_launches.md")},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)


def run_single(args):
    """One workload's kernel, W warm-up + K timed steps (for ncu captures)."""
    torch.cuda.set_device(0)
    flush_buf = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    flush = lambda: flush_buf.zero_()
    shapes = {"c2": ((4, 32, 8, 4096, 128), True, "bshd"), "c3d64": ((8, 16, 16, 2048, 64), False, "bhsd"),
              "c3d128": ((8, 16, 16, 2048, 128), False, "bhsd"), "refshape": ((8, 12, 4, 4096, 64), True, "bhsd")}
    if args.workload in shapes:
        r = bench_prefill(*shapes[args.workload], flush, args.steps, args.warmup)
    elif args.workload == "c4paged16":
        r = bench_decode_paged(flush, args.steps, args.warmup, page_size=16)
    elif args.workload == "normrope":
        r = bench_norm_rope(flush, args.steps, args.warmup)
    else:
        r = bench_decode(flush, args.steps, args.warmup, len_div=8 if args.workload == "c4small" else 1)
    print(json.dumps({"workload": args.workload, **r}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="pieces the host-buffer e2e call pipelines (sequence chunks for causal C2)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="short run for profiler captures: no secondary configs, no CPU baseline")
    ap.add_argument("--workload", choices=["c2", "c3d64", "c3d128", "c4", "c4small", "c4paged16", "refshape",
                                           "normrope"],
                    default=None,
                    help="profiler aid: run only this workload's kernel and print its timing")
    args = ap.parse_args()
    if args.workload:
        run_single(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
