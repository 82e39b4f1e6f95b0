"""Benchmark: SupraDiT attention workload per Euler step on 1..8 B200.

One step = one Euler step of the DiT's attention: 14 blocks x (self-attention over 256 patch
tokens + cross-attention to the sequence's cached projected T5 K/V of ragged length L ~ U{1..128}),
9 heads x 64, for 1024 prompts with CFG (2048 sequences), sharded by prompt across the ranks
(strong scaling), the last step's outputs gathered to rank 0. Each attention call is issued as the
reference issues it (one ops.attention per sample, app/models/dit.js:170-173,182-185) through
the C ABI; the library groups the 2048 calls of a block into one launch. Self and cross
attention of a block are flushed separately because the model's cross-attention query depends
on the self-attention output.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0. `value` = sequence-attentions per second over all ranks
(one sequence-attention = one sample's all-head attention at one call; a step has
2048 x 14 x 2 of them), inputs resident in HBM. `e2e` = the same metric through the public API
with the step's inputs uploaded from pinned host memory and its output read back inside the
timed region. `roofline` = the fused FP32 kernel's algorithmic FLOPs per launch over its
CUDA-event launch time, against the FP32 FFMA peak. `cpu_baseline` = tools/reference.py's CPU
attention (restated in oracle/) on this host's cores, on a bounded sample.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "supra2-img-web_b200"))
sys.path.insert(0, ROOT)

N_HEADS, HEAD_DIM, TOKENS, DIM = 9, 64, 256, 576
BLOCKS = 14
METRIC = "dit_attention_sequences_per_s"
UNIT = "seq/s"


# ---------------------------------------------------------------------------------------------
def workload_lengths(prompts: int, seed: int):
    """Cross-attention K/V length of every sequence (2 per prompt: cond, uncond), L ~ U{1..128}."""
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(1, 129, (2 * prompts,), generator=g).tolist()


def shard_prompts(lengths, world: int, rank: int):
    """Prompts dealt to ranks longest-first in a snake order so that every rank gets the same
    number of prompts and near-equal sum of K/V lengths (the cross-attention work)."""
    prompts = len(lengths) // 2
    order = sorted(range(prompts), key=lambda p: -(lengths[2 * p] + lengths[2 * p + 1]))
    mine = []
    for i, p in enumerate(order):
        r = i % (2 * world)
        r = r if r < world else 2 * world - 1 - r
        if r == rank:
            mine.append(p)
    return sorted(mine)


def bind_to_gpu_cpus(torch, dev_index: int):
    """Pins this process to the host CPUs nearest its GPU (the PCI device's local_cpulist), so the
    pinned host buffers it allocates afterwards land on that NUMA node. With N ranks each moving
    its step's inputs over PCIe, buffers on the far socket cost the copies host-link bandwidth.
    Returns the CPU list applied, or None when the host does not say."""
    try:
        p = torch.cuda.get_device_properties(dev_index)
        path = (f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/"
                "local_cpulist")
        with open(path) as f:
            spec = f.read().strip()
        cpus = parse_cpulist(spec)
        if not cpus or len(cpus) >= (os.cpu_count() or 1):
            return None
        os.sched_setaffinity(0, cpus)
        return spec
    except (OSError, ValueError, AttributeError, RuntimeError):
        return None


def parse_cpulist(spec: str) -> set:
    """The CPUs of a sysfs CPU list such as "0-47,96-143"."""
    cpus = set()
    for part in spec.split(","):
        if part.strip():
            lo, _, hi = part.strip().partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def site_shard(n: int, rank: int, world: int, shardable: bool = True):
    """A call site's problems on this rank: (indices, replicas). Sharded round-robin (problem i on
    rank i % world) when the site may be split and has at least `world` problems; otherwise every
    rank runs the whole batch as a replica."""
    if world <= 1:
        return list(range(n)), False
    if not shardable or n < world:
        return list(range(n)), True
    return [i for i in range(n) if i % world == rank], False


class ClockSampler:
    """nvidia-smi clocks/power/throttle reasons every 200 ms while the timed region runs."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.lines = []
        self.t_begin = None
        self.t_end = None

    def mark_begin(self):
        self.t_begin = time.monotonic()

    def mark_end(self):
        self.t_end = time.monotonic()

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append((time.monotonic(), ln.strip()))

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, power, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines:
            if (self.t_begin and ts < self.t_begin) or (self.t_end and ts > self.t_end + 0.25):
                continue  # only samples taken while the timed region ran
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10 or (self.uuid and self.uuid not in f[1]):
                continue
            try:
                sm.append(float(f[2]))
                smax = float(f[3])
                power.append(float(f[4]))
            except ValueError:
                continue
            for n, val in zip(names, f[6:10]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def sgemm_tflops(torch, dev, n=8192, reps=5):
    """Measured FP32 reference rate on this GPU: cuBLAS SGEMM (torch.matmul, TF32 off) on n^3,
    best of `reps`, CUDA events. The FP32 counterpart of MEASURED_PEAKS.json's cuBLAS bf16 figure."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = torch.empty(n, n, device=dev)
        torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        return 2.0 * n ** 3 / (best / 1e3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ---------------------------------------------------------------------------------------------
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            return next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), "")
    except OSError:
        return ""


def workload_config(args, world: int) -> dict:
    """The configs[4] workload both arms report (the reference arm runs the same config on the CPU)."""
    return {"workload": f"supradit_attention_step (configs[4]): {args.prompts} prompts x CFG = {2 * args.prompts} "
                        "seqs, 14 blocks x (self 256x256 + cross 256xL, L~U{1..128}), 9x64 heads",
            "prompts": args.prompts, "global_batch": 2 * args.prompts, "seq_len": TOKENS,
            "parallelism": f"prompt-sharded x{world}, outputs gathered to rank 0",
            "l2": "inputs larger than L2 (qkv 3.6 GB, K/V 8.5 GB per step at N=1)"}


class CpuStep:
    """One configs[4] step on the host cores through the port of tools/reference.py's CPU attention
    (oracle.sdpa_port, tools/reference.py:72-79), torch fp32 on all host threads: per block,
    self-attention per CFG pair (the reference runs cond and uncond as one batch of 2,
    tools/reference.py:173) and cross-attention per sequence at its true length L
    (app/models/dit.js:184). Every one of the step's 2 x 14 x n sequence-attentions runs.

    Inputs are built once from a seeded pool: sequence i reads Q/K/V rows of pool entry
    i % pool (256 sequences, 0.6 GB, larger than the host's last-level cache) and its K/V from a
    pool of 32768 rows at a running offset; one K/V pool serves all 14 blocks. The pools tile 8 M
    seeded N(0,1) values; the values do not change the CPU cost of an attention call."""

    POOL, KV_ROWS = 256, 32768

    def __init__(self, lengths, seed: int):
        import torch

        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        g = torch.Generator().manual_seed(seed)
        self.n = len(lengths)
        self.lengths = list(lengths)
        pool = min(self.POOL, self.n)
        base = torch.randn(1 << 23, generator=g)  # seeded N(0,1) values, tiled into the pool

        def fill(*shape):
            n = math.prod(shape)
            return base.repeat((n + base.numel() - 1) // base.numel())[:n].view(*shape)

        self.qkv = fill(pool, TOKENS, 3, DIM)
        self.qx = fill(pool, TOKENS, DIM)
        self.kv = fill(self.KV_ROWS, 2 * DIM)
        self.kv_off, off = [], 0
        for L in self.lengths:
            if off + L > self.KV_ROWS:
                off = 0
            self.kv_off.append(off)
            off += L

    def block(self):
        import oracle

        pool = self.qkv.shape[0]
        for b in range(0, self.n, 2):  # a CFG pair is two consecutive sequences
            p = self.qkv[b % pool:b % pool + 2]
            oracle.sdpa_port(p[:, :, 0], p[:, :, 1], p[:, :, 2], N_HEADS)
        for i in range(self.n):
            kv = self.kv[self.kv_off[i]:self.kv_off[i] + self.lengths[i]][None]
            oracle.sdpa_port(self.qx[i % pool:i % pool + 1], kv[:, :, :DIM], kv[:, :, DIM:], N_HEADS)

    def step(self):
        for _ in range(BLOCKS):
            self.block()

    def seq_calls(self) -> int:
        return 2 * BLOCKS * self.n

    def describe(self, steps: int, seconds: float) -> str:
        return (f"{steps} whole configs[4] step(s): {self.n} sequences x {BLOCKS} blocks x (self 256x256 per CFG "
                f"pair + cross 256xL at each sequence's true L) = {self.seq_calls()} sequence-attentions per step, "
                f"torch CPU fp32 SDPA (tools/reference.py:72-79 port), {self.threads} threads, {seconds:.1f} s; "
                f"CPU: {cpu_model()}")


def cpu_baseline_leg(lengths, seed: int, seconds: float):
    """The cpu_baseline of the GPU arm: CpuStep after a one-block warm-up, whole steps until
    `seconds` have passed (at least one). The reference arm times the same steps the same way."""
    cpu = CpuStep(lengths, seed)
    cpu.block()
    steps, t0 = 0, time.perf_counter()
    while True:
        cpu.step()
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    rate = steps * cpu.seq_calls() / el
    return {"value": rate, "unit": UNIT, "cores": cpu.threads, "kind": "port", "ms_per_step": el / steps * 1e3,
            "sample": cpu.describe(steps, el)}


def run_reference(args, rank, world):
    """`--impl reference`: the reference's CPU attention (the port of tools/reference.py:72-79,
    oracle.sdpa_port) on this host's cores, rank 0 only. Every step is the whole configs[4] step
    (CpuStep): W untimed warm-up steps, then K steps, each timed with the host clock."""
    if rank != 0:
        return
    lengths = workload_lengths(args.prompts, args.seed)
    cpu = CpuStep(lengths, args.seed)
    for _ in range(args.warmup):
        cpu.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu.step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = args.steps * cpu.seq_calls() / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,1) Q/K/V, L~U{1..128})", "impl": "reference",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu.threads, "kind": "port",
                         "sample": cpu.describe(args.steps, total)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "step_s": {"min": min(times), "median": statistics.median(times), "max": max(times)},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
def measure_call_sites(gpu, torch, dev, seed: int, reps: int = 5, only=None, cpu_reps: int = 3, rank: int = 0,
                       world: int = 1, dist=None):
    """BASELINE.json configs[0..3] as extra figures: DiT self (B=2), DiT cross (128 ragged
    sequences), T5 (256 prompts, ragged L, bias), VAE mid-block (1, 8, 64 images). Each rep is one
    flush of the call site's calls, timed with CUDA events after the L2 is flushed; FP32 and TF32
    requests both reported with the kernels that ran (TF32 requests the tensor-core kernel does
    not cover run the FP32 kernels). only: names of the call sites to run (default all).
    With world > 1 every rank runs its share of a site's batch (problem i on rank i % world; a
    batch smaller than world, and the B = 2 self-attention pair, run whole on every rank as
    replicas), each rep starts after a barrier, and a rep's time is the max over ranks; the
    f-rows (whole blocks, K/V preparation) run on one GPU only."""
    import supra_attn

    if world > 1:  # the f-rows are single-GPU figures
        keep = {"dit_self_b2", "dit_cross_128", "t5_256", "t5_256_table", "vae"}
        only = keep if only is None else set(only) & keep

    peaks = measured_peaks()
    fp32_peak = 148 * 128 * 2 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    flush = torch.empty(64 * 1024 * 1024, device=dev)  # 256 MB > L2
    g = torch.Generator(device=dev).manual_seed(seed)
    gc = torch.Generator().manual_seed(seed)
    out = {}
    want = lambda name: only is None or name in only

    tf_peak = float(peaks.get("bf16_tflops", 1590.0)) / 2.0  # TF32 dense peak: half of measured bf16

    def run(name, units, unit_name, make_descs, flops, bytes_, cpu=None, out_fn=None, shardable=True):
        """Times the call site's flush for each variant; with `cpu` (runs the site's calls through
        the torch CPU port on all host cores and returns the flat output) also times that, and
        compares each variant's output (`out_fn`) with it."""
        import oracle

        res = {}
        mine, replicas = site_shard(units, rank, world, shardable)
        if replicas:  # every rank runs the whole batch: the job does world times the work
            units, flops, bytes_ = units * world, flops * world, bytes_ * world
        if world > 1:
            res["ranks"] = {"world": world, "mode": "replicas" if replicas else "sharded (problem i on rank i % N)"}
        ref = None
        if cpu is not None and cpu_reps > 0:
            import torch as _t

            cpu()  # warm-up
            ts = []
            for _ in range(cpu_reps):
                t0 = time.perf_counter()
                ref = cpu()
                ts.append(time.perf_counter() - t0)
            cms = statistics.median(ts) * 1e3
            res["cpu"] = {"ms": cms, f"{unit_name}_per_s": units / (cms / 1e3), "tflops": flops / (cms / 1e3) / 1e12,
                          "cores": _t.get_num_threads(), "kind": "port"}
        for variant in ("fp32", "tf32", "tf32x3"):
            descs = make_descs(variant)
            if len(mine) != len(descs):
                descs = (supra_attn.Desc * len(mine))(*[descs[i] for i in mine])
            gpu.enqueue_batch(descs)
            gpu.sync()
            times = []
            for prof_on in (False, True):  # timed without the profiler's events, then profiled apart
                gpu.profile(prof_on)
                gpu.profile_reset()
                for _ in range(reps):
                    flush.fill_(1.0)
                    if world > 1:
                        dist.barrier(device_ids=[dev.index])
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    gpu.enqueue_batch(descs)
                    gpu.flush()
                    e1.record()
                    torch.cuda.synchronize()
                    if not prof_on:
                        times.append(e0.elapsed_time(e1))
            prof = gpu.profile_report()
            gpu.profile(False)
            if world > 1:  # each rep's time is the slowest rank's
                tt = torch.tensor(times, device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                times = tt.tolist()
            ms = statistics.median(times)
            per = {}
            for r in prof:
                per[r["name"]] = per.get(r["name"], 0.0) + r["ms"] / reps
            tensor = any(k.startswith(("linear_tc", "attn_tf32")) for k in per)
            e = {"ms": ms, f"{unit_name}_per_s": units / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12,
                 "gbs": bytes_ / (ms / 1e3) / 1e9, "frac_hbm": bytes_ / (ms / 1e3) / 1e9 / hbm,
                 "kernels": sorted(per), "ms_per_kernel": {k: round(v, 4) for k, v in sorted(per.items())}}
            if tensor:  # issued TF32 MMA work (3 products per product in the split form) against the TF32 peak
                e["frac_tf32_peak"] = (3 if variant == "tf32x3" else 1) * flops / (ms / 1e3) / 1e12 / tf_peak
            else:  # the FFMA kernels ran (an FP32 request, or a tensor request they cover instead)
                e["frac_fp32_peak"] = flops / (ms / 1e3) / 1e12 / fp32_peak
            if ref is not None and out_fn is not None:
                got = out_fn()
                e["parity_vs_cpu"] = {"max_rel": oracle.max_rel(got, ref), "rel_l2": oracle.rel_l2(got, ref)}
            res[variant] = e
        out[name] = res

    enq = supra_attn.lib.supra_attn_enqueue_linear
    VCODES = {"fp32": supra_attn._lib.FP32, "tf32x3": supra_attn._lib.TF32X3, "tf32": supra_attn._lib.TF32}

    def timed_variants(fn, descs, per_kernel=False):
        # each numeric variant on the same recorded calls: median ms over reps, kernels launched
        res = {}
        for vname, code in VCODES.items():
            for d in descs:
                d.variant = code
            fn()
            gpu.sync()
            times = []
            for prof_on in (False, True):  # timed without the profiler's events, then profiled apart
                gpu.profile(prof_on)
                gpu.profile_reset()
                for _ in range(reps):
                    flush.fill_(1.0)
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    torch.cuda.synchronize()
                    if not prof_on:
                        times.append(e0.elapsed_time(e1))
            prof = gpu.profile_report()
            gpu.profile(False)
            per = {}
            for r in prof:
                per[r["name"]] = per.get(r["name"], 0.0) + r["ms"] / reps
            res[vname] = (statistics.median(times), sorted(per), per)
        for d in descs:
            d.variant = VCODES["fp32"]
        return res

    if want("dit_self_b2"):
        # DiT self-attention, B = 2, interleaved qkv
        qkv = torch.randn(2 * 256 * 1728, device=dev, generator=g)
        o1 = torch.empty(2 * 256 * 576, device=dev)

        def c1(variant):
            arr = (supra_attn.Desc * 2)()
            for b in range(2):
                r = b * 256 * 1728
                arr[b] = supra_attn.make_desc(q=qkv, k=qkv, v=qkv, out=o1, Lq=256, Lk=256, H=9, D=64, ldq=1728, ldk=1728,
                                              ldv=1728, qOff=r, kOff=r + 576, vOff=r + 1152, oOff=b * 256 * 576,
                                              variant=variant)
            return arr

        f1 = 2 * 4.0 * 256 * 256 * 64 * 9
        qkv_c = qkv.cpu().view(2, 256, 3, 576)

        def cpu1():  # tools/reference.py:72-79 on the CFG pair, as tools/reference.py:173 runs it
            import oracle
            return oracle.sdpa_port(qkv_c[:, :, 0], qkv_c[:, :, 1], qkv_c[:, :, 2], 9).reshape(-1).numpy()

        run("dit_self_b2", 2, "seq", c1, f1, 2 * 4.0 * (2 * 256 * 576 + 2 * 256 * 576), cpu=cpu1,
            out_fn=lambda: o1.cpu().numpy(), shardable=False)

    if want("dit_cross_128"):
        # DiT cross-attention, 64 prompts x CFG, ragged L
        Ls = torch.randint(1, 129, (128,), generator=gc).tolist()
        q2 = torch.randn(128 * 256 * 576, device=dev, generator=g)
        kv2 = [torch.randn(L * 1152, device=dev, generator=g) for L in Ls]
        o2 = torch.empty_like(q2)

        def c2(variant):
            arr = (supra_attn.Desc * 128)()
            for b, L in enumerate(Ls):
                arr[b] = supra_attn.make_desc(q=q2, k=kv2[b], v=kv2[b], out=o2, Lq=256, Lk=L, H=9, D=64, ldq=576,
                                              ldk=1152, ldv=1152, qOff=b * 256 * 576, kOff=0, vOff=576,
                                              oOff=b * 256 * 576, variant=variant)
            return arr

        q2_c = q2.cpu().view(128, 256, 576)
        kv2_c = [x.cpu().view(1, -1, 1152) for x in kv2]

        def cpu2():  # one call per sequence at its true L (app/models/dit.js:184)
            import oracle
            return torch.cat([oracle.sdpa_port(q2_c[b:b + 1], kv2_c[b][:, :, :576], kv2_c[b][:, :, 576:], 9)
                              for b in range(128)]).reshape(-1).numpy()

        run("dit_cross_128", 128, "seq", c2, sum(4.0 * 256 * L * 64 * 9 for L in Ls),
            sum(4.0 * (2 * 256 * 576 + 2 * L * 576) for L in Ls), cpu=cpu2, out_fn=lambda: o2.cpu().numpy())

    if want("t5_256") or want("t5_256_table"):  # (the table form reuses these inputs)
        # T5 encoder attention, 256 prompts, ragged L, relative-position bias, scale 1
        Lt = torch.randint(1, 129, (256,), generator=gc).tolist()
        table = (torch.randn(32 * 12, generator=gc) * 0.1).to(dev)
        qs = [torch.randn(L * 768, device=dev, generator=g) for L in Lt]
        ks = [torch.randn(L * 768, device=dev, generator=g) for L in Lt]
        vs = [torch.randn(L * 768, device=dev, generator=g) for L in Lt]
        os_ = [torch.empty(L * 768, device=dev) for L in Lt]
        biases = [gpu.wrap(torch.empty(12 * L * L, device=dev)) for L in Lt]
        for L, bt in zip(Lt, biases):
            supra_attn.position_bias(gpu, table, L, H=12, out=bt)
        gpu.sync()

        def c3(variant):
            arr = (supra_attn.Desc * 256)()
            for i, L in enumerate(Lt):
                arr[i] = supra_attn.make_desc(q=qs[i], k=ks[i], v=vs[i], out=os_[i], bias=biases[i], Lq=L, Lk=L, H=12, D=64,
                                              ldq=768, ldk=768, ldv=768, scale=1.0, variant=variant)
            return arr

        qs_c, ks_c, vs_c = ([x.cpu().view(-1, 768) for x in xs] for xs in (qs, ks, vs))
        bias_c = [torch.from_numpy(gpu.read(bt)).view(12, L, L) for L, bt in zip(Lt, biases)]

        def cpu3():  # transformers' T5Attention arithmetic per prompt (oracle.t5_sdpa_port)
            import oracle
            return torch.cat([oracle.t5_sdpa_port(qs_c[i], ks_c[i], vs_c[i], bias_c[i], 12).reshape(-1)
                              for i in range(len(Lt))]).numpy()

        out3 = lambda: torch.cat([o.reshape(-1) for o in os_]).cpu().numpy()
        if want("t5_256"):
            run("t5_256", 256, "prompt", c3, sum(4.0 * L * L * 64 * 12 for L in Lt),
                sum(4.0 * (4 * L * 768 + 12 * L * L) for L in Lt), cpu=cpu3, out_fn=out3)

    if want("t5_256_table"):
        # the same T5 calls with the [32, 12] table in place of the expanded bias (the kernels form
        # the bias; the host's per-prompt bias build and its 48*L^2 bytes drop out)
        def c3t(variant):
            arr = (supra_attn.Desc * 256)()
            for i, L in enumerate(Lt):
                arr[i] = supra_attn.make_desc(q=qs[i], k=ks[i], v=vs[i], out=os_[i], t5_table=table, Lq=L, Lk=L, H=12,
                                              D=64, ldq=768, ldk=768, ldv=768, scale=1.0, variant=variant)
            return arr

        run("t5_256_table", 256, "prompt", c3t, sum(4.0 * L * L * 64 * 12 for L in Lt),
            sum(4.0 * (4 * L * 768 + 32 * 12) for L in Lt), cpu=cpu3, out_fn=out3)

    if want("vae"):
        # VAE mid-block single-head attention, 1024 tokens x 512 channels
        for nimg in (1, 8, 64):
            qv = torch.randn(nimg * 1024 * 512, device=dev, generator=g)
            kvv = torch.randn(nimg * 1024 * 512, device=dev, generator=g)
            vv = torch.randn(nimg * 1024 * 512, device=dev, generator=g)
            ov = torch.empty_like(qv)

            def c4(variant, nimg=nimg, qv=qv, kvv=kvv, vv=vv, ov=ov):
                arr = (supra_attn.Desc * nimg)()
                for i in range(nimg):
                    o = i * 1024 * 512
                    arr[i] = supra_attn.make_desc(q=qv, k=kvv, v=vv, out=ov, Lq=1024, Lk=1024, H=1, D=512, ldq=512,
                                                  ldk=512, ldv=512, qOff=o, kOff=o, vOff=o, oOff=o, variant=variant)
                return arr

            qc, kc, vc = (x.cpu().view(nimg, 1, 1024, 512) for x in (qv, kvv, vv))

            def cpu4(nimg=nimg, qc=qc, kc=kc, vc=vc):  # the reference's attention() with one head, per image
                import oracle
                return torch.cat([oracle.sdpa_port(qc[i], kc[i], vc[i], 1) for i in range(nimg)]).reshape(-1).numpy()

            run(f"vae_{nimg}", nimg, "image", c4, nimg * 4.0 * 1024 * 1024 * 512, nimg * 4.0 * 4 * 1024 * 512,
                cpu=cpu4, out_fn=lambda ov=ov: ov.cpu().numpy())
            del qv, kvv, vv, ov

    if want("vae_block_8"):
        # VAE mid-block attention, whole block fused (app/models/vae.js:77-94), 8 images of 32x32:
        # GroupNorm folded into one stacked q/k/v product, attention reading q/k/v in place, residual
        # folded into the output projection.
        nimg, hw, C = 8, 1024, 512
        xv = torch.randn(nimg * hw * C, device=dev, generator=g)
        gam = 1 + 0.1 * torch.randn(C, device=dev, generator=g)
        bet = 0.1 * torch.randn(C, device=dev, generator=g)
        wqkv = torch.randn(3 * C * C, device=dev, generator=g) * C ** -0.5
        bqkv = 0.1 * torch.randn(3 * C, device=dev, generator=g)
        wo = torch.randn(C * C, device=dev, generator=g) * C ** -0.5
        bo = 0.1 * torch.randn(C, device=dev, generator=g)
        qkv_v = torch.empty(nimg * hw * 3 * C, device=dev)
        a_v = torch.empty(nimg * hw * C, device=dev)
        y_v = torch.empty(nimg * hw * C, device=dev)
        dq = supra_attn.make_linear_desc(x=xv, w=wqkv, bias=bqkv, y=qkv_v, M=nimg * hw, N=3 * C, K=C,
                                         groupnorm=dict(gamma=gam, beta=bet, groups=32, rows_per_image=hw))
        do = supra_attn.make_linear_desc(x=a_v, w=wo, bias=bo, y=y_v, M=nimg * hw, N=C, K=C, resid=xv)
        da = (supra_attn.Desc * nimg)()
        for i in range(nimg):
            r = i * hw
            da[i] = supra_attn.make_desc(q=qkv_v, k=qkv_v, v=qkv_v, out=a_v, Lq=hw, Lk=hw, H=1, D=C, ldq=3 * C,
                                         ldk=3 * C, ldv=3 * C, qOff=r * 3 * C, kOff=r * 3 * C + C, vOff=r * 3 * C + 2 * C,
                                         oOff=r * C)
        def vae_block():
            supra_attn._lib.check(enq(gpu.ctx, supra_attn._lib.C.byref(dq)), gpu.ctx)
            gpu.enqueue_batch(da)  # reads qkv: flushes the projection first
            supra_attn._lib.check(enq(gpu.ctx, supra_attn._lib.C.byref(do)), gpu.ctx)
            gpu.flush()

        flops = nimg * (2.0 * hw * C * 3 * C + 4.0 * hw * hw * C + 2.0 * hw * C * C)
        out["vae_block_8"] = {}
        for vname, (ms, kernels, per) in timed_variants(vae_block, [dq, do] + list(da)).items():
            out["vae_block_8"][vname] = {"ms": ms, "image_per_s": nimg / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12,
                                         "kernels": kernels}
            if vname == "fp32":  # (mixed kernels in the other variants: no single peak applies)
                out["vae_block_8"][vname]["frac_fp32_peak"] = flops / (ms / 1e3) / 1e12 / fp32_peak
        del xv, qkv_v, a_v, y_v

    if want("ctx_prep_2048"):
        # Cross-attention K/V preparation for configs[4]'s 2048 sequences (app/models/dit.js:137-144):
        # ctx_proj over every sequence's T5 rows at once, then the 14 blocks' kv projections as one
        # product with the stacked [14*1152, 576] weights (the cross attention reads its K/V in place).
        # Two flushes (the second reads the first's output); fp32 FFMA (a TF32 request runs the same).
        Lc = workload_lengths(1024, seed)
        rows = sum(Lc)
        ctx = torch.randn(rows * 768, device=dev, generator=g)
        wp = torch.randn(576 * 768, device=dev, generator=g) * 768 ** -0.5
        bp = torch.randn(576, device=dev, generator=g) * 0.1
        wkv = torch.randn(14 * 1152 * 576, device=dev, generator=g) * 576 ** -0.5
        bkv = torch.randn(14 * 1152, device=dev, generator=g) * 0.1
        p = torch.empty(rows * 576, device=dev)
        kv_all = torch.empty(rows * 14 * 1152, device=dev)
        d1 = supra_attn.make_linear_desc(x=ctx, w=wp, bias=bp, y=p, M=rows, N=576, K=768)
        d2 = supra_attn.make_linear_desc(x=p, w=wkv, bias=bkv, y=kv_all, M=rows, N=14 * 1152, K=576)
        enq = supra_attn.lib.supra_attn_enqueue_linear

        def prep():
            supra_attn._lib.check(enq(gpu.ctx, supra_attn._lib.C.byref(d1)), gpu.ctx)
            supra_attn._lib.check(enq(gpu.ctx, supra_attn._lib.C.byref(d2)), gpu.ctx)  # hazard: flushes d1 first
            gpu.flush()

        flops = 2.0 * rows * (768 * 576 + 576 * 14 * 1152)
        bytes_ = 4.0 * (rows * 768 + 576 * 768 + rows * 576 * 2 + 14 * 1152 * 576 + rows * 14 * 1152)
        tf_peak = float(peaks.get("bf16_tflops", 1590.0)) / 2.0
        out["ctx_prep_2048"] = {}
        for vname, (ms, kernels, per) in timed_variants(prep, [d1, d2]).items():
            r = {"ms": ms, "seq_per_s": 2048 / (ms / 1e3), "rows": rows, "tflops": flops / (ms / 1e3) / 1e12,
                 "gbs": bytes_ / (ms / 1e3) / 1e9, "frac_hbm": bytes_ / (ms / 1e3) / 1e9 / hbm, "kernels": kernels,
                 "ms_per_kernel": {k: round(v, 4) for k, v in sorted(per.items())}}
            if vname == "fp32":
                r["frac_fp32_peak"] = flops / (ms / 1e3) / 1e12 / fp32_peak
            else:  # issued TF32 MMA work (3 products per product in the split form) against the TF32 peak
                r["frac_tf32_peak"] = (3 if vname == "tf32x3" else 1) * flops / (ms / 1e3) / 1e12 / tf_peak
            out["ctx_prep_2048"][vname] = r
        del ctx, p, kv_all, wkv

    if want("dit_block_32"):
        # One whole DiT block (app/models/dit.js:161-194) for 32 images of 256 tokens with ragged
        # prompts: LayerNorm (+ adaLN modulation) folded into the qkv / q / fc1 products, the residual
        # updates in place with their gates, GELU(tanh) on fc1: 8 recorded calls, 6 products and the
        # two attentions, plus the LayerNorm statistics. fp32 throughout.
        nimg, N, D = 32, 256, 576
        Lb = workload_lengths(nimg, seed + 7)
        xb = torch.randn(nimg * N * D, device=dev, generator=g)
        modb = 0.5 * torch.randn(6 * D, device=dev, generator=g)
        wb = {}
        for nm, (o, i) in [("qkv", (3 * D, D)), ("proj", (D, D)), ("q", (D, D)), ("cproj", (D, D)),
                           ("fc1", (4 * D, D)), ("fc2", (D, 4 * D))]:
            wb[nm] = torch.randn(o * i, device=dev, generator=g) * i ** -0.5
            wb["b" + nm] = 0.1 * torch.randn(o, device=dev, generator=g)
        kvb = [torch.randn(L * 2 * D, device=dev, generator=g) for L in Lb]
        R = nimg * N
        qkv_b, a_b, q_b, c_b, f_b = (torch.empty(R * n, device=dev) for n in (3 * D, D, D, D, 4 * D))
        L = supra_attn.make_linear_desc
        lin = [
            L(x=xb, w=wb["qkv"], bias=wb["bqkv"], y=qkv_b, M=R, N=3 * D, K=D, layernorm=dict(mod=modb, shiftOff=0, scaleOff=D)),
            L(x=a_b, w=wb["proj"], bias=wb["bproj"], y=xb, M=R, N=D, K=D, resid=True, gate=modb, gOff=2 * D),
            L(x=xb, w=wb["q"], bias=wb["bq"], y=q_b, M=R, N=D, K=D, layernorm={}),
            L(x=c_b, w=wb["cproj"], bias=wb["bcproj"], y=xb, M=R, N=D, K=D, resid=True),
            L(x=xb, w=wb["fc1"], bias=wb["bfc1"], y=f_b, M=R, N=4 * D, K=D, act="gelu_tanh",
              layernorm=dict(mod=modb, shiftOff=3 * D, scaleOff=4 * D)),
            L(x=f_b, w=wb["fc2"], bias=wb["bfc2"], y=xb, M=R, N=D, K=4 * D, resid=True, gate=modb, gOff=5 * D),
        ]
        sa, ca = (supra_attn.Desc * nimg)(), (supra_attn.Desc * nimg)()
        for b in range(nimg):
            r = b * N * 3 * D
            sa[b] = supra_attn.make_desc(q=qkv_b, k=qkv_b, v=qkv_b, out=a_b, Lq=N, Lk=N, H=9, D=64, ldq=3 * D, ldk=3 * D,
                                         ldv=3 * D, qOff=r, kOff=r + D, vOff=r + 2 * D, oOff=b * N * D)
            ca[b] = supra_attn.make_desc(q=q_b, k=kvb[b], v=kvb[b], out=c_b, Lq=N, Lk=Lb[b], H=9, D=64, ldq=D,
                                         ldk=2 * D, ldv=2 * D, qOff=b * N * D, kOff=0, vOff=D, oOff=b * N * D)

        def block():
            e = lambda d: supra_attn._lib.check(enq(gpu.ctx, supra_attn._lib.C.byref(d)), gpu.ctx)
            e(lin[0])
            gpu.enqueue_batch(sa)
            e(lin[1])
            e(lin[2])
            gpu.enqueue_batch(ca)
            e(lin[3])
            e(lin[4])
            e(lin[5])
            gpu.flush()

        lin_flops = 2.0 * R * D * (3 * D + D + D + D + 4 * D + 4 * D)
        att_flops = 4.0 * N * D * (nimg * N + sum(Lb))
        flops = lin_flops + att_flops
        out["dit_block_32"] = {}
        tfp = float(peaks.get("bf16_tflops", 1590.0)) / 2.0  # TF32 dense peak: half of measured bf16
        for vname, (ms, kernels, per) in timed_variants(block, lin + list(sa) + list(ca)).items():
            r = {"ms": ms, "image_per_s": nimg / (ms / 1e3), "tflops": flops / (ms / 1e3) / 1e12,
                 "ms_per_kernel": {k: round(v, 4) for k, v in sorted(per.items())}}
            if vname == "fp32":
                r["frac_fp32_peak"] = flops / (ms / 1e3) / 1e12 / fp32_peak
            else:  # issued TF32 MMA work (3 products per product in the split form) against the TF32 peak
                r["frac_tf32_peak"] = (3 if vname == "tf32x3" else 1) * flops / (ms / 1e3) / 1e12 / tfp
            out["dit_block_32"][vname] = r
    return out


def rounded(x, digits: int = 5):
    """The JSON line's floats to `digits` significant digits (shorter lines, same information)."""
    if isinstance(x, float):
        return float(f"{x:.{digits}g}") if math.isfinite(x) else x
    if isinstance(x, dict):
        return {k: rounded(v, digits) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [rounded(v, digits) for v in x]
    return x


def compact_variant(v: dict) -> dict:
    """The figures of one tensor-core variant of the step, without its kernel list."""
    r = v.get("roofline") or {}
    return {"value": v["value"], "ms_per_step": v["ms_per_step"], "tflops": v["tflops"],
            "roofline": {k: r.get(k) for k in ("bound", "kernel", "achieved", "peak", "unit", "frac", "tensor_frac")},
            "parity": {k: v["parity"][k] for k in ("max_rel", "rel_l2", "n_checked")}, "tolerance": v["tolerance"],
            "sm_mhz": v["clocks"].get("sm_mhz"), "reasons": v["clocks"].get("reasons")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompts", type=int, default=1024)
    ap.add_argument("--seed", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-tf32", action="store_true", help="skip the tensor-core passes (tf32, tf32x3)")
    ap.add_argument("--no-sites", action="store_true", help="skip the per-call-site figures (configs[0..3])")
    ap.add_argument("--sites", default=None,
                    help="comma-separated call sites to run (dit_self_b2, dit_cross_128, t5_256, t5_256_table, vae, "
                         "vae_block_8, ctx_prep_2048, dit_block_32); default all")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import datetime

    # NCCL would print its version line on stdout, which must carry exactly one JSON line
    os.environ["NCCL_DEBUG"] = "WARN"

    import torch
    import torch.distributed as dist

    import supra_attn

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    # with several ranks, each keeps its host threads and pinned buffers beside its GPU (the
    # single-GPU run keeps every core: its CPU baseline uses them all)
    cpus_near_gpu = bind_to_gpu_cpus(torch, local_rank) if world > 1 else None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    # one compute stream for torch's copies/events and the library's launches
    torch.cuda.set_stream(torch.cuda.Stream(device=dev))

    # ---- workload shard --------------------------------------------------------------------
    lengths = workload_lengths(args.prompts, args.seed)
    mine = shard_prompts(lengths, world, rank)
    seqs = [s for p in mine for s in (2 * p, 2 * p + 1)]
    S = len(seqs)
    Ls = [lengths[s] for s in seqs]
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    qkv = torch.randn(S * TOKENS * 3 * DIM, device=dev, generator=gen)
    qx = torch.randn(S * TOKENS * DIM, device=dev, generator=gen)
    out_self = torch.empty(S * TOKENS * DIM, device=dev)
    out_cross = torch.empty(S * TOKENS * DIM, device=dev)
    kv_off = [0]
    for L in Ls:
        kv_off.append(kv_off[-1] + L * 2 * DIM)
    kv = [torch.randn(kv_off[-1], device=dev, generator=gen) for _ in range(BLOCKS)]  # cached per block

    gpu = supra_attn.GPU(local_rank, stream=torch.cuda.current_stream())
    self_d = (supra_attn.Desc * S)()
    for i in range(S):  # app/models/dit.js:172
        r = i * TOKENS * 3 * DIM
        self_d[i] = supra_attn.make_desc(q=qkv, k=qkv, v=qkv, out=out_self, Lq=TOKENS, Lk=TOKENS, H=N_HEADS,
                                         D=HEAD_DIM, ldq=3 * DIM, ldk=3 * DIM, ldv=3 * DIM, qOff=r, kOff=r + DIM,
                                         vOff=r + 2 * DIM, oOff=i * TOKENS * DIM)
    cross_d = []
    for b in range(BLOCKS):  # app/models/dit.js:184, K/V [L, 1152] cached per prompt and block
        arr = (supra_attn.Desc * S)()
        for i in range(S):
            arr[i] = supra_attn.make_desc(q=qx, k=kv[b], v=kv[b], out=out_cross, Lq=TOKENS, Lk=Ls[i], H=N_HEADS,
                                          D=HEAD_DIM, ldq=DIM, ldk=2 * DIM, ldv=2 * DIM, qOff=i * TOKENS * DIM,
                                          kOff=kv_off[i], vOff=kv_off[i] + DIM, oOff=i * TOKENS * DIM)
        cross_d.append(arr)

    flops_step = sum(4.0 * TOKENS * TOKENS * HEAD_DIM * N_HEADS + 4.0 * TOKENS * L * HEAD_DIM * N_HEADS for L in Ls) * BLOCKS
    flops_total = 0.0
    for L in lengths:
        flops_total += (4.0 * TOKENS * TOKENS + 4.0 * TOKENS * L) * HEAD_DIM * N_HEADS * BLOCKS

    # The only collective: after the timed steps rank 0 gathers every rank's output of the last step
    # (NCCL gather over NVLink, one per timed run, inside the timed region and timed on its own).
    # Prompts are independent, so nothing is exchanged between steps (app/pipeline.js:97-117 keeps
    # each prompt's K/V with its sampler).
    shard_max = max(len(shard_prompts(lengths, world, r)) for r in range(world)) * 2 * TOKENS * DIM
    send_buf = torch.empty(shard_max, device=dev) if world > 1 else None
    recv = [torch.empty(shard_max, device=dev) for _ in range(world)] if (world > 1 and rank == 0) else None
    gather_ms = []

    def gather_outputs(oc):
        if world == 1:
            return
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        send_buf[: oc.numel()].copy_(oc)
        dist.gather(send_buf, recv if rank == 0 else None, dst=0)
        g1.record()
        gather_ms.append((g0, g1))

    def step(sd=self_d, cd=cross_d):
        for b in range(BLOCKS):
            gpu.enqueue_batch(sd)
            gpu.flush()
            gpu.enqueue_batch(cd[b])
            gpu.flush()

    # ---- the checker: a sample of the step's outputs against the float64 oracle (outside the
    # timed regions). One sequence per L-bucket of 16 on each rank; the self-attention output of
    # the last block and its cross-attention output (block 13's K/V). ---------------------------------
    picks = []
    for lo in range(1, 129, 16):
        i = next((j for j, L in enumerate(Ls) if lo <= L < lo + 16 and j not in picks), None)
        if i is not None:
            picks.append(i)

    def check_step(oself, ocross, qkv_t=qkv, qx_t=qx):
        import numpy as np

        import oracle

        worst = [0.0, 0.0]
        kvl = kv[BLOCKS - 1]
        for i in picks:
            qr = qkv_t[i * TOKENS * 3 * DIM:(i + 1) * TOKENS * 3 * DIM].view(TOKENS, 3 * DIM).cpu().numpy()
            ref_s = oracle.attention_heads(qr[:, :DIM], qr[:, DIM:2 * DIM], qr[:, 2 * DIM:], N_HEADS)
            got_s = oself[i * TOKENS * DIM:(i + 1) * TOKENS * DIM].cpu().numpy()
            xr = qx_t[i * TOKENS * DIM:(i + 1) * TOKENS * DIM].view(TOKENS, DIM).cpu().numpy()
            kr = kvl[kv_off[i]:kv_off[i + 1]].view(-1, 2 * DIM).cpu().numpy()
            ref_c = oracle.attention_heads(xr, kr[:, :DIM], kr[:, DIM:], N_HEADS)
            got_c = ocross[i * TOKENS * DIM:(i + 1) * TOKENS * DIM].cpu().numpy()
            for got, ref in ((got_s, ref_s), (got_c, ref_c)):
                worst[0] = max(worst[0], oracle.max_rel(got, ref))
                worst[1] = max(worst[1], oracle.rel_l2(got, ref))
        t = torch.tensor(worst + [2.0 * len(picks)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t[:2], op=dist.ReduceOp.MAX)
            n = t[2:].clone()
            dist.all_reduce(n)
            t[2:] = n
        return {"max_rel": float(t[0]), "rel_l2": float(t[1]), "n_checked": int(t[2]),
                "what": "per rank one sequence per L-bucket of 16: the last block's self- and cross-attention "
                        "output vs the float64 oracle"}

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    gather_outputs(out_cross)
    torch.cuda.synchronize()

    # ---- timed region (device time, max over ranks) ---------------------------------------------
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local_rank).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    gpu.profile(True)
    gpu.profile_reset()
    launches0 = gpu.launch_count()
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.5)  # nvidia-smi is sampling before the timed region starts
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    clocks.mark_begin()
    ev0.record()
    for _ in range(args.steps):
        step()
    gather_outputs(out_cross)
    ev1.record()
    torch.cuda.synchronize()
    clocks.mark_end()
    time.sleep(0.3)
    clk = clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1)
    gather = None
    if world > 1:
        gt = torch.tensor([gather_ms[-1][0].elapsed_time(gather_ms[-1][1])], device=dev)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gather = {"ms": float(gt.item()), "bytes_to_rank0": 4 * TOKENS * DIM * 2 * args.prompts * (world - 1) // world,
                  "what": "NCCL gather of the last step's cross-attention output to rank 0, once per timed run, "
                          "inside the timed region"}
    parity = check_step(out_self, out_cross)
    launches = gpu.launch_count() - launches0
    prof = gpu.profile_report()
    gpu.profile(False)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    seq_calls = 2 * args.prompts * BLOCKS * 2 * args.steps
    value = seq_calls / (ms_max / 1e3)

    # ---- roofline of the dominant kernel ---------------------------------------------------------
    top = max(prof, key=lambda r: r["ms"]) if prof else None
    peaks = measured_peaks()
    sm_max = float(peaks.get("sm_max_mhz", 1965.0))
    fp32_peak = 148 * 128 * 2 * sm_max * 1e6 / 1e12  # TFLOP/s: SMs x FP32 lanes x FMA x clock
    roofline = None
    if top:
        achieved = top["flops"] / (top["ms"] / 1e3) / 1e12
        traffic = None
        tf = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tf):
            with open(tf) as f:
                tj = json.load(f).get(top["name"])
            if tj:  # ncu DRAM bytes per algorithmic byte, applied to this bench's launch
                traffic = tj["dram_bytes_per_alg_byte"] * top["bytes"] / top["count"]
        roofline = {"bound": "fp32", "kernel": top["name"], "achieved": achieved, "peak": fp32_peak,
                    "unit": "TFLOP/s", "frac": achieved / fp32_peak, "traffic": traffic,
                    "alg_bytes_per_launch": top["bytes"] / top["count"],
                    "alg_flops_per_launch": top["flops"] / top["count"],
                    "launch_ms": top["ms"] / top["count"],
                    "peak_source": f"nominal FP32 FFMA: 148 SMs x 128 lanes x 2 x {sm_max:.0f} MHz "
                                   "(MEASURED_PEAKS.json has no FP32 figure)",
                    "hbm_gbs_achieved": top["bytes"] / (top["ms"] / 1e3) / 1e9,
                    "hbm_peak_gbs": peaks.get("hbm_gbs")}
        sg = sgemm_tflops(torch, dev)  # after the timed regions: nothing of it is timed
        roofline["sgemm_tflops_measured"] = sg
        roofline["frac_of_sgemm"] = achieved / sg

    # ---- end to end through the public API with host buffers ------------------------------------
    # Every step uploads its inputs (Q/K/V of the self-attention, Q of the cross-attention) from
    # pinned host memory with supra_attn_upload and reads its result back with supra_attn_download
    # (fromArray / read of app/gpu/device.js). The copies go through two more library contexts on
    # their own streams, and the inputs and outputs are double-buffered, so step s computes while
    # step s+1's inputs arrive and step s-1's output leaves. All copies of all K steps lie inside
    # the timed region: it starts before the first upload and ends after the last read-back.
    e2e = None
    if not args.no_e2e:
        h_qkv = torch.empty(qkv.numel(), dtype=torch.float32, pin_memory=True)
        h_qx = torch.empty(qx.numel(), dtype=torch.float32, pin_memory=True)
        h_out = torch.empty(out_cross.numel(), dtype=torch.float32, pin_memory=True)
        h_qkv.copy_(qkv)
        h_qx.copy_(qx)

        sets = [(qkv, qx, out_cross, self_d, cross_d)]
        qkv2, qx2, oc2 = torch.empty_like(qkv), torch.empty_like(qx), torch.empty_like(out_cross)
        sd2 = (supra_attn.Desc * S)()
        for i in range(S):
            sd2[i] = self_d[i]
            sd2[i].q = sd2[i].k = sd2[i].v = qkv2.data_ptr()
        cd2 = []
        for b in range(BLOCKS):
            arr = (supra_attn.Desc * S)()
            for i in range(S):
                arr[i] = cross_d[b][i]
                arr[i].q = qx2.data_ptr()
                arr[i].out = oc2.data_ptr()
            cd2.append(arr)
        sets.append((qkv2, qx2, oc2, sd2, cd2))

        up_stream = torch.cuda.Stream(device=dev)
        down_stream = torch.cuda.Stream(device=dev)
        up_gpu = supra_attn.GPU(local_rank, stream=up_stream)
        down_gpu = supra_attn.GPU(local_rank, stream=down_stream)
        up, down = supra_attn.lib.supra_attn_upload, supra_attn.lib.supra_attn_download
        comp = torch.cuda.current_stream()

        # The first step's inputs and the last step's output cannot hide behind other steps: those
        # two steps run in CH sequence chunks, each chunk's compute waiting only for its own upload
        # and each chunk's read-back starting once it is computed. The steps between them run whole.
        CH = min(4, S)
        cb = [S * c // CH for c in range(CH + 1)]
        dsz = supra_attn._lib.C.sizeof(supra_attn.Desc)

        def sub(arr, a, b):  # descriptors a .. b-1 of a descriptor array (no copy)
            return (supra_attn.Desc * (b - a)).from_buffer(arr, a * dsz)

        chunk_descs = []  # [set][chunk] -> (self descs, [cross descs per block])
        for q_s, x_s, o_s, sd_s, cd_s in sets:
            chunk_descs.append([(sub(sd_s, cb[c], cb[c + 1]), [sub(cd_s[b], cb[c], cb[c + 1]) for b in range(BLOCKS)])
                                for c in range(CH)])
        q_row, x_row = TOKENS * 3 * DIM, TOKENS * DIM  # floats per sequence in qkv / qx / out

        def run_e2e(nsteps):
            """Uploads, steps and read-backs of `nsteps` steps, pipelined over the two sets."""
            computed = [None, None]  # the last event of the step that read each set
            arrived = [None, None]   # per set: the upload event of each chunk
            done_chunks = [None, None]

            def upload(s):
                q_s, x_s = sets[s % 2][0], sets[s % 2][1]
                if computed[s % 2] is not None:  # step s-2 read this set
                    up_stream.wait_event(computed[s % 2])
                evs = []
                for c in range(CH):
                    a, b = cb[c], cb[c + 1]
                    supra_attn._lib.check(up(up_gpu.ctx, q_s.data_ptr() + 4 * a * q_row, h_qkv.data_ptr() + 4 * a * q_row,
                                             (b - a) * q_row), up_gpu.ctx)
                    supra_attn._lib.check(up(up_gpu.ctx, x_s.data_ptr() + 4 * a * x_row, h_qx.data_ptr() + 4 * a * x_row,
                                             (b - a) * x_row), up_gpu.ctx)
                    ev = torch.cuda.Event()
                    ev.record(up_stream)
                    evs.append(ev)
                arrived[s % 2] = evs

            def compute(s, chunked):
                _, _, o_s, sd_s, cd_s = sets[s % 2]
                evs = []
                if chunked:
                    for c in range(CH):
                        comp.wait_event(arrived[s % 2][c])
                        sd_c, cd_c = chunk_descs[s % 2][c]
                        for b in range(BLOCKS):
                            gpu.enqueue_batch(sd_c)
                            gpu.flush()
                            gpu.enqueue_batch(cd_c[b])
                            gpu.flush()
                        ev = torch.cuda.Event()
                        ev.record(comp)
                        evs.append(ev)
                else:
                    comp.wait_event(arrived[s % 2][-1])
                    step(sd_s, cd_s)
                    ev = torch.cuda.Event()
                    ev.record(comp)
                    evs = [ev] * CH
                computed[s % 2] = evs[-1]
                done_chunks[s % 2] = evs

            def readback(s):  # blocks the host until the copies are issued
                o_p = sets[s % 2][2]
                for c in range(CH):
                    a, b = cb[c], cb[c + 1]
                    down_stream.wait_event(done_chunks[s % 2][c])
                    supra_attn._lib.check(down(down_gpu.ctx, h_out.data_ptr() + 4 * a * x_row,
                                               o_p.data_ptr() + 4 * a * x_row, (b - a) * x_row), down_gpu.ctx)

            upload(0)
            for s in range(nsteps + 1):
                if s + 1 < nsteps:  # issued before step s is recorded: it lands while step s computes
                    upload(s + 1)
                if s < nsteps:
                    compute(s, chunked=(s == 0 or s == nsteps - 1))
                if s > 0:  # read back step s-1 while step s computes
                    readback(s - 1)
            comp.wait_stream(down_stream)

        run_e2e(2)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        up_stream.wait_event(e0)
        down_stream.wait_event(e0)
        run_e2e(args.steps)
        gather_outputs(sets[(args.steps - 1) % 2][2])
        e1.record(comp)
        torch.cuda.synchronize()
        barrier()
        t2 = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        e2e = {"value": seq_calls / (float(t2.item()) / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": 4 * (qkv.numel() + qx.numel()) * world,
               "d2h_bytes_per_step": 4 * out_cross.numel() * world,
               "ms_per_step": float(t2.item()) / args.steps,
               "pipeline": ("inputs and outputs double-buffered; uploads, compute and read-backs on three streams; "
                            f"the first and last steps in {CH} sequence chunks"),
               "host_cpus": cpus_near_gpu or "all",
               "copy_volume": ("per step every rank uploads its sequences' self-attention q/k/v and cross-attention q "
                               "once and reads its cross-attention output back once; the 14 blocks of the step reuse "
                               "those inputs (in the model the projections produce them on the device), so the "
                               "copies are 1/14 of the bytes the step's attention reads")}
        up_gpu.close()
        down_gpu.close()
        del qkv2, qx2, oc2

    # ---- the tensor-core variants on the same workload: TF32 (its own tolerance, 2e-3) and the
    # split-precision 3xTF32 (the FP32 bar, 1e-5) ---------------------------------------------------
    def run_variant(code, dtype, tolerance, mma_per_flop):
        for arr in [self_d] + cross_d:
            for i in range(S):
                arr[i].variant = code
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        clocks_v = ClockSampler(uuid)
        gpu.profile(True)
        gpu.profile_reset()
        l0 = gpu.launch_count()
        barrier()
        torch.cuda.synchronize()
        clocks_v.start()
        time.sleep(0.5)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        clocks_v.mark_begin()
        t0.record()
        for _ in range(args.steps):
            step()
        gather_outputs(out_cross)
        t1.record()
        torch.cuda.synchronize()
        clocks_v.mark_end()
        time.sleep(0.3)
        clk_v = clocks_v.stop()
        barrier()
        lv = gpu.launch_count() - l0
        prof_v = gpu.profile_report()
        gpu.profile(False)
        tt = torch.tensor([t0.elapsed_time(t1)], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_v = float(tt.item())
        top = max(prof_v, key=lambda r: r["ms"]) if prof_v else None
        roof = None
        if top:
            gbs = top["bytes"] / (top["ms"] / 1e3) / 1e9
            hbm = float(peaks.get("hbm_gbs", 6650.0))
            tf_peak = float(peaks.get("bf16_tflops", 1590.0)) / 2.0  # TF32 dense rate is half of bf16
            traffic = None
            tf = os.path.join(ROOT, "profiles", "traffic.json")
            if os.path.exists(tf):
                with open(tf) as f:
                    tj = json.load(f).get(top["name"])
                if tj:
                    traffic = tj["dram_bytes_per_alg_byte"] * top["bytes"] / top["count"]
            issued = mma_per_flop * top["flops"] / (top["ms"] / 1e3) / 1e12
            roof = {"bound": "hbm", "kernel": top["name"], "achieved": gbs, "peak": hbm, "unit": "GB/s",
                    "frac": gbs / hbm, "traffic": traffic,
                    "alg_bytes_per_launch": top["bytes"] / top["count"],
                    "launch_ms": top["ms"] / top["count"],
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6.65 TB/s",
                    "tensor_tflops": issued, "tensor_peak_tflops": tf_peak, "tensor_frac": issued / tf_peak,
                    "tensor_peak_source": "half of MEASURED_PEAKS.json bf16_tflops (TF32 dense = bf16 dense / 2)"}
            if mma_per_flop > 1:  # tensor-bound: report the tensor roofline as the bound
                roof.update({"bound": "tensor", "achieved": issued, "peak": tf_peak, "unit": "TFLOP/s",
                             "frac": issued / tf_peak, "hbm_gbs_achieved": gbs, "hbm_peak_gbs": hbm,
                             "note": f"{mma_per_flop} TF32 MMA FLOPs per algorithmic FLOP (hi/lo split)"})
        res = {"value": seq_calls / (ms_v / 1e3), "unit": UNIT, "ms_per_step": ms_v / args.steps, "dtype": dtype,
               "tolerance": tolerance, "tflops": flops_total * args.steps / (ms_v / 1e3) / 1e12, "gpu_launches": lv,
               "clocks": clk_v, "roofline": roof, "kernels": prof_v, "parity": check_step(out_self, out_cross)}
        for arr in [self_d] + cross_d:
            for i in range(S):
                arr[i].variant = supra_attn._lib.FP32
        return res

    variants = {}
    if not args.no_tf32:
        variants["tf32"] = run_variant(supra_attn._lib.TF32, "tf32 operands, f32 accumulate",
                                       "max|d|/max|ref| and rel-L2 <= 2e-3", 1)
        variants["tf32x3"] = run_variant(supra_attn._lib.TF32X3,
                                         "f32 operands split hi+lo into 3 TF32 products, f32 accumulate",
                                         "max|d|/max|ref| and rel-L2 <= 1e-5 (the FP32 bar)", 3)

    sites = None
    if not args.no_sites:  # (every rank: with N > 1 each runs its share of a site's batch)
        sites = measure_call_sites(gpu, torch, dev, args.seed, only=set(args.sites.split(",")) if args.sites else None,
                                   cpu_reps=0 if (args.no_cpu or world > 1) else 3, rank=rank, world=world, dist=dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_leg(lengths, args.seed, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) Q/K/V, L~U{1..128})",
            "config": workload_config(args, world),
            "tflops": flops_total * args.steps / (ms_max / 1e3) / 1e12,
            "gpu_launches": launches,
            "clocks": clk,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "parity": parity,
            "gather": gather,
            "kernels": prof,
            "variants_detail": variants,
            "call_sites": sites,
            # last, so that a reader of the line's tail sees the tensor-core step figures
            "variants": {k: compact_variant(v) for k, v in variants.items()},
        }
        print(json.dumps(rounded(line)), flush=True)

    gpu.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
