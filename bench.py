"""Benchmark of the speculative verify step on B200.

One step = one batched verify pass over 64 sequences per GPU, the workload
BASELINE.json's metric is quoted on (config 1), run by
kyro_b200.step.VerifyStep:
  verify attention with RoPE of the new q/k rows at context_len + j and
  the paged store of the new K/V in its prologue (Llama-3-8B layer: Hq 32,
  Hkv 8, D 128, bf16 paged KV, block 16, context ~ U[512, 4096]) -> acceptance
  sampling (k = 5, V = 128256, fp32, T = 1.0) -> kv_commit of the accepted
  slots and kv_reserve of the next step's k+1 slots (the decode-loop form:
  kyro_spec_accept_commit runs the commit beside the acceptance's final
  pass and the reserve in the same launch as the commit).
Every timed step first restores the KV bookkeeping state (one device copy),
so every step sees the same context lengths; the step is captured once as
a CUDA graph and replayed, so every replay also reuses the Philox step
number of the capture (the work and its timing do not depend on the draws).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; sequences are sharded by
rank (weak scaling, no collective on the data path).  `value` is verified
positions per second over all ranks, device-timed with CUDA events, max
over ranks.  `e2e` is the same metric through the public step API with host
buffers: each step copies its inputs from pinned host memory and reads its
results back.  `--impl reference` times the CPU restatement of the
reference path (oracle/; the reference itself is Rust and cannot be built
here) on the host cores.

Besides the headline, the default run adds (outside the headline's timed
region, each timed on its own):
  config0   acceptance only (B 8, k 4, V 32000): launch-bound
  config2   the tree verify step (64-node tree, context 8192)
  tp_accept config 3's vocabulary-sharded acceptance (B 256, k 8,
            V 128256 over the N ranks as one tensor-parallel group, both
            exchange transports), after a bit-exact check of the sharded
            kernels against tests/golden/tp_accept_golden.json; at N = 1 the
            single-GPU acceptance of the same rows (the strong-scaling base)
  per_rank  every rank's context tokens, bytes and kernel times (N > 1)
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "spec-verify tokens/s (attn+accept)"
UNIT = "verified positions/s"
# untimed steps after the timed region that carry CUDA events around the kernels
PER_KERNEL_STEPS = 10
TP_GOLDEN = os.path.join(ROOT, "tests", "golden", "tp_accept_golden.json")


def workload_desc(cfg, n):
    return {
        "workload": "config1: chain verify (RoPE + paged KV store, paged attention, accept, KV "
                    "commit), Llama-3-8B layer Hq32/Hkv8/D128 bf16 KV block16, ctx U[512,4096], "
                    "k=5 (+1), V=128256 fp32, T=1.0",
        "batch_per_gpu": cfg.batch, "global_batch": cfg.batch * n, "k": cfg.k,
        "vocab": cfg.vocab, "kv_blocks_per_gpu": cfg.num_blocks,
        "parallelism": f"batch-sharded x{n} (no collective)",
        "l2": "inputs larger than L2 each step (~0.6 GB KV + 0.36 GB logits)",
    }


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def load_traffic():
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


class NvmlClockSampler:
    """SM clock and clock-event reasons sampled through NVML every ~2 ms
    while the timed region runs (reads only; changes no GPU setting)."""

    def __init__(self, gpu_index):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        self.samples = []
        self.stop_flag = threading.Event()

    def _run(self):
        nv = self.nv
        while not self.stop_flag.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        while not self.samples and self.t.is_alive():
            time.sleep(0.001)

    def stop(self):
        self.stop_flag.set()
        self.t.join(timeout=2)
        nv = self.nv
        if not self.samples:
            return None
        names = {nv.nvmlClocksEventReasonHwSlowdown: "hw_slowdown",
                 nv.nvmlClocksEventReasonHwThermalSlowdown: "hw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwThermalSlowdown: "sw_thermal_slowdown",
                 nv.nvmlClocksEventReasonSwPowerCap: "sw_power_cap"}
        reasons = sorted({n for _, r in self.samples for bit, n in names.items() if r & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "nvml"}


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r)
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows)}


def start_clocks(rank, local):
    """The clock sampler of rank 0 (None elsewhere), on the physical GPU."""
    if rank != 0:
        return None
    phys = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if vis:
        ids = [v.strip() for v in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            phys = int(ids[local])
    try:
        clocks = NvmlClockSampler(phys)
    except Exception:
        clocks = ClockSampler(phys)
    clocks.start()
    return clocks


def bind_numa_local(local):
    """Restrict this process to the CPUs next to its GPU (read from sysfs
    through the GPU's PCI bus id), so that pinned host buffers allocated
    afterwards land on the GPU's NUMA node.  Returns (node, cpu count) or
    None when the topology is not available."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(local)
        bus = pynvml.nvmlDeviceGetPciInfo(h).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        dev = "/sys/bus/pci/devices/" + bus.lower()[-12:]
        with open(dev + "/local_cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        node = -1
        try:
            with open(dev + "/numa_node") as f:
                node = int(f.read().strip())
        except Exception:
            pass
        return {"numa_node": node, "cpus": len(cpus)}
    except Exception:
        return None


class KvStateSnapshot:
    """The KV bookkeeping tensors of a PagedState (block table, context
    lengths, free stack and top, ref counts) moved into one device buffer,
    with a copy of their starting values.  Every timed step starts from the
    same state, and resetting it is one device-to-device copy."""

    NAMES = ("block_table", "context_lens", "free_stack", "free_top", "ref_counts")

    def __init__(self, st):
        import torch
        layout, off = [], 0
        for n in self.NAMES:
            t = getattr(st, n)
            nbytes = t.numel() * t.element_size()
            layout.append((n, off, nbytes, t.dtype, tuple(t.shape)))
            off += (nbytes + 255) // 256 * 256
        self.buf = torch.empty(off, dtype=torch.uint8, device=st.block_table.device)
        self._views = {}
        for n, o, nb, dt, sh in layout:
            v = self.buf[o:o + nb].view(dt).view(sh)
            v.copy_(getattr(st, n))
            setattr(st, n, v)
            self._views[n] = (o, nb, dt, sh)
        self.snap = self.buf.clone()

    def restore(self):
        self.buf.copy_(self.snap, non_blocking=True)

    def initial(self, name):
        o, nb, dt, sh = self._views[name]
        return self.snap[o:o + nb].view(dt).view(sh)


def kv_of(st):
    from kyro_b200.step import KVState
    return KVState(st.block_table, st.context_lens, st.free_stack, st.free_top, st.ref_counts,
                   st.k_cache, st.v_cache)


def init_ranks(args, timeout_s=120):
    """(world, rank, local, device), with the NCCL process group up for N > 1."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=dev)
    return world, rank, local, dev


def max_over_ranks(vals, world, dev):
    import torch
    import torch.distributed as dist
    if world == 1:
        return [float(v) for v in vals]
    t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def gather_rows(vals, world, dev):
    """Every rank's row of floats, on every rank: [world][len(vals)]."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
    if world == 1:
        return [t.cpu().tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.cpu().tolist() for o in out]


def acceptance_stats(acc, k):
    """(mean accepted fraction a/k, per-token acceptance rate): the second
    counts accepted drafts over accept tests run (a test runs at every
    position up to the first rejection)."""
    a = acc.detach().cpu().numpy().astype(np.int64)
    tests = np.where(a < k, a + 1, k)
    return float(a.mean() / k) if k else 0.0, float(a.sum() / max(1, tests.sum()))


# --------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    import torch.distributed as dist

    from kyro_b200.step import VerifyStep
    from kyro_b200.verify import Context, sample_tokens
    from kyro_b200.workloads import CONFIG1, accept_inputs, chain_bytes_per_step, paged_state

    world, rank, local, dev = init_ranks(args)
    numa = bind_numa_local(local)
    cfg = CONFIG1
    ctx = Context(local)
    seq_offset = rank * cfg.batch
    st = paged_state(cfg, dev, seed=1000 + rank)
    tgt, drf = accept_inputs(cfg.batch, cfg.k, cfg.vocab, dev, seed=2000 + rank)
    drafts, _ = sample_tokens(ctx, drf, cfg.temperature, seed=0, seq_offset=seq_offset)
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    nq = cfg.num_query
    k_new = torch.randn(cfg.batch, nq, cfg.num_kv_heads, cfg.head_dim, generator=g, device=dev,
                        dtype=torch.bfloat16)
    v_new = torch.randn(cfg.batch, nq, cfg.num_kv_heads, cfg.head_dim, generator=g, device=dev,
                        dtype=torch.bfloat16)
    # The decode-loop form of the step: the commit also reserves the next
    # step's k + 1 slots (kyro_spec_accept_commit), so the state every step
    # starts from has its slots reserved.  Every step starts from that same
    # state, so each step sees the same context lengths; the reset is one
    # device-to-device copy (~0.5 MB).
    from kyro_b200.verify import kv_reserve
    kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
               st.ref_counts, cfg.block_size)
    kvsnap = KvStateSnapshot(st)
    kv = kv_of(st)
    vstep = VerifyStep(ctx, cfg.batch, cfg.k, cfg.num_heads, kv, cfg.vocab, cfg.block_size,
                       temperature=cfg.temperature, seed=0, seq_offset=seq_offset,
                       rope_theta=10000.0)
    ev = {}

    def step(i, events=None):
        kvsnap.restore()
        return vstep(kv, st.q, k_new, v_new, tgt, drf, drafts, step=i, events=events,
                     reserve=False, reserve_next=nq)

    # the step runs on a side stream as a CUDA graph (captured once after the
    # warm-up steps); the library context is bound to that stream
    side = torch.cuda.Stream(dev)
    graph = None
    with torch.cuda.stream(side):
        ctx.bind_stream()
        for i in range(args.warmup):
            step(i)
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step(args.warmup)
            for _ in range(3):
                graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = start_clocks(rank, local)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        t0.record(side)
        for i in range(args.warmup, args.warmup + args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(i)
        t1.record(side)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms_rank = t0.elapsed_time(t1)
    # per-kernel times from separate steps with events around attention and
    # acceptance (events between kernels would perturb the timed steps)
    with torch.cuda.stream(side):
        for i in range(PER_KERNEL_STEPS):
            _, _, acc, _, _ = step(args.warmup + args.steps + i, events=ev)
    torch.cuda.synchronize()
    del graph
    ctx.bind_stream()  # back to the default stream for the end-to-end run
    status = ctx.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the timed region")

    # algorithmic bytes per step, from the context lengths every step starts from
    lens0 = kvsnap.initial("context_lens").cpu().numpy()
    per = chain_bytes_per_step(lens0, cfg, separate_rope=not vstep.fused_rope)
    att_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["attention"]]))
    acc_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["accept"]]))
    rows = gather_rows([rank, int(lens0.sum()), per["attention"], per["accept"], att_ms, acc_ms,
                        ms_rank / args.steps], world, dev)
    ms = max(r[6] for r in rows) * args.steps
    # with RoPE fused, the attention launch also reads the new K/V rows and
    # stores them in their paged slots
    att_bytes = float(per["attention"] + (per["new_rows"] if vstep.fused_rope else 0))
    acc_bytes = float(per["accept"])
    peak, peak_kind = load_peaks()
    traffic = load_traffic()
    if att_ms >= acc_ms:
        dom, dbytes, dms = "verify_attention_kernel", att_bytes, att_ms
    else:
        dom, dbytes, dms = "accept_stats_kernel", acc_bytes, acc_ms
    achieved = dbytes / (dms * 1e-3) / 1e9
    units = cfg.batch * nq * world * args.steps
    value = units / (ms * 1e-3)
    step_bytes = float(per["total"])
    frac_acc, per_token = acceptance_stats(acc, cfg.k)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; BASELINE config 1 shapes and distributions)",
        "config": workload_desc(cfg, world),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic.get(dom.split(" ")[0])},
        "kernels": {
            "verify_attention": {"ms": att_ms, "algorithmic_bytes": att_bytes,
                                 "GBps": att_bytes / (att_ms * 1e-3) / 1e9,
                                 "frac": att_bytes / (att_ms * 1e-3) / 1e9 / peak},
            "accept": {"ms": acc_ms, "algorithmic_bytes": acc_bytes,
                       "GBps": acc_bytes / (acc_ms * 1e-3) / 1e9,
                       "frac": acc_bytes / (acc_ms * 1e-3) / 1e9 / peak},
            "step_algorithmic_bytes": step_bytes,
            "step_frac_of_hbm": step_bytes / (ms / args.steps * 1e-3) / 1e9 / peak,
        },
        "timing": "CUDA graph replays of the step" if not args.no_graph else "stream launches",
        "mean_accepted_fraction": frac_acc,
        "per_token_acceptance": per_token,
        "gpu_launches": vstep.launches(reserve=False) * args.steps,
        "clocks": clk,
    }
    if world > 1:
        slow = max(rows, key=lambda r: r[6])
        line["per_rank"] = {
            "fields": ["rank", "context_tokens", "attention_bytes", "accept_bytes", "attention_ms",
                       "accept_ms", "step_ms"],
            "rows": rows,
            "slowest_rank": int(slow[0]), "slowest_context_tokens": int(slow[1]),
            "note": "each rank draws its own contexts (seed 1000 + rank); the job's step time is "
                    "the slowest rank's"}
        line["config"]["attention_bytes_all_ranks"] = sum(r[2] for r in rows)
    if not args.no_e2e:
        line["e2e"] = run_e2e(args, ctx, cfg, st, kv, vstep, tgt, drf, drafts, k_new, v_new,
                              world, dev, kvsnap.restore, numa)
    if not args.no_extras:
        line["extras"] = run_extras(args, ctx, world, rank, local, dev)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, st, tgt, drf, drafts, k_new, v_new, args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, ctx, cfg, st, kv, vstep, tgt, drf, drafts, k_new, v_new, world, dev, restore,
            numa):
    """The same step through the public step API with host buffers: inputs
    copied from pinned host memory each step, results read back each step."""
    import torch
    h = {n: t.cpu().pin_memory() for n, t in
         dict(q=st.q, k_new=k_new, v_new=v_new, tgt=tgt, drf=drf, drafts=drafts).items()}
    d = {n: torch.empty_like(t, device=dev) for n, t in h.items()}
    nq = cfg.num_query
    out_h = {n: torch.empty(s, dtype=torch.int32).pin_memory()
             for n, s in dict(acc=(cfg.batch,), toks=(cfg.batch, nq), num=(cfg.batch,)).items()}
    stream = torch.cuda.current_stream(dev)
    h2d = sum(t.numel() * t.element_size() for t in h.values())
    d2h = sum(t.numel() * t.element_size() for t in out_h.values())
    steps = max(3, min(args.steps, 10))

    def step(i):
        restore()
        for n in h:
            d[n].copy_(h[n], non_blocking=True)
        _, _, acc, toks, num = vstep(kv, d["q"], d["k_new"], d["v_new"], d["tgt"], d["drf"],
                                     d["drafts"], step=1000 + i, reserve=False,
                                     reserve_next=cfg.num_query)
        out_h["acc"].copy_(acc, non_blocking=True)
        out_h["toks"].copy_(toks, non_blocking=True)
        out_h["num"].copy_(num, non_blocking=True)
        stream.synchronize()  # the caller reads the emitted tokens

    step(0)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        step(1 + i)
    t1.record(stream)
    torch.cuda.synchronize()
    ms_rank = t0.elapsed_time(t1)
    rows = gather_rows([ms_rank / steps, h2d / (ms_rank / steps * 1e-3) / 1e9], world, dev)
    ms = max(r[0] for r in rows) * steps
    value = cfg.batch * nq * world * steps / (ms * 1e-3)
    out = {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "steps": steps, "ms_per_step": ms / steps,
           "h2d_GBps_per_rank": [r[1] for r in rows],
           "h2d_GBps_all_ranks": h2d * world / (ms / steps * 1e-3) / 1e9,
           "limit": "the logits (366 MB per step and rank) cross the host link and host memory; "
                    "with N ranks the host's memory bandwidth is shared",
           "host_binding": numa}
    return out


# ------------------------------------------------------------------ extras
def run_extras(args, ctx, world, rank, local, dev):
    """Configs 0, 2, 3 and 4 on the same ranks, each with its own short timed
    region (max over ranks).  Every rank takes the same collective steps."""
    out = {}
    out["config0"] = extra_config0(ctx, world, dev)
    out["config2"] = tree_measure(ctx, world, rank, dev, steps=args.extra_steps, warmup=3)
    out["tp_accept"] = tp_measure(world, rank, local, dev, steps=args.extra_steps, warmup=3)
    out["config4"] = extra_config4(args, world, rank, local, dev)
    return out


def extra_config4(args, world, rank, local, dev):
    """Config 4 (the end-to-end speculative step, bench.py --config 4) in
    short: a few graph-replayed steps, the step time and its parts."""
    import types
    a = types.SimpleNamespace(warmup=3, steps=max(3, args.extra_steps // 4), no_graph=False,
                              requests=None, target_layers=None)
    m = e2e_model_measure(a, world, rank, local, dev)
    cfg, k, ms = m["cfg"], m["k"], m["ms"]
    return {"workload": "config4: end-to-end speculative step, 16-layer Llama target + 2-layer "
                        "draft, k 4, T 0.7, 512 requests split over the ranks (strong scaling)",
            "steps": a.steps, "ms_per_step": ms / a.steps,
            "positions_per_s": cfg.requests * (k + 1) * a.steps / (ms * 1e-3),
            "emitted_tokens_per_s": m["emitted"] / (ms * 1e-3),
            "parts_ms_per_step": m["part"],
            "target_attention": {"GBps": m["att_gbs"], "frac_hbm": m["att_gbs"] / m["peak"]},
            "accept": {"GBps": m["acc_gbs"], "frac_hbm": m["acc_gbs"] / m["peak"]},
            "timing": "CUDA graph replays of the step, max over ranks"}


def extra_config0(ctx, world, dev, steps=200):
    """Config 0: acceptance only (B 8, k 4, V 32000, T 1.0), CUDA graph
    replays.  9.2 MB per call: launch-bound, reported as such."""
    import torch
    from kyro_b200.verify import sample_tokens, spec_accept
    from kyro_b200.workloads import CONFIG0, accept_inputs
    B, k, V = CONFIG0["batch"], CONFIG0["k"], CONFIG0["vocab"]
    tgt, drf = accept_inputs(B, k, V, dev, seed=0)
    drafts, _ = sample_tokens(ctx, drf, 1.0, seed=0)
    acc = torch.empty(B, dtype=torch.int32, device=dev)
    toks = torch.empty(B, k + 1, dtype=torch.int32, device=dev)
    num = torch.empty(B, dtype=torch.int32, device=dev)
    side = torch.cuda.Stream(dev)
    with torch.cuda.stream(side):
        ctx.bind_stream()
        for i in range(3):
            spec_accept(ctx, tgt, drf, drafts, seed=0, step=i, out=(acc, toks, num, None))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for i in range(10):  # ten calls per replay
                spec_accept(ctx, tgt, drf, drafts, seed=0, step=i, out=(acc, toks, num, None))
        graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        t0.record(side)
        for _ in range(steps // 10):
            graph.replay()
        t1.record(side)
    torch.cuda.synchronize()
    del graph
    ctx.bind_stream()
    us = max_over_ranks([t0.elapsed_time(t1) / steps * 1e3], world, dev)[0]
    bytes_ = (2 * k + 1) * V * 4 * B
    return {"workload": "config0: acceptance only, B 8, k 4, V 32000, T 1.0 (per rank)",
            "us_per_call": us, "positions_per_s": B * (k + 1) * world / (us * 1e-6),
            "GBps": bytes_ / (us * 1e-6) / 1e9, "algorithmic_bytes": bytes_,
            "timing": "CUDA graph of 10 back-to-back calls, max over ranks",
            "bound": "launch latency (9.2 MB per call)"}


def tree_measure(ctx, world, rank, dev, steps, warmup):
    """Config 2 on this rank (batch-sharded): KV reserve and write of the 64
    tree nodes, paged attention of 64 query heads over 8 KV heads (context
    8192) under the ancestor mask, multi-candidate acceptance over vocabulary
    32000, and the tree commit of the accepted path."""
    import torch
    from kyro_b200.verify import (kv_commit_tree, kv_reserve, kv_write, spec_accept_tree,
                                  verify_attention)
    from kyro_b200.workloads import CONFIG2, bfs_tree, paged_state, tree_mask_bits
    cfg = CONFIG2
    B, N, V = cfg.batch, cfg.num_query, cfg.vocab
    st = paged_state(cfg, dev, seed=8000 + rank)
    par = bfs_tree(N)
    pars = torch.from_numpy(np.broadcast_to(par[None], (B, N)).copy()).to(dev)
    mask = torch.from_numpy(np.broadcast_to(tree_mask_bits(par)[None], (B, N)).copy()).to(dev)
    g = torch.Generator(device=dev).manual_seed(8100 + rank)
    tgt = torch.randn(B, N, V, generator=g, device=dev) * cfg.logit_std
    drf = tgt + torch.randn(B, N, V, generator=g, device=dev) * cfg.draft_noise
    # each child's token sampled from its parent's draft distribution
    tok = torch.zeros(B, N, dtype=torch.int32, device=dev)
    q = torch.softmax(drf[:, torch.from_numpy(par[1:]).long().to(dev), :] / cfg.temperature, dim=2)
    tok[:, 1:] = torch.multinomial(q.reshape(-1, V), 1, generator=g).reshape(B, N - 1).int()
    del q
    k_new = torch.randn(B, N, cfg.num_kv_heads, cfg.head_dim, generator=g, device=dev,
                        dtype=torch.bfloat16)
    v_new = torch.randn_like(k_new)
    attn_out = torch.empty_like(st.q)
    ok = torch.empty(B, dtype=torch.int32, device=dev)
    kvsnap = KvStateSnapshot(st)
    stream = torch.cuda.current_stream(dev)
    ev = {"attention": [], "accept": []}
    ctx.bind_stream()

    def step(i, timed):
        kvsnap.restore()
        kv_reserve(ctx, N, st.block_table, st.context_lens, st.free_stack, st.free_top,
                   st.ref_counts, cfg.block_size, out_ok=ok)
        kv_write(ctx, k_new, v_new, st.block_table, st.context_lens, st.k_cache, st.v_cache,
                 cfg.block_size)
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                         tree_mask=mask, out=attn_out)
        if timed:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
        path, plen, _, _ = spec_accept_tree(ctx, tgt, drf, tok, pars, temperature=cfg.temperature,
                                            seed=0, step=i, seq_offset=rank * B)
        if timed:
            e2 = torch.cuda.Event(enable_timing=True)
            e2.record(stream)
            ev["attention"].append((e0, e1))
            ev["accept"].append((e1, e2))
        kv_commit_tree(ctx, N, path, plen, [st.k_cache], [st.v_cache], st.block_table,
                       st.context_lens, st.free_stack, st.free_top, st.ref_counts, cfg.block_size)
        return plen

    for i in range(warmup):
        step(i, False)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    plens = [step(i, False) for i in range(warmup, warmup + steps)]
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    # per-kernel times from separate steps, so that no event sits between the
    # chained launches of the timed ones
    for i in range(warmup + steps, warmup + steps + PER_KERNEL_STEPS):
        step(i, True)
    torch.cuda.synchronize()
    att_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["attention"]]))
    acc_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["accept"]]))
    ms, att_ms, acc_ms = max_over_ranks([ms, att_ms, acc_ms], world, dev)
    status = ctx.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the config-2 steps")
    peak, _ = load_peaks()
    kv_bytes = B * (cfg.ctx_max + N) * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    flops = 4.0 * B * cfg.num_heads * N * cfg.head_dim * (cfg.ctx_max + N)
    acc_bytes = 2 * B * N * V * 4
    tpk = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpk = float(json.load(f)["bf16_tflops"])
    except Exception:
        tpk = 1590.0
    return {
        "workload": "config2: tree verify (paged attention under a 64-node ancestor mask + "
                    "multi-candidate acceptance + tree commit), Hq64/Hkv8/D128 bf16, ctx 8192, "
                    "tree 4,4,4 cut to 64, V 32000 fp32, T 1.0, B 32 per rank",
        "nodes_per_s": B * N * world * steps / (ms * 1e-3), "ms_per_step": ms / steps,
        "steps": steps, "mean_path_len": float(torch.stack(plens).float().mean().item()),
        "attention": {"ms": att_ms, "TFLOPs": flops / (att_ms * 1e-3) / 1e12,
                      "tensor_frac_of_burst": flops / (att_ms * 1e-3) / 1e12 / tpk,
                      "kv_GBps": kv_bytes / (att_ms * 1e-3) / 1e9, "flops": flops},
        "accept": {"ms": acc_ms, "bytes": acc_bytes, "GBps": acc_bytes / (acc_ms * 1e-3) / 1e9,
                   "hbm_frac": acc_bytes / (acc_ms * 1e-3) / 1e9 / peak},
        "timing": "stream launches, max over ranks",
    }


def _tp_parity(ctx, world, rank, dev):
    """The sharded kernels on this group against the oracle's outputs for
    num_shards = world (tests/golden/tp_accept_golden.json): True iff every
    case matches bit for bit on this rank."""
    import torch
    from kyro_b200.verify import spec_accept, spec_accept_tp
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    from make_tp_golden import inputs
    with open(TP_GOLDEN) as f:
        fixture = json.load(f)
    ok = True
    for case in fixture["cases"]:
        B, k, V, mode, T, seed = (case[n] for n in ("B", "k", "V", "mode", "T", "seed"))
        want = case["shards"].get(str(world))
        if want is None:
            return None
        tgt, drf = inputs(B, k, V, seed)
        Vs = V // world
        ts = torch.from_numpy(tgt[:, :, rank * Vs:(rank + 1) * Vs].copy()).to(dev)
        ds = torch.from_numpy(drf[:, :, rank * Vs:(rank + 1) * Vs].copy()).to(dev)
        drafts = torch.tensor(case["drafts"], dtype=torch.int32).reshape(B, k).to(dev)
        if world == 1:
            acc, toks, num, probs = spec_accept(ctx, ts, ds if mode == 0 else None, drafts,
                                                mode=mode, temperature=T, seed=seed,
                                                want_probs=mode == 0)
        else:
            acc, toks, num, probs = spec_accept_tp(ctx, ts, ds if mode == 0 else None, drafts, V,
                                                   mode=mode, temperature=T, seed=seed,
                                                   want_probs=mode == 0)
        torch.cuda.synchronize(dev)
        ok &= acc.cpu().tolist() == want["accept_len"]
        ok &= toks.cpu().tolist() == want["tokens"]
        ok &= num.cpu().tolist() == want["num_tokens"]
        if mode == 0:
            ok &= probs.cpu().numpy().view(np.uint32).tolist() == want["probs_bits"]
    return bool(ok)


def tp_measure(world, rank, local, dev, steps, warmup):
    """Config 3 over the N ranks as one tensor-parallel group: parity against
    the golden fixture, then the timed step (acceptance of B 256 x k 8 over
    V 128256 split N ways, plus KV reserve/commit on a 32768-block table) for
    each exchange transport.  At N = 1: the single-GPU acceptance of the
    same rows."""
    import torch
    import torch.distributed as dist
    from kyro_b200.verify import Context, kv_commit, kv_reserve, spec_accept_tp, tp_unique_id
    from kyro_b200.workloads import CONFIG3, paged_state
    cfg = CONFIG3
    B, k, V, T = cfg.batch, cfg.k, cfg.vocab, cfg.temperature
    Vs = V // world
    transports = ["single"] if world == 1 else ["peer", "nccl"]
    res = {"workload": f"config3: vocabulary-sharded acceptance (B 256, k 8, V 128256 over "
                       f"{world} rank(s), T 0.8) + KV reserve/commit on a 32768-block table",
           "columns_per_rank": Vs, "scaling": "strong (the same rows split over the ranks)"}

    def shard(r):  # rank r's columns of the (never materialised) full logits
        g = torch.Generator(device=dev).manual_seed(5000 + r)
        t = torch.randn(B, k + 1, Vs, generator=g, device=dev) * cfg.logit_std
        d = t[:, :k, :] + torch.randn(B, k, Vs, generator=g, device=dev) * cfg.draft_noise
        return t.contiguous(), d.contiguous()

    tgt, drf = shard(rank)
    drafts = torch.zeros(B, k, dtype=torch.int32, device=dev)
    if rank == 0:
        full = torch.cat([shard(r)[1] for r in range(world)], dim=2)
        g = torch.Generator(device=dev).manual_seed(6000)
        probs = torch.softmax(full.reshape(B * k, V) / T, dim=1)
        drafts.copy_(torch.multinomial(probs, 1, generator=g).reshape(B, k).int())
        del full, probs
    if world > 1:
        dist.broadcast(drafts, 0)
    st = paged_state(cfg, dev, seed=7000, fill_cache=False)
    kvsnap = KvStateSnapshot(st)
    nq = k + 1
    ok = torch.empty(B, dtype=torch.int32, device=dev)
    peak, _ = load_peaks()
    rank_bytes = (2 * k + 1) * B * Vs * 4
    for tr in transports:
        prev = os.environ.get("KYRO_TP_TRANSPORT")
        ctx = Context(local)
        try:
            if world > 1:
                if tr == "nccl":
                    os.environ["KYRO_TP_TRANSPORT"] = "nccl"
                uid = torch.zeros(128, dtype=torch.uint8, device=dev)
                if rank == 0:
                    uid.copy_(torch.frombuffer(bytearray(tp_unique_id()), dtype=torch.uint8))
                dist.broadcast(uid, 0)
                ctx.tp_init(bytes(uid.cpu().numpy().tobytes()), rank, world)
        finally:
            if prev is None:
                os.environ.pop("KYRO_TP_TRANSPORT", None)
            else:
                os.environ["KYRO_TP_TRANSPORT"] = prev
        got = ctx.tp_transport if world > 1 else "none"
        parity = _tp_parity(ctx, world, rank, dev)
        # every rank's verdict, combined with a collective all ranks take
        flags = torch.tensor([0 if parity is None else (1 if parity else 2)], device=dev)
        if world > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX)
        parity_ok = {0: None, 1: True, 2: False}[int(flags.item())]
        ev = []

        def step(i, timed):
            s = torch.cuda.current_stream(dev)
            kvsnap.restore()
            kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                       st.ref_counts, cfg.block_size, out_ok=ok)
            if timed:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(s)
            acc, _, _, _ = spec_accept_tp(ctx, tgt, drf, drafts, V, temperature=T, seed=0, step=i)
            if timed:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(s)
                ev.append((e0, e1))
            kv_commit(ctx, nq, acc, st.block_table, st.context_lens, st.free_stack, st.free_top,
                      st.ref_counts, cfg.block_size)
            return acc

        # the timed steps replay one captured step (every rank captures the
        # same sequence of kernels and collectives), so that host launch time
        # does not set the pace; the per-call events come from plain steps
        side = torch.cuda.Stream(dev)
        graph = None
        with torch.cuda.stream(side):
            ctx.bind_stream()
            for i in range(warmup):
                step(i, False)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step(warmup, False)
            for _ in range(3):
                graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            t0.record(side)
            for i in range(steps):
                graph.replay()
            t1.record(side)
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        with torch.cuda.stream(side):
            for i in range(PER_KERNEL_STEPS):
                step(warmup + steps + i, True)
        torch.cuda.synchronize()
        del graph  # before the context (and its NCCL communicator) goes
        ctx.bind_stream()
        acc_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
        ms, acc_ms = max_over_ranks([ms, acc_ms], world, dev)
        status = ctx.device_status()
        ctx.close()
        if world > 1:
            dist.barrier()
        res[tr] = {"transport": got, "parity_ok": parity_ok, "ms_per_step": ms / steps,
                   "timing": "CUDA graph replays of the step (restore, reserve, accept, commit)",
                   "accept_ms": acc_ms, "positions_per_s": B * nq * steps / (ms * 1e-3),
                   "per_rank_GBps": rank_bytes / (acc_ms * 1e-3) / 1e9,
                   "frac_hbm_per_rank": rank_bytes / (acc_ms * 1e-3) / 1e9 / peak,
                   "device_status": status}
    res["parity_ok"] = all(res[t]["parity_ok"] for t in transports)
    return res


# ------------------------------------------------------------------ CPU side
def _host_inputs(st, tgt, drf, drafts, k_new, v_new):
    from kyro_b200.workloads import bf16_bits
    return {"q": bf16_bits(st.q), "k_cache": bf16_bits(st.k_cache),
            "v_cache": bf16_bits(st.v_cache), "block_table": st.block_table.cpu().numpy(),
            "context_lens": st.context_lens.cpu().numpy(), "free_stack": st.free_stack.cpu().numpy(),
            "free_top": st.free_top.cpu().numpy(), "ref_counts": st.ref_counts.cpu().numpy(),
            "tgt": tgt.cpu().numpy(), "drf": drf.cpu().numpy(), "drafts": drafts.cpu().numpy(),
            "k_new": bf16_bits(k_new), "v_new": bf16_bits(v_new)}


def _cpu_step(O, cfg, inp, seqs, step, nthreads):
    """The reference path's verify step on host cores for the sequences in
    `seqs` (oracle restatement, composed as the GPU step is)."""
    sel = np.asarray(seqs)
    state = {"block_table": inp["block_table"][sel].copy(),
             "context_lens": inp["context_lens"][sel].copy(),
             "free_stack": inp["free_stack"].copy(), "free_top": inp["free_top"].copy(),
             "ref_counts": inp["ref_counts"].copy(), "k_cache": inp["k_cache"],
             "v_cache": inp["v_cache"]}
    O.verify_step(state, inp["q"][sel], inp["k_new"][sel], inp["v_new"][sel], inp["tgt"][sel],
                  inp["drf"][sel], inp["drafts"][sel], cfg.block_size,
                  temperature=cfg.temperature, seed=0, step=step, rope_theta=10000.0,
                  nthreads=nthreads)


def cpu_baseline(cfg, st, tgt, drf, drafts, k_new, v_new, args):
    """The oracle's verify step over the whole config-1 batch on the host
    cores, repeated for about ten seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    inp = _host_inputs(st, tgt, drf, drafts, k_new, v_new)
    nthreads = len(os.sched_getaffinity(0)) or 1
    seqs = list(range(cfg.batch))
    done, t0 = 0, time.perf_counter()
    while True:
        _cpu_step(O, cfg, inp, seqs, done, nthreads)
        done += 1
        dt = time.perf_counter() - t0
        if dt > args.cpu_seconds or done >= 50:
            break
    return {"value": done * len(seqs) * cfg.num_query / dt, "unit": UNIT, "cores": nthreads,
            "kind": "port",
            "sample": f"{done} verify steps over the full config-1 batch ({cfg.batch} sequences: "
                      f"RoPE + kv write + attention + accept + commit), {dt:.1f} s"}


def run_reference(args):
    """CPU restatement of the reference path on the host cores, same config."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    from kyro_b200.workloads import CONFIG1, accept_inputs, paged_state
    cfg = CONFIG1
    st = paged_state(cfg, "cpu", seed=1000)
    tgt, drf = accept_inputs(cfg.batch, cfg.k, cfg.vocab, "cpu", seed=2000)
    nthreads = os.cpu_count() or 1
    drafts, _ = O.sample_tokens(drf.numpy(), cfg.temperature, seed=0, nthreads=nthreads)
    g = torch.Generator().manual_seed(3000)
    shape = (cfg.batch, cfg.num_query, cfg.num_kv_heads, cfg.head_dim)
    k_new = torch.randn(shape, generator=g).to(torch.bfloat16)
    v_new = torch.randn(shape, generator=g).to(torch.bfloat16)
    inp = _host_inputs(st, tgt, drf, torch.from_numpy(drafts), k_new, v_new)
    sample = min(cfg.batch, args.cpu_sample)
    for i in range(args.warmup):
        _cpu_step(O, cfg, inp, list(range(sample)), i, nthreads)
    times = []
    for i in range(args.steps):
        seqs = [(i * sample + j) % cfg.batch for j in range(sample)]
        t = time.perf_counter()
        _cpu_step(O, cfg, inp, seqs, args.warmup + i, nthreads)
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = sample * cfg.num_query * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; BASELINE config 1 shapes and distributions)",
        "config": workload_desc(cfg, 1), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": f"{sample} of {cfg.batch} config-1 sequences per step"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- standalone configs
def run_tree(args):
    """--config 2: the tree verify step alone, with its own JSON line."""
    import torch.distributed as dist
    from kyro_b200.verify import Context
    world, rank, local, dev = init_ranks(args)
    ctx = Context(local)
    clocks = start_clocks(rank, local)
    r = tree_measure(ctx, world, rank, dev, steps=args.steps, warmup=args.warmup)
    clk = clocks.stop() if clocks else None
    if rank == 0:
        print(json.dumps({
            "metric": "spec-verify tree nodes/s (config 2)", "unit": "verified tree nodes/s",
            "value": r["nodes_per_s"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config 2 shapes and distributions)",
            "config": {"workload": r["workload"], "parallelism": f"batch-sharded x{world}"},
            "kernels": {"attention": r["attention"], "accept": r["accept"]},
            "mean_path_len": r["mean_path_len"], "clocks": clk}), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_tp(args):
    """--config 3: the vocabulary-sharded acceptance alone, with its own line."""
    import torch.distributed as dist
    world, rank, local, dev = init_ranks(args)
    if 128256 % world:
        raise SystemExit(f"vocab 128256 does not split over {world} ranks")
    clocks = start_clocks(rank, local)
    r = tp_measure(world, rank, local, dev, steps=args.steps, warmup=args.warmup)
    clk = clocks.stop() if clocks else None
    if rank == 0:
        best = min((r[t] for t in ("single", "peer", "nccl") if t in r),
                   key=lambda x: x["ms_per_step"])
        print(json.dumps({
            "metric": "TP spec-accept verified positions/s (config 3)", "unit": UNIT,
            "value": best["positions_per_s"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": best["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config 3 shapes and distributions)",
            "config": {"workload": r["workload"], "parallelism": f"tp{world} (vocabulary)"},
            "tp_accept": r, "clocks": clk}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class _EventTimer:
    """Sums CUDA-event intervals per name over the current stream."""

    def __init__(self, stream):
        import torch
        self.torch, self.stream, self.open, self.pairs = torch, stream, {}, {}

    def begin(self, name):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record(self.stream)
        self.open[name] = e

    def end(self, name):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record(self.stream)
        self.pairs.setdefault(name, []).append((self.open.pop(name), e))

    def ms(self, name, per):
        return sum(a.elapsed_time(b) for a, b in self.pairs.get(name, [])) / per


def e2e_model_measure(args, world, rank, local, dev):
    """Config 4: the end-to-end batched speculative step over a random-init
    16-layer Llama target and a 2-layer draft (kyro_b200/e2e_model.py).
    512 requests in total, split over the N ranks (strong scaling, no
    collective); every step drafts k = 4 tokens per request, verifies k + 1
    positions through the target, accepts, and commits, with the contexts
    growing from step to step.  Timed as CUDA graph replays of one step
    (args: warmup, steps, no_graph, requests, target_layers).  Returns the
    measurements (max over ranks, byte counts over all ranks) on every rank;
    every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist

    from kyro_b200.e2e_model import CONFIG4, CONFIG4_SHAPE, SpecModels, SpecStep, context_lengths
    from kyro_b200.verify import Context
    from kyro_b200.workloads import ChainConfig, paged_state

    cfg, shape = CONFIG4, CONFIG4_SHAPE
    if args.requests or args.target_layers:
        # a smaller case of the same step, for profiler captures (not a bench line)
        import dataclasses
        cfg = dataclasses.replace(cfg, requests=args.requests or cfg.requests)
        shape = dataclasses.replace(shape, layers=args.target_layers or shape.layers)
    if cfg.requests % world:
        raise SystemExit(f"{cfg.requests} requests do not split over {world} ranks")
    B = cfg.requests // world
    lens = context_lengths(cfg, seed=0)[rank * B:(rank + 1) * B]
    bs, k = cfg.block_size, cfg.k
    grow = (k + 1) * (args.warmup + args.steps + PER_KERNEL_STEPS + 8)
    need_blocks = int(sum(-(-(int(c) + grow) // bs) for c in lens))
    kvcfg = ChainConfig(batch=B, k=k, num_heads=1, num_kv_heads=1, head_dim=8,
                        num_blocks=need_blocks + 256, ctx_min=1, ctx_max=cfg.ctx_max,
                        headroom_tokens=grow)
    kv = paged_state(kvcfg, dev, seed=4000 + rank, ctx_lens=lens, num_query=1, fill_cache=False)
    del kv.k_cache, kv.v_cache, kv.q
    models = SpecModels(shape, cfg, kvcfg.num_blocks, dev, seed=4100)
    ctx_t, ctx_d = Context(local), Context(local)
    spec = SpecStep(models, ctx_t, ctx_d, kv, seed=0, seq_offset=rank * B)
    side = torch.cuda.Stream(dev)
    graph = None
    with torch.cuda.stream(side):
        for i in range(args.warmup):
            spec(i)
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                spec(args.warmup)
    torch.cuda.synchronize()
    lens0 = kv.context_lens.cpu().numpy().copy()
    if world > 1:
        dist.barrier()
    clocks = start_clocks(rank, local)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):
        t0.record(side)
        for i in range(args.warmup, args.warmup + args.steps):
            if graph is not None:
                graph.replay()
            else:
                spec(i)
        t1.record(side)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1)
    lens1 = kv.context_lens.cpu().numpy().copy()
    emitted = float(lens1.sum() - lens0.sum())  # accept_len + 1 per request and step
    # per-kernel times from eager steps with events around the parts
    timer = _EventTimer(side)
    with torch.cuda.stream(side):
        lens_k = kv.context_lens.cpu().numpy().copy()
        for i in range(PER_KERNEL_STEPS):
            spec(args.warmup + args.steps + i, timer=timer)
    torch.cuda.synchronize()
    del graph
    status = ctx_t.device_status() | ctx_d.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the timed region")
    part = {n: timer.ms(n, PER_KERNEL_STEPS) for n in ("draft", "target", "attention", "accept")}
    # target verify attention, all layers of one step: K and V of every
    # cached token plus the k + 1 new ones, and Q and O (bf16)
    kv_tok = 2 * shape.kv_heads * shape.head_dim * 2
    att_bytes = float(shape.layers * ((lens_k + k + 1).sum() * kv_tok
                                      + 2 * B * (k + 1) * shape.heads * shape.head_dim * 2))
    acc_bytes = float((2 * k + 1) * shape.vocab * 4 * B)
    att_ms, acc_ms = part["attention"], part["accept"]
    if world > 1:
        # step time and part times: max over ranks; kernel bandwidth: every
        # rank's bytes over every rank's time (ranks hold unequal contexts)
        t = torch.tensor([ms] + [part[n] for n in ("draft", "target", "attention", "accept")],
                         dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sums = torch.tensor([emitted, att_bytes, att_ms, acc_bytes, acc_ms], dtype=torch.float64,
                            device=dev)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
        ms = float(t[0])
        part = dict(zip(("draft", "target", "attention", "accept"), [float(x) for x in t[1:]]))
        emitted, att_bytes, att_ms, acc_bytes, acc_ms = [float(x) for x in sums]
    peak, peak_kind = load_peaks()
    att_gbs = att_bytes / (att_ms * 1e-3) / 1e9
    acc_gbs = acc_bytes / (acc_ms * 1e-3) / 1e9
    # DRAM bytes of one target attention launch: a capture of a 128-request
    # case scaled by this launch's algorithmic bytes (traffic follows them)
    small = load_traffic().get("verify_attention_kernel_config4_small")
    traffic4 = (small["dram_bytes"] / small["algorithmic_bytes"] * att_bytes / world / shape.layers
                if small else None)
    ctx_t.close()
    ctx_d.close()
    return {"cfg": cfg, "shape": shape, "B": B, "k": k, "ms": ms, "emitted": emitted,
            "part": part, "att_bytes": att_bytes, "att_ms": att_ms, "att_gbs": att_gbs,
            "acc_bytes": acc_bytes, "acc_ms": acc_ms, "acc_gbs": acc_gbs, "peak": peak,
            "peak_kind": peak_kind, "traffic4": traffic4, "clocks": clk}


def run_e2e_model(args):
    """Config 4 as its own bench line (bench.py --config 4)."""
    import torch.distributed as dist

    world, rank, local, dev = init_ranks(args, timeout_s=300)
    m = e2e_model_measure(args, world, rank, local, dev)
    cfg, shape, B, k, ms, emitted, part = (m[n] for n in ("cfg", "shape", "B", "k", "ms", "emitted",
                                                          "part"))
    att_bytes, att_ms, att_gbs = m["att_bytes"], m["att_ms"], m["att_gbs"]
    acc_bytes, acc_ms, acc_gbs = m["acc_bytes"], m["acc_ms"], m["acc_gbs"]
    peak, peak_kind, traffic4, clk = m["peak"], m["peak_kind"], m["traffic4"], m["clocks"]
    if rank == 0:
        line = {
            "metric": "spec-decode verified positions/s, end-to-end step (config 4)",
            "unit": "verified positions/s",
            "value": cfg.requests * (k + 1) * args.steps / (ms * 1e-3), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights; BASELINE config 4 shapes; "
                    "lognormal contexts with sigma 1.0 assumed)",
            "config": {"workload": "config4: end-to-end speculative step, 16-layer Llama target "
                                   "(hidden 2048, 32/8 heads, D 64, FFN 8192, V 128256, bf16) + "
                                   "2-layer draft, k 4, T 0.7, 512 requests, ctx lognormal "
                                   "(median 1024, max 16384)",
                       "requests": cfg.requests, "requests_per_gpu": B,
                       "target_layers": shape.layers,
                       "reduced_for_profiling": bool(args.requests or args.target_layers),
                       "parallelism": f"batch-sharded x{world} (no collective)",
                       "l2": "inputs larger than L2 (~30 GB of K/V per GPU at N=1)"},
            "emitted_tokens_per_s": emitted / (ms * 1e-3),
            "mean_emitted_per_request_step": emitted / (cfg.requests * args.steps),
            "roofline": {"bound": "hbm", "kernel": "verify_attention_kernel (16 target layers)",
                         "achieved": att_gbs, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": att_gbs / peak, "traffic": traffic4},
            "parts_ms_per_step": part,
            "kernels": {
                # means over ranks (one rank's figures at N = 1)
                "target_attention": {"ms": att_ms / world, "algorithmic_bytes": att_bytes / world,
                                     "GBps": att_gbs, "frac": att_gbs / peak},
                "accept": {"ms": acc_ms / world, "algorithmic_bytes": acc_bytes / world,
                           "GBps": acc_gbs, "frac": acc_gbs / peak},
            },
            "timing": "stream launches" if args.no_graph else "CUDA graph replays of the step",
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample", type=int, default=8,
                    help="sequences per CPU step (cpu_baseline and --impl reference)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="wall time the cpu_baseline leg repeats whole-batch steps for")
    ap.add_argument("--no-graph", action="store_true",
                    help="time config 1 as plain launches instead of CUDA graph replays")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer leg (profiling runs)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config 0 / 2 / 3 measurements after the headline")
    ap.add_argument("--extra-steps", type=int, default=20,
                    help="timed steps of each extra configuration")
    ap.add_argument("--requests", type=int, default=0,
                    help="config 4 only: requests in all (default 512; smaller for profiling)")
    ap.add_argument("--target-layers", type=int, default=0,
                    help="config 4 only: target layers (default 16; fewer for profiling)")
    ap.add_argument("--config", choices=["1", "2", "3", "4"], default="1",
                    help="1: chain verify step (the headline); 2: tree verify step; "
                         "3: vocabulary-sharded acceptance over the N ranks of one TP group; "
                         "4: end-to-end speculative step of a 16-layer Llama + 2-layer draft")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "2":
        run_tree(args)
    elif args.config == "3":
        run_tp(args)
    elif args.config == "4":
        run_e2e_model(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
