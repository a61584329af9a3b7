"""Benchmark of the speculative verify step on B200.

One step = one verify pass over a batch of 64 sequences per GPU, the
workload BASELINE.json's metric is quoted on (config 1):
  kv_reserve (k+1 slots) -> kv_write (new K/V rows) -> verify attention
  (Llama-3-8B layer: Hq 32, Hkv 8, D 128, bf16 paged KV, block 16,
  context ~ U[512, 4096]) -> acceptance sampling (k = 5, V = 128256, fp32,
  T = 1.0) -> kv_commit.
Contexts grow by the committed tokens from step to step, as in decoding.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; sequences are sharded by
rank (weak scaling, no collective on the data path).  `value` is verified
positions per second over all ranks, device-timed with CUDA events, max
over ranks.  `e2e` is the same metric through the C ABI with host buffers:
each step copies its inputs from pinned host memory and reads its results
back.  `--impl reference` times the CPU restatement of the reference path
(oracle/, the reference itself is Rust and cannot be built here) on the
host cores.
"""
from __future__ import annotations

import argparse
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


def workload_desc(cfg, n):
    return {
        "workload": "config1: chain verify (paged attention + accept + KV commit), Llama-3-8B "
                    "layer Hq32/Hkv8/D128 bf16 KV block16, ctx U[512,4096], k=5 (+1), "
                    "V=128256 fp32, T=1.0",
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


# --------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    import torch.distributed as dist

    from kyro_b200 import _lib
    from kyro_b200.verify import (Context, kv_commit, kv_reserve, kv_write, rope_kv_write,
                                  sample_tokens, spec_accept, verify_attention)
    from kyro_b200.workloads import CONFIG1, accept_inputs, chain_bytes_per_step, paged_state

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
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
    attn_out = torch.empty_like(st.q)
    acc = torch.empty(cfg.batch, dtype=torch.int32, device=dev)
    toks = torch.empty(cfg.batch, nq, dtype=torch.int32, device=dev)
    num = torch.empty(cfg.batch, dtype=torch.int32, device=dev)
    ok = torch.empty(cfg.batch, dtype=torch.int32, device=dev)
    L = _lib.load()
    from kyro_b200.verify import attn_params
    import ctypes as C
    from kyro_b200._lib import AcceptParams
    ws_attn = torch.empty(max(256, L.kyro_verify_attention_workspace_size(
        C.byref(attn_params(st.q, st.k_cache, st.block_table)))), dtype=torch.uint8, device=dev)
    ws_acc = torch.empty(max(256, L.kyro_spec_accept_workspace_size(C.byref(AcceptParams(
        cfg.batch, cfg.k, cfg.vocab, 0, cfg.temperature, 0, 0, 0)))), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = {n: [] for n in ("attention", "accept")}
    # every step starts from the same KV state, so each step sees the same
    # context lengths; the reset is one device-to-device copy (~0.5 MB)
    kvsnap = KvStateSnapshot(st)
    restore = kvsnap.restore

    def step(i, timed):
        restore()
        kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                   st.ref_counts, cfg.block_size, out_ok=ok)
        kv_write(ctx, k_new, v_new, st.block_table, st.context_lens, st.k_cache, st.v_cache,
                 cfg.block_size)
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        verify_attention(ctx, st.q, st.k_cache, st.v_cache, st.block_table, st.context_lens,
                         out=attn_out, workspace=ws_attn)
        if timed:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
        spec_accept(ctx, tgt, drf, drafts, temperature=cfg.temperature, seed=0, step=i,
                    seq_offset=seq_offset, out=(acc, toks, num, None), workspace=ws_acc)
        if timed:
            e2 = torch.cuda.Event(enable_timing=True)
            e2.record()
            ev["attention"].append((e0, e1))
            ev["accept"].append((e1, e2))
        kv_commit(ctx, nq, acc, st.block_table, st.context_lens, st.free_stack, st.free_top,
                  st.ref_counts, cfg.block_size)

    # the step runs on a side stream as a CUDA graph (captured once after the
    # warm-up steps); the library context is bound to that stream
    side = torch.cuda.Stream(dev)
    graph = None
    with torch.cuda.stream(side):
        ctx.bind_stream()
        for i in range(args.warmup):
            step(i, False)
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                step(args.warmup, False)
            for _ in range(3):
                graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    phys = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    if vis:
        ids = [v.strip() for v in vis.split(",")]
        if local < len(ids) and ids[local].isdigit():
            phys = int(ids[local])
    clocks = None
    if rank == 0:
        try:
            clocks = NvmlClockSampler(phys)
        except Exception:
            clocks = ClockSampler(phys)
    if clocks:
        clocks.start()
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
                step(i, False)
        t1.record(side)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1)
    # per-kernel times from separate steps with events around attention and
    # acceptance (events between kernels would perturb the timed steps)
    with torch.cuda.stream(side):
        for i in range(PER_KERNEL_STEPS):
            step(args.warmup + args.steps + i, True)
        # the fused rotary embedding + paged K/V store on the step's new tokens
        # (kyro_rope_kv_write, the alternative to kv_write for un-rotated
        # projections), timed back to back: its ~9 MB stay in L2
        restore()
        kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                   st.ref_counts, cfg.block_size, out_ok=ok)
        q_rot = torch.empty_like(st.q)
        for _ in range(3):
            rope_kv_write(ctx, st.q, k_new, v_new, st.block_table, st.context_lens, st.k_cache,
                          st.v_cache, cfg.block_size, q_out=q_rot)
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(20):
            rope_kv_write(ctx, st.q, k_new, v_new, st.block_table, st.context_lens, st.k_cache,
                          st.v_cache, cfg.block_size, q_out=q_rot)
        r1.record()
    torch.cuda.synchronize()
    rope_us = r0.elapsed_time(r1) / 20 * 1e3
    rope_bytes = 2.0 * q_rot.numel() * 2 + 4.0 * k_new.numel() * 2
    del graph
    ctx.bind_stream()  # back to the default stream for the end-to-end run
    if world > 1:
        tms = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tms, op=dist.ReduceOp.MAX)
        ms = float(tms.item())
    status = ctx.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the timed region")

    # algorithmic bytes per step, from the context lengths every step starts from
    per = [chain_bytes_per_step(kvsnap.initial("context_lens").cpu().numpy(), cfg)]
    att_ms = np.mean([a.elapsed_time(b) for a, b in ev["attention"]])
    acc_ms = np.mean([a.elapsed_time(b) for a, b in ev["accept"]])
    att_bytes = float(np.mean([p["attention"] for p in per]))
    acc_bytes = float(np.mean([p["accept"] for p in per]))
    peak, peak_kind = load_peaks()
    traffic = load_traffic()
    if att_ms >= acc_ms:
        dom, dbytes, dms = "verify_attention_kernel", att_bytes, att_ms
    else:
        dom, dbytes, dms = "accept_stats_kernel", acc_bytes, acc_ms
    achieved = dbytes / (dms * 1e-3) / 1e9
    units = cfg.batch * nq * world * args.steps
    value = units / (ms * 1e-3)
    step_bytes = att_bytes + acc_bytes
    # kv_reserve, kv_write, verify_attention, accept_stats, accept_decide,
    # accept_final, kv_commit (the attention split counters are zeroed by a
    # driver memset only the first time a workspace is used)
    launches_per_step = 7
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
            "step_frac_of_hbm": step_bytes / (ms / args.steps * 1e-3) / 1e9 / peak,
            "rope_kv_write": {"us": rope_us, "bytes": rope_bytes,
                              "GBps": rope_bytes / (rope_us * 1e-6) / 1e9,
                              "note": "outside the step; back-to-back launches, L2-resident"},
        },
        "timing": "CUDA graph replays of the step" if not args.no_graph else "stream launches",
        "acceptance_rate": float(acc.float().mean().item() / cfg.k),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
    }
    if not args.no_e2e:
        line["e2e"] = run_e2e(args, ctx, cfg, st, tgt, drf, drafts, k_new, v_new, seq_offset,
                              world, dist if world > 1 else None, dev, restore)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, st, tgt, drf, drafts, k_new, v_new, args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _attn_splits(st, cfg):
    import ctypes as C
    from kyro_b200 import _lib
    from kyro_b200.verify import attn_params
    p = attn_params(st.q, st.k_cache, st.block_table)
    return _lib.load().kyro_verify_attention_workspace_size(C.byref(p)) > 0


def run_e2e(args, ctx, cfg, st, tgt, drf, drafts, k_new, v_new, seq_offset, world, dist, dev,
            restore):
    """The same step through the C ABI with host buffers: inputs copied from
    pinned host memory each step, results read back each step."""
    import torch
    from kyro_b200.verify import kv_commit, kv_reserve, kv_write, spec_accept, verify_attention
    nq = cfg.num_query
    h = {n: t.cpu().pin_memory() for n, t in
         dict(q=st.q, k_new=k_new, v_new=v_new, tgt=tgt, drf=drf, drafts=drafts).items()}
    d = {n: torch.empty_like(t, device=dev) for n, t in h.items()}
    out_h = {n: torch.empty(s, dtype=torch.int32).pin_memory()
             for n, s in dict(acc=(cfg.batch,), toks=(cfg.batch, nq), num=(cfg.batch,)).items()}
    out_d = {n: torch.empty(t.shape, dtype=torch.int32, device=dev) for n, t in out_h.items()}
    attn_out = torch.empty_like(st.q)
    stream = torch.cuda.current_stream(dev)
    h2d = sum(t.numel() * t.element_size() for t in h.values())
    d2h = sum(t.numel() * t.element_size() for t in out_h.values())
    steps = max(3, min(args.steps, 10))

    def step(i):
        restore()
        for n in h:
            d[n].copy_(h[n], non_blocking=True)
        kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                   st.ref_counts, cfg.block_size)
        kv_write(ctx, d["k_new"], d["v_new"], st.block_table, st.context_lens, st.k_cache,
                 st.v_cache, cfg.block_size)
        verify_attention(ctx, d["q"], st.k_cache, st.v_cache, st.block_table, st.context_lens,
                         out=attn_out)
        spec_accept(ctx, d["tgt"], d["drf"], d["drafts"], temperature=cfg.temperature, seed=0,
                    step=1000 + i, seq_offset=seq_offset,
                    out=(out_d["acc"], out_d["toks"], out_d["num"], None))
        kv_commit(ctx, nq, out_d["acc"], st.block_table, st.context_lens, st.free_stack,
                  st.free_top, st.ref_counts, cfg.block_size)
        for n in out_h:
            out_h[n].copy_(out_d[n], non_blocking=True)
        stream.synchronize()  # the caller reads the emitted tokens

    step(0)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        step(1 + i)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if dist:
        tms = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tms, op=dist.ReduceOp.MAX)
        ms = float(tms.item())
    value = cfg.batch * nq * world * steps / (ms * 1e-3)
    return {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "ms_per_step": ms / steps}


# ------------------------------------------------------------------ CPU side
def _cpu_step(O, cfg, inp, seqs, step, nthreads):
    """The reference path's verify step on host cores for the sequences in
    `seqs`: KV write, attention, acceptance, commit (oracle restatement)."""
    sel = np.asarray(seqs)
    nq = cfg.num_query
    bt, cl = inp["bt"][sel].copy(), inp["cl"][sel].copy()
    fs, top, rc = inp["fs"].copy(), inp["top"].copy(), inp["rc"].copy()
    O.kv_reserve(nq, bt, cl, fs, top, rc, cfg.block_size)
    O.kv_write(inp["k_new"][sel], inp["v_new"][sel], bt, cl, inp["kc"], inp["vc"],
               cfg.block_size)
    O.paged_attention(inp["q"][sel], inp["kc"], inp["vc"], bt, cl, cfg.block_size,
                      nthreads=nthreads)
    acc, _, _, _ = O.spec_accept(inp["tgt"][sel], inp["drf"][sel], inp["drafts"][sel],
                                 temperature=cfg.temperature, seed=0, step=step,
                                 nthreads=nthreads)
    O.kv_commit(nq, acc, bt, cl, fs, top, rc, cfg.block_size)


def _host_inputs(st, tgt, drf, drafts, k_new, v_new):
    from kyro_b200.workloads import bf16_bits
    return {"q": bf16_bits(st.q), "kc": bf16_bits(st.k_cache), "vc": bf16_bits(st.v_cache),
            "bt": st.block_table.cpu().numpy(), "cl": st.context_lens.cpu().numpy(),
            "fs": st.free_stack.cpu().numpy(), "top": st.free_top.cpu().numpy(),
            "rc": st.ref_counts.cpu().numpy(), "tgt": tgt.cpu().numpy(),
            "drf": drf.cpu().numpy(), "drafts": drafts.cpu().numpy(),
            "k_new": bf16_bits(k_new), "v_new": bf16_bits(v_new)}


def cpu_baseline(cfg, st, tgt, drf, drafts, k_new, v_new, args):
    """The oracle's verify step over the whole config-1 batch on the host
    cores, repeated for about ten seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    inp = _host_inputs(st, tgt, drf, drafts, k_new, v_new)
    nthreads = os.cpu_count() or 1
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
                      f"kv write + attention + accept + commit), {dt:.1f} s"}


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
    drafts, _ = O.sample_tokens(drf.numpy(), cfg.temperature, seed=0, nthreads=os.cpu_count())
    g = torch.Generator().manual_seed(3000)
    shape = (cfg.batch, cfg.num_query, cfg.num_kv_heads, cfg.head_dim)
    k_new = torch.randn(shape, generator=g).to(torch.bfloat16)
    v_new = torch.randn(shape, generator=g).to(torch.bfloat16)
    inp = _host_inputs(st, tgt, drf, torch.from_numpy(drafts), k_new, v_new)
    nthreads = os.cpu_count() or 1
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


def run_tree(args):
    """Config 2: tree verification.  Per step and GPU (batch-sharded, no
    collective): KV reserve and write of the 64 tree nodes, paged attention
    of 64 query heads over 8 KV heads (context 8192) under the ancestor mask,
    multi-candidate acceptance over vocabulary 32000, and the tree commit of
    the accepted path."""
    import datetime

    import torch
    import torch.distributed as dist

    from kyro_b200.verify import (Context, kv_commit_tree, kv_reserve, kv_write,
                                  spec_accept_tree, verify_attention)
    from kyro_b200.workloads import CONFIG2, bfs_tree, paged_state, tree_mask_bits

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = CONFIG2
    B, N, V = cfg.batch, cfg.num_query, cfg.vocab
    ctx = Context(local)
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

    for i in range(args.warmup):
        step(i, False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = None
    if rank == 0:
        try:
            clocks = NvmlClockSampler(local)
        except Exception:
            clocks = ClockSampler(local)
        clocks.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    plens = []
    for i in range(args.warmup, args.warmup + args.steps):
        plens.append(step(i, False))
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1)
    # per-kernel times from separate steps, so that no event sits between the
    # chained launches of the timed ones
    for i in range(args.warmup + args.steps, args.warmup + args.steps + PER_KERNEL_STEPS):
        step(i, True)
    torch.cuda.synchronize()
    att_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["attention"]]))
    acc_ms = float(np.mean([a.elapsed_time(b) for a, b in ev["accept"]]))
    if world > 1:
        t = torch.tensor([ms, att_ms, acc_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, att_ms, acc_ms = float(t[0]), float(t[1]), float(t[2])
    status = ctx.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the timed region")
    peak, peak_kind = load_peaks()
    kv_bytes = B * (cfg.ctx_max + N) * 2 * cfg.num_kv_heads * cfg.head_dim * 2
    flops = 4.0 * B * cfg.num_heads * N * cfg.head_dim * (cfg.ctx_max + N)
    acc_bytes = 2 * B * N * V * 4
    mean_path = float(torch.stack(plens).float().mean().item())
    if rank == 0:
        line = {
            "metric": "spec-verify tree nodes/s (config 2)", "unit": "verified tree nodes/s",
            "value": B * N * world * args.steps / (ms * 1e-3), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config 2 shapes and distributions)",
            "config": {"workload": "config2: tree verify (paged attention under a 64-node "
                                   "ancestor mask + multi-candidate acceptance + tree commit), "
                                   "Hq64/Hkv8/D128 bf16, ctx 8192, tree 4,4,4 cut to 64, "
                                   "V 32000 fp32, T 1.0",
                       "batch_per_gpu": B, "global_batch": B * world, "nodes": N,
                       "parallelism": f"batch-sharded x{world} (no collective)"},
            "kernels": {
                "attention": {"ms": att_ms, "kv_bytes": kv_bytes, "flops": flops,
                              "GBps": kv_bytes / (att_ms * 1e-3) / 1e9,
                              "hbm_frac": kv_bytes / (att_ms * 1e-3) / 1e9 / peak,
                              "TFLOPs": flops / (att_ms * 1e-3) / 1e12},
                "accept": {"ms": acc_ms, "bytes": acc_bytes,
                           "GBps": acc_bytes / (acc_ms * 1e-3) / 1e9,
                           "hbm_frac": acc_bytes / (acc_ms * 1e-3) / 1e9 / peak},
            },
            "mean_path_len": mean_path,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
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


def run_e2e_model(args):
    """Config 4: the end-to-end batched speculative step over a random-init
    16-layer Llama target and a 2-layer draft (kyro_b200/e2e_model.py).
    512 requests in total, split over the N ranks (strong scaling, no
    collective); every step drafts k = 4 tokens per request, verifies k + 1
    positions through the target, accepts, and commits, with the contexts
    growing from step to step.  Timed as CUDA graph replays of one step."""
    import datetime

    import torch
    import torch.distributed as dist

    from kyro_b200.e2e_model import CONFIG4, CONFIG4_SHAPE, SpecModels, SpecStep, context_lengths
    from kyro_b200.verify import Context
    from kyro_b200.workloads import ChainConfig, paged_state

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
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
    clocks = None
    if rank == 0:
        try:
            clocks = NvmlClockSampler(local)
        except Exception:
            clocks = ClockSampler(local)
        clocks.start()
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
    ctx_t.close()
    ctx_d.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_tp(args):
    """Config 3: vocabulary-sharded acceptance (kyro_spec_accept_tp) over the
    N ranks of one tensor-parallel group, plus KV reserve/commit on a
    32768-block table.  Total work is fixed as N grows (strong scaling):
    each rank holds V/N columns of the same [256, 9 | 8, V] logits."""
    import datetime

    import torch
    import torch.distributed as dist

    from kyro_b200.verify import (Context, kv_commit, kv_reserve, spec_accept_tp,
                                  tp_unique_id)
    from kyro_b200.workloads import CONFIG3, paged_state

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = CONFIG3
    B, k, V, T = cfg.batch, cfg.k, cfg.vocab, cfg.temperature
    if V % world:
        raise SystemExit(f"vocab {V} does not split over {world} ranks")
    Vs = V // world
    ctx = Context(local)
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(tp_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        ctx.tp_init(bytes(uid.cpu().numpy().tobytes()), rank, world)

    def shard(r):  # rank r's columns of the (never materialised) full logits
        g = torch.Generator(device=dev).manual_seed(5000 + r)
        t = torch.randn(B, k + 1, Vs, generator=g, device=dev) * cfg.logit_std
        d = t[:, :k, :] + torch.randn(B, k, Vs, generator=g, device=dev) * cfg.draft_noise
        return t.contiguous(), d.contiguous()

    tgt, drf = shard(rank)
    # draft tokens sampled from the full draft rows (rank 0 regenerates every
    # shard once, before the timed region) and broadcast
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
    stream = torch.cuda.current_stream(dev)
    ev = []

    def step(i, timed):
        kvsnap.restore()
        kv_reserve(ctx, nq, st.block_table, st.context_lens, st.free_stack, st.free_top,
                   st.ref_counts, cfg.block_size, out_ok=ok)
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        acc, _, _, _ = spec_accept_tp(ctx, tgt, drf, drafts, V, temperature=T, seed=0, step=i)
        if timed:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
            ev.append((e0, e1))
        kv_commit(ctx, nq, acc, st.block_table, st.context_lens, st.free_stack, st.free_top,
                  st.ref_counts, cfg.block_size)
        return acc

    for i in range(args.warmup):
        step(i, False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = None
    if rank == 0:
        try:
            clocks = NvmlClockSampler(local)
        except Exception:
            clocks = ClockSampler(local)
        clocks.start()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    accs = []
    for i in range(args.warmup, args.warmup + args.steps):
        accs.append(step(i, False))
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1)
    for i in range(args.warmup + args.steps, args.warmup + args.steps + PER_KERNEL_STEPS):
        step(i, True)
    torch.cuda.synchronize()
    acc_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    if world > 1:
        t = torch.tensor([ms, acc_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, acc_ms = float(t[0]), float(t[1])
    status = ctx.device_status()
    if status:
        raise SystemExit(f"device status word 0x{status:x} after the timed region")
    rate = float(torch.stack(accs).float().mean().item()) / k
    peak, peak_kind = load_peaks()
    rank_bytes = (2 * k + 1) * B * Vs * 4  # every logit of this rank's columns once
    achieved = rank_bytes / (acc_ms * 1e-3) / 1e9
    if rank == 0:
        line = {
            "metric": "TP spec-accept verified positions/s (config 3)", "unit": UNIT,
            "value": B * nq * args.steps / (ms * 1e-3), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config 3 shapes and distributions)",
            "config": {"workload": "config3: vocabulary-sharded acceptance (B 256, k 8, "
                                   f"V 128256 over {world} ranks, T 0.8) + KV reserve/commit "
                                   "on a 32768-block table",
                       "global_batch": B, "k": k, "vocab": V, "columns_per_rank": Vs,
                       "parallelism": f"tp{world} (vocabulary)",
                       "l2": f"{rank_bytes / 1e9:.2f} GB of logits per rank per step"},
            "roofline": {"bound": "hbm", "kernel": "kyro_spec_accept_tp (per rank)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": None},
            "accept_ms": acc_ms, "acceptance_rate": rate,
            "gpu_launches": (2 + (7 if world > 1 else 3)) * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
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
