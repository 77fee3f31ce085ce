"""Benchmark: logits rows sampled/sec at 512 x 151936 (heterogeneous top-k/top-p).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one batched sampling call over the 512-row fp32 batch of the
heterogeneous configuration (Zipf-like logits; per-row top_k in
{0,1,20,50,200}, top_p ~ U(0.5,1], temperature ~ U(0.2,1.5); seeded
synthetic data).  The 311 MB batch is larger than the 126 MB L2, so no flush
is needed between steps.

`value` is device-resident throughput (inputs already in HBM), timed with CUDA
events on the launching stream.  `e2e` goes through the public
``Sampler.sample_batch`` API from pinned host memory: every step copies the
logits and per-row parameters host->device and reads tokens, probabilities and
statuses back, inside the timed region.  Under torchrun each rank samples its
own batch (rows are independent; no collective on the data path), timing is
the max over ranks and `value` the total rows of all ranks over that time.

`--impl reference` times the reference algorithm on the host cores instead:
the float64 Python restatement of miniserve's Sampler.sample (oracle/, the
reference is Python) over a bounded sample of the same rows, one process per
core.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "logits rows sampled/sec at 512x151936 top-k/top-p; % of B200 HBM roofline"
WORKLOAD = "config3: 512x151936 fp32, heterogeneous per-row top_k/top_p/temperature"


def config3_config(B: int, V: int, world: int) -> dict:
    """The `config` of the metric's line, the same for both arms."""
    return {"workload": WORKLOAD, "batch_rows": B, "vocab": V, "global_batch": B * world,
            "parallelism": f"dp{world} (independent rows per rank)",
            "l2": "inputs (311 MB) larger than L2 (126 MB); no flush"}
FALLBACK_HBM_GBS = 6650.0


def profiled_traffic():
    """DRAM bytes per launch of the streaming kernel on this workload, from the
    committed ncu summary (dram__bytes_read.sum + dram__bytes_write.sum)."""
    path = os.path.join(ROOT, "profiles", "stream_kernel_config3_full.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------- CPU side
def _ref_rows(args):
    """Worker: the reference algorithm (Python float64 restatement) on rows."""
    logits, T, K, P, U = args
    from oracle import sampler_oracle as so
    out = []
    for b in range(len(T)):
        out.append(so.sample_token(logits[b].tolist(), float(T[b]), int(K[b]), float(P[b]), float(U[b])))
    return out


def cpu_reference_rate(batch, rows, pool, cores):
    """rows/s of the reference algorithm on `rows`, spread over `cores` processes."""
    chunks = [rows[i::cores] for i in range(cores)]
    chunks = [c for c in chunks if len(c)]
    jobs = [(batch.logits[c], batch.temperature[c], batch.top_k[c], batch.top_p[c], batch.uniforms[c])
            for c in chunks]
    t0 = time.perf_counter()
    pool.map(_ref_rows, jobs)
    dt = time.perf_counter() - t0
    return len(rows) / dt, dt


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons, read on a thread.

    Started before the timed region; `wait_first()` blocks until the first
    sample arrives so the timed region is covered from its start."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: int = 20):
        # nvidia-smi numbers the physical GPUs and ignores CUDA_VISIBLE_DEVICES:
        # address this process's GPU by its UUID
        self.gpu = str(gpu_index)
        try:
            import torch
            self.gpu = f"GPU-{torch.cuda.get_device_properties(gpu_index).uuid}"
        except Exception:
            pass
        self.interval = interval_ms
        self.proc = None
        self.lines = []
        self._first = threading.Event()

    def _reader(self):
        for line in self.proc.stdout:
            if line.strip():
                self.lines.append(line)
                self._first.set()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._reader, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def wait_first(self, timeout=5.0):
        self._first.wait(timeout)
        self.start_count = len(self.lines)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines[getattr(self, "start_count", 0):]:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms), "window": "device-timed and e2e regions"}


# ----------------------------------------------------------------- GPU side
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    from miniserve_b200 import Sampler, _lib, workloads

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cores = os.cpu_count() or 1
    pool = None
    if rank == 0 and not args.no_cpu_baseline:
        pool = mp.get_context("spawn").Pool(cores)  # started before GPU work
        pool.map(int, range(cores))
    batch = workloads.config3(3 + rank)
    B, V = batch.B, batch.V
    sampler = Sampler()
    L = _lib.lib()
    x = torch.from_numpy(batch.logits).to(dev)
    T = torch.from_numpy(batch.temperature).to(dev)
    K = torch.from_numpy(batch.top_k).to(dev)
    P = torch.from_numpy(batch.top_p).to(dev)
    U = torch.from_numpy(batch.uniforms).to(dev)
    tok = torch.empty(B, dtype=torch.int64, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def step():
        rc = L.ms_sample(x.data_ptr(), 0, B, V, V, T.data_ptr(), K.data_ptr(), P.data_ptr(), U.data_ptr(),
                         None, 0, tok.data_ptr(), prob.data_ptr(), st.data_ptr(), sptr)
        if rc != 0:
            _lib.check(rc, "ms_sample")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    clocks = ClockSampler(local_rank).__enter__()
    clocks.wait_first()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs[0].record(stream)
    for i in range(args.steps):
        step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per_launch = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    elapsed_ms = evs[0].elapsed_time(evs[-1])
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_step = max_ms / args.steps
    value = world * B * args.steps / (max_ms / 1e3)

    # correctness spot check of the timed outputs against the pinned oracle
    # is done by the tests; here only the row statuses are checked
    assert int((st != 0).sum().item()) == 0

    # ------------------------------------------------------------ e2e (host buffers)
    pin = lambda a: torch.from_numpy(a).pin_memory()
    hx, hT, hK, hP, hU = (pin(batch.logits), pin(batch.temperature), pin(batch.top_k),
                          pin(batch.top_p), pin(batch.uniforms))
    otok = torch.empty(B, dtype=torch.int64).pin_memory()
    oprob = torch.empty(B, dtype=torch.float32).pin_memory()
    ost = torch.empty(B, dtype=torch.int32).pin_memory()
    dx = torch.empty_like(x)
    dT, dK, dP, dU = (torch.empty_like(T), torch.empty_like(K), torch.empty_like(P), torch.empty_like(U))
    h2d = sum(a.numel() * a.element_size() for a in (hx, hT, hK, hP, hU))
    d2h = sum(a.numel() * a.element_size() for a in (otok, oprob, ost))

    def e2e_step():
        for d, h in ((dx, hx), (dT, hT), (dK, hK), (dP, hP), (dU, hU)):
            d.copy_(h, non_blocking=True)
        t_, p_, s_ = sampler.sample_batch(dx, dT, dK, dP, uniforms=dU, out=(tok, prob, st))
        otok.copy_(t_, non_blocking=True)
        oprob.copy_(p_, non_blocking=True)
        ost.copy_(s_, non_blocking=True)

    e2e_steps = max(1, min(args.steps, 10))
    for _ in range(min(args.warmup, 3)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * B * e2e_steps / (float(te.item()) / 1e3)
    clocks.__exit__(None, None, None)
    assert np.array_equal(otok.numpy(), tok.cpu().numpy())

    shard = sharded_line(args, rank, world, dev, peak=hbm_peak()[0])
    if rank != 0:
        return None
    # roofline of the sampling kernel: algorithmic bytes per launch / launch time
    alg_bytes = B * (V * 4 + 8 + 4 + 8 + 8 + 8 + 4 + 4)
    avg_launch_ms = sum(per_launch) / len(per_launch)
    achieved = alg_bytes / (avg_launch_ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    cpu = None
    if pool is not None:
        sample_rows = list(range(B))  # the whole batch: ~0.15 core-s per row
        rate, dt = cpu_reference_rate(batch, sample_rows, pool, cores)
        cpu = {"value": round(rate, 3), "unit": "rows/s", "cores": cores, "kind": "port",
               "sample": f"{len(sample_rows)} rows of the same batch, token-only float64 restatement "
                         f"of the reference's steps, {cores} processes, {dt:.1f}s"}
        pool.close()
    return {
        "metric": METRIC, "value": round(value, 1), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Zipf-like logits, no dataset exists for this path)",
        "config": config3_config(B, V, world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profiled_traffic(),
                     "traffic_unit": "DRAM bytes per launch (ncu, profiles/stream_kernel_config3_full.md)",
                     "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                     "alg_bytes_per_launch": alg_bytes, "avg_launch_us": round(avg_launch_ms * 1e3, 2)},
        "e2e": {"value": round(e2e_value, 1), "unit": "rows/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * launches_per_call(),
        "clocks": clocks.summary(),
        "sharded": shard,
    }


def sharded_line(args, rank, world, dev, peak):
    """Config 5 (1024 x 256000 fp32, top_k 50, top_p 0.95, T 0.9) with the
    vocabulary split into contiguous slices over the ranks, sampled through
    ShardedSampler.sample: the default path, the fused peer exchange (the
    streaming kernel stores each row's record, every word tagged with the
    call's epoch, into every other rank's buffer over NVLink; the merge
    kernel waits for each row's tags), and beside it the all-gather path
    (shard pass, NCCL all-gather of the candidate records, merge kernel).  Strong scaling: the same rows
    on every N.  Each phase timed with CUDA events on the launching stream;
    the step time is the max over ranks."""
    import torch
    import torch.distributed as dist
    from miniserve_b200 import sharded, workloads
    b = workloads.config5(5)
    B, V = b.B, b.V
    v0, v1 = sharded.shard_bounds(V, world, rank)
    x = torch.from_numpy(b.logits[:, v0:v1].copy()).to(dev)
    del b.logits
    U = torch.from_numpy(b.uniforms).to(dev)
    T, K, P = float(b.temperature[0]), int(b.top_k[0]), float(b.top_p[0])  # uniform over the rows
    steps = max(3, min(args.steps, 20))

    def run(mode):
        ss = sharded.ShardedSampler(V, exchange=mode)
        for _ in range(max(args.warmup, 3)):
            ss.sample(x, v0, T, K, P, uniforms=U)
        torch.cuda.synchronize()
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            tok, prob, st = ss.sample(x, v0, T, K, P, uniforms=U, events=evs[i])
        torch.cuda.synchronize()
        used = ss.last_exchange
        ss.close()
        ph = torch.tensor([[e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2]), e[2].elapsed_time(e[3])]
                           for e in evs], dtype=torch.float64, device=dev)
        per_step = ph.sum(dim=1)
        stats = torch.stack([per_step.mean(), ph[:, 0].mean(), ph[:, 1].mean(), ph[:, 2].mean()])
        if world > 1:
            dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        return used, [float(v) for v in stats.tolist()], int((st != 0).sum())

    try:
        used, (step_ms, k_ms, m_ms, _), flagged = run("auto")
        peer_error = None
    except sharded.PeerExchangeError as e:  # every rank raises it (bounded waits that ran out)
        used, peer_error = "nccl", str(e)
    _, (g_step, g_shard, g_gather, g_merge), g_flagged = run("nccl")
    if peer_error is not None:
        step_ms, flagged = g_step, g_flagged
    alg = B * ((v1 - v0) * 4 + 52)  # this rank's logits slice and per-row parameters
    gather = {"value": round(B / (g_step / 1e3), 1), "unit": "rows/s", "ms_per_step": round(g_step, 5),
              "phase_us": {"shard_pass": round(g_shard * 1e3, 2), "all_gather": round(g_gather * 1e3, 2),
                           "merge": round(g_merge * 1e3, 2)},
              "gather_bytes_per_rank": B * sharded.record_words(50) * 4, "rows_flagged": g_flagged}
    line = {
        "workload": "config5: 1024x256000 fp32, vocab sliced over the GPUs, top_k 50, top_p 0.95, T 0.9",
        "api": "miniserve_b200.sharded.ShardedSampler.sample", "scaling": "strong", "ranks": world,
        "exchange": used,
        "value": round(B / (step_ms / 1e3), 1), "unit": "rows/s", "ms_per_step": round(step_ms, 5),
        "rows_flagged": flagged, "steps": steps,
        "timing": "CUDA events per phase on the launching stream, max over ranks; device time",
    }
    if used == "peer":
        line["phase_us"] = {"shard_pass_with_peer_stores": round(k_ms * 1e3, 2),
                            "merge_with_tag_wait": round(m_ms * 1e3, 2)}
        line["peer_bytes_per_rank"] = B * sharded.record_words(50) * 8 * max(world - 1, 0)
        kernel_ms, kname = k_ms, "shard pass with peer stores"
        line["all_gather_path"] = gather
    else:
        line["phase_us"] = gather["phase_us"]
        line["gather_bytes_per_rank"] = gather["gather_bytes_per_rank"]
        kernel_ms, kname = g_shard, "shard pass"
        line["peer_exchange"] = {"unavailable": peer_error or "CUDA IPC mapping of the exchange buffers failed"}
    line["per_gpu_hbm"] = {"achieved": round(alg / (kernel_ms / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(alg / (kernel_ms / 1e3) / 1e9 / peak, 4), "kernel": kname}
    return line


# ------------------------------------------------------- other BASELINE configs
def _time_ms(step, steps, warmup, stream, world):
    """Device ms per step: CUDA events on the launching stream, max over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) / steps


def run_workload(args, rank, world, local_rank):
    """--workload config2 / config4 / config5: the BASELINE configurations other
    than the metric's, device-timed (one JSON line, rank 0)."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from miniserve_b200 import _lib, sharded, workloads
    from miniserve_b200.grammar import JsonMaskBuilder
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    peak, _ = hbm_peak()
    out = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
           "vs_baseline": None, "data": "synthetic (seeded; BASELINE.json configuration)"}
    clocks = ClockSampler(local_rank).__enter__()
    clocks.wait_first()
    if args.workload == "config1":
        lines = {}
        for greedy in (False, True):
            b = workloads.config1(1 + rank, greedy=greedy)
            B, V = b.B, b.V
            x = torch.from_numpy(b.logits).to(dev)
            T, K, P, U = (torch.from_numpy(a).to(dev) for a in (b.temperature, b.top_k, b.top_p, b.uniforms))
            tok = torch.empty(B, dtype=torch.int64, device=dev)
            prob = torch.empty(B, dtype=torch.float32, device=dev)
            st = torch.empty(B, dtype=torch.int32, device=dev)

            def step():
                _lib.check(L.ms_sample(x.data_ptr(), 0, B, V, V, T.data_ptr(), K.data_ptr(), P.data_ptr(),
                                       U.data_ptr(), None, 0, tok.data_ptr(), prob.data_ptr(), st.data_ptr(),
                                       sptr), "ms_sample")
            lines["greedy" if greedy else "sampled"] = _time_ms(step, args.steps, args.warmup, stream, world)
        ms = lines["sampled"]
        out.update(metric="latency of one 8x151936 sampling call (config 1)", value=round(ms * 1e3, 2),
                   unit="us/call", higher_is_better=False, ms_per_step=round(ms, 5), scaling="weak",
                   dtype="f32", config={"workload": "config1: 8x151936 fp32, T 0.7, top_k 50, top_p 0.9",
                                        "batch_rows": 8, "vocab": 151936},
                   greedy_us_per_call=round(lines["greedy"] * 1e3, 2),
                   note="latency-bound (8 rows on 148 SMs); the L2 holds the 4.9 MB batch between calls")
    elif args.workload == "cliff":
        # config 3 with one NaN row and one top_k 300 row: the cost of rows the
        # streaming passes do not finish (the NaN row takes the generic kernel)
        b = workloads.config3(3 + rank)
        B, V = b.B, b.V
        logits = b.logits.copy()
        logits[5, 1234] = np.nan
        K = b.top_k.copy()
        K[6] = 300
        x = torch.from_numpy(logits).to(dev)
        x0 = torch.from_numpy(b.logits).to(dev)
        T, Kt, K0, P, U = (torch.from_numpy(a).to(dev) for a in (b.temperature, K, b.top_k, b.top_p, b.uniforms))
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)

        def call(xx, kk):
            _lib.check(L.ms_sample(xx.data_ptr(), 0, B, V, V, T.data_ptr(), kk.data_ptr(), P.data_ptr(),
                                   U.data_ptr(), None, 0, tok.data_ptr(), prob.data_ptr(), st.data_ptr(), sptr),
                       "ms_sample")
        ms_clean = _time_ms(lambda: call(x0, K0), args.steps, args.warmup, stream, world)
        ms = _time_ms(lambda: call(x, Kt), args.steps, args.warmup, stream, world)
        nonfinite = int((st.cpu() & _lib.MS_ROW_NONFINITE != 0).sum())
        out.update(metric="config 3 with one NaN row and one top_k 300 row: us per 512-row call",
                   value=round(ms * 1e3, 2), unit="us/call", higher_is_better=False, ms_per_step=round(ms, 5),
                   scaling="weak", dtype="f32",
                   config={"workload": "config3 + row 5 holding a NaN + row 6 with top_k 300", "batch_rows": B,
                           "vocab": V},
                   clean_us_per_call=round(ms_clean * 1e3, 2), ratio_to_clean=round(ms / ms_clean, 3),
                   rows_nonfinite=nonfinite)
    elif args.workload == "config2":
        b = workloads.config2(2 + rank)
        B, V = b.B, b.V
        esz = 2 if args.bf16 else 4
        x = torch.from_numpy(b.logits).to(dev)
        if args.bf16:
            x = x.to(torch.bfloat16)
        T, K, P, U = (torch.from_numpy(a).to(dev) for a in (b.temperature, b.top_k, b.top_p, b.uniforms))
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)

        def step():
            _lib.check(L.ms_sample(x.data_ptr(), 1 if args.bf16 else 0, B, V, V, T.data_ptr(), K.data_ptr(),
                                   P.data_ptr(), U.data_ptr(), None, 0, tok.data_ptr(), prob.data_ptr(),
                                   st.data_ptr(), sptr), "ms_sample")
        ms = _time_ms(step, args.steps, args.warmup, stream, world)
        alg = B * (V * esz + 52)
        out.update(metric="logits rows sampled/sec at 256x151936 greedy + temperature (config 2)",
                   value=round(world * B / (ms / 1e3), 1), unit="rows/s", ms_per_step=round(ms, 5),
                   scaling="weak", dtype="bf16" if args.bf16 else "f32",
                   config={"workload": "config2", "batch_rows": B, "vocab": V},
                   roofline={"bound": "hbm", "achieved": round(alg / (ms / 1e3) / 1e9, 1), "peak": peak,
                             "unit": "GB/s", "frac": round(alg / (ms / 1e3) / 1e9 / peak, 4), "traffic": None})
    elif args.workload == "config4":
        b = workloads.config4(4 + rank)
        B, V = b.B, b.V
        builder = JsonMaskBuilder(b.extra["vocab"], device=dev)
        states = builder.init(b.extra["prefixes"])
        x = torch.from_numpy(b.logits).to(dev)
        T, K, P, U = (torch.from_numpy(a).to(dev) for a in (b.temperature, b.top_k, b.top_p, b.uniforms))
        W = (V + 31) // 32
        mask = torch.empty((B, W), dtype=torch.int32, device=dev)
        mst = torch.empty(B, dtype=torch.int32, device=dev)
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)

        def build():  # the builder's default path: fixed-width tokens in (length, bytes) order
            _lib.check(L.ms_build_json_mask_ordered(states.data_ptr(), B, builder.vocab_bytes.data_ptr(),
                                                    builder.vocab_off.data_ptr(), builder.packed.data_ptr(),
                                                    builder.lens.data_ptr(), builder.order.data_ptr(), V,
                                                    mask.data_ptr(), W, mst.data_ptr(), sptr),
                       "ms_build_json_mask_ordered")

        def sample():
            _lib.check(L.ms_sample(x.data_ptr(), 0, B, V, V, T.data_ptr(), K.data_ptr(), P.data_ptr(),
                                   U.data_ptr(), mask.data_ptr(), W, tok.data_ptr(), prob.data_ptr(),
                                   st.data_ptr(), sptr), "ms_sample")

        def step():
            build()
            sample()
        ms_build = _time_ms(build, args.steps, args.warmup, stream, world)
        ms_sample = _time_ms(sample, args.steps, args.warmup, stream, world)
        ms = _time_ms(step, args.steps, args.warmup, stream, world)
        alg = B * (V * 4 + 4 * W + 52)
        out.update(metric="JSON-grammar rows sampled/sec at 128x151936 (config 4: mask build + masked sampling)",
                   value=round(world * B / (ms / 1e3), 1), unit="rows/s", ms_per_step=round(ms, 5),
                   scaling="weak", dtype="f32",
                   config={"workload": "config4", "batch_rows": B, "vocab": V,
                           "vocab_bytes": int(builder.vocab_bytes.numel()),
                           "prefix_chars": int(sum(len(p) for p in b.extra["prefixes"]))},
                   mask_build_us=round(ms_build * 1e3, 2), masked_sample_us=round(ms_sample * 1e3, 2),
                   roofline={"bound": "hbm", "kernel": "masked sampling",
                             "achieved": round(alg / (ms_sample / 1e3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(alg / (ms_sample / 1e3) / 1e9 / peak, 4), "traffic": None})
    elif args.workload == "graphed":
        # a decode step shaped like Qwen2.5-0.5B's last layer (hidden 896, fp32
        # LM head over 151936 tokens, the max bucket of 32 rows) captured as a
        # CUDA graph: the reference flow (replay, clone of the static logits,
        # sampling of the clone) against sampling captured into the graph,
        # reading the static buffer in place
        from miniserve_b200.graphed import GraphedSampler
        B, V, d = 32, workloads.QWEN_VOCAB, 896
        gen = torch.Generator(device="cpu").manual_seed(6 + rank)
        head = (torch.randn(V, d, generator=gen) * 0.05).to(dev)
        hidden = torch.randn(B, d, generator=gen).to(dev)
        out_buf = torch.zeros(B, V, dtype=torch.float32, device=dev)
        gs = GraphedSampler(out_buf)
        seeds = [1000 + i for i in range(B)]
        gs.set_params(B, temperature=0.7, top_k=50, top_p=0.9, seeds=seeds)

        def lm_head():
            out_buf[:B] = hidden @ head.T

        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            lm_head()
        stream.wait_stream(side)
        g_ref, g_ours = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_ref):
            lm_head()
        with torch.cuda.graph(g_ours):
            lm_head()
            gs.enqueue(B)
        torch.cuda.synchronize(dev)
        T, K, P = gs.temperature[:B].clone(), gs.top_k[:B].clone(), gs.top_p[:B].clone()
        U = gs.uniforms[:B].clone()
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)

        def sample_on(x):
            _lib.check(L.ms_sample(x.data_ptr(), 0, B, V, V, T.data_ptr(), K.data_ptr(), P.data_ptr(),
                                   U.data_ptr(), None, 0, tok.data_ptr(), prob.data_ptr(), st.data_ptr(),
                                   sptr), "ms_sample")

        def step_ref():  # model_runner.py:321, then the sampler on the copy
            g_ref.replay()
            sample_on(out_buf[:B].clone())

        ms_head = _time_ms(g_ref.replay, args.steps, args.warmup, stream, world)
        ms_ref = _time_ms(step_ref, args.steps, args.warmup, stream, world)
        ms = _time_ms(g_ours.replay, args.steps, args.warmup, stream, world)
        ms_sample = _time_ms(lambda: sample_on(out_buf), args.steps, args.warmup, stream, world)
        same = torch.equal(tok, gs.result(B)[0])
        out.update(metric="decode-step rows/s at B 32 (fp32 LM head 896 -> 151936 + sampling in one CUDA graph)",
                   value=round(world * B / (ms / 1e3), 1), unit="rows/s", ms_per_step=round(ms, 5),
                   scaling="weak", dtype="f32",
                   config={"workload": "graphed: LM head [151936, 896] fp32, B 32, T 0.7, top_k 50, top_p 0.9",
                           "batch_rows": B, "vocab": V, "hidden": d},
                   in_graph_us=round(ms * 1e3, 2), clone_flow_us=round(ms_ref * 1e3, 2),
                   lm_head_us=round(ms_head * 1e3, 2), sampling_us=round(ms_sample * 1e3, 2),
                   clone_bytes_per_step=B * V * 4, tokens_equal=bool(same),
                   note="the clone flow copies the static logits before sampling (model_runner.py:321); "
                        "the in-graph flow samples them in place")
        del g_ref, g_ours
    elif args.workload == "nucleus":
        # config 5's logits with top_k off (top_p 0.95 and top_p 1 rows, T 0.9
        # and 1.5), vocab-sharded over the ranks, through ShardedSampler: rows
        # the records settle, rows the distributed nucleus finishes (no logits
        # exchanged), against the full-row path for the same rows (all-gather
        # of their logits and ms_sample on every rank)
        B = 256
        b = workloads.config5(5, B=B)
        V = b.V
        v0, v1 = sharded.shard_bounds(V, world, rank)
        x = torch.from_numpy(np.ascontiguousarray(b.logits[:, v0:v1])).to(dev)
        del b.logits
        rng = np.random.default_rng(55)
        Th = np.where(rng.random(B) < 0.5, 0.9, 1.5)
        Ph = np.where(rng.random(B) < 0.25, 1.0, 0.95)
        Kh = np.zeros(B, np.int32)
        T, K, P, U = (torch.from_numpy(a).to(dev) for a in (Th, Kh, Ph, b.uniforms))
        ss = sharded.ShardedSampler(V)
        kmax = sharded.choose_kmax(Kh.tolist(), Th.tolist(), Ph.tolist(), V)

        def step():
            ss.sample(x, v0, T, K, P, uniforms=U, kmax=kmax)

        ms = _time_ms(step, args.steps, args.warmup, stream, world)
        tok, prob, st = ss.sample(x, v0, T, K, P, uniforms=U, kmax=kmax)
        n_nuc, n_full = ss.last_nucleus_rows, ss.last_full_rows
        rows = torch.arange(B, device=dev)
        single = sharded.Sampler()

        def full_rows():  # the alternative for every row: gather the logits, sample the full rows
            full = sharded.gather_rows(x, rows, V)
            single.sample_batch(full, T, K, P, uniforms=U)

        ms_full = _time_ms(full_rows, args.steps, args.warmup, stream, world)
        out.update(metric="rows/s of vocab-sharded rows without top-k (config-5 logits, 256 rows)",
                   value=round(B / (ms / 1e3), 1), unit="rows/s", ms_per_step=round(ms, 5), scaling="strong",
                   dtype="f32",
                   config={"workload": "nucleus: config-5 logits 256x256000 fp32, top_k 0, top_p 0.95/1.0, "
                                       "T 0.9/1.5, vocab sliced over the GPUs",
                           "batch_rows": B, "vocab": V, "nccl_ranks": world, "kmax": kmax},
                   rows_settled_by_records=B - n_nuc - n_full, rows_distributed_nucleus=n_nuc,
                   rows_full_row_path=n_full, full_row_gather_us=round(ms_full * 1e3, 2),
                   full_row_gather_bytes_per_rank=B * (v1 - v0) * 4,
                   note="device time of the whole call (CUDA events), host reads of the flag counts included")
    else:  # config5: vocab-sharded over the ranks
        b = workloads.config5(5)
        B, V = b.B, b.V
        v0, v1 = sharded.shard_bounds(V, world, rank)
        x = torch.from_numpy(np.ascontiguousarray(b.logits[:, v0:v1])).to(dev)
        del b.logits
        T, K, P, U = (torch.from_numpy(a).to(dev) for a in (b.temperature, b.top_k, b.top_p, b.uniforms))
        kmax = 50
        Wr = sharded.record_words(kmax)
        rec = torch.empty((B, Wr), dtype=torch.int32, device=dev)
        allrec = torch.empty((world * B, Wr), dtype=torch.int32, device=dev)
        tok = torch.empty(B, dtype=torch.int64, device=dev)
        prob = torch.empty(B, dtype=torch.float32, device=dev)
        st = torch.empty(B, dtype=torch.int32, device=dev)

        def step():
            _lib.check(L.ms_shard_candidates(x.data_ptr(), 0, B, v1 - v0, v1 - v0, v0, V, T.data_ptr(),
                                             K.data_ptr(), None, 0, kmax, rec.data_ptr(), sptr),
                       "ms_shard_candidates")
            if world > 1:
                dist.all_gather_into_tensor(allrec, rec)
                src = allrec
            else:
                src = rec
            _lib.check(L.ms_shard_merge(src.data_ptr(), world, B, kmax, V, T.data_ptr(), K.data_ptr(),
                                        P.data_ptr(), U.data_ptr(), tok.data_ptr(), prob.data_ptr(),
                                        st.data_ptr(), sptr), "ms_shard_merge")
        ms = _time_ms(step, args.steps, args.warmup, stream, world)
        alg = B * ((v1 - v0) * 4 + 52)
        out.update(metric="logits rows sampled/sec at 1024x256000, vocab sharded over the GPUs (config 5)",
                   value=round(B / (ms / 1e3), 1), unit="rows/s", ms_per_step=round(ms, 5), scaling="strong",
                   dtype="f32", config={"workload": "config5", "batch_rows": B, "vocab": V,
                                        "parallelism": f"vocab slices x{world}", "kmax": kmax,
                                        "gather_bytes_per_rank": B * Wr * 4},
                   roofline={"bound": "hbm", "per_gpu": True, "achieved": round(alg / (ms / 1e3) / 1e9, 1),
                             "peak": peak, "unit": "GB/s", "frac": round(alg / (ms / 1e3) / 1e9 / peak, 4),
                             "traffic": None})
    clocks.__exit__(None, None, None)
    out["clocks"] = clocks.summary()
    return out if rank == 0 else None


def launches_per_call():
    """ms_sample launches the streaming kernel and the pending-row pass."""
    return 2


def run_reference(args, rank):
    """Reference arm: the reference algorithm on host cores, bounded sample per step."""
    from miniserve_b200 import workloads
    if rank != 0:
        return None
    cores = os.cpu_count() or 1
    pool = mp.get_context("spawn").Pool(cores)
    batch = workloads.config3(3)
    n = min(batch.B, max(cores, 8))
    rows = list(range(n))
    for _ in range(args.warmup):
        cpu_reference_rate(batch, rows[: min(n, cores)], pool, cores)
    times = []
    for s in range(args.steps):
        rr = [(r + s * n) % batch.B for r in rows]
        t0 = time.perf_counter()
        cpu_reference_rate(batch, rr, pool, cores)
        times.append(time.perf_counter() - t0)
    pool.close()
    total = sum(times)
    value = n * args.steps / total
    sample = (f"{n} rows per step of the 512-row batch; token-only float64 restatement of "
              f"miniserve Sampler.sample (its steps and builtin calls), {cores} processes")
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded Zipf-like logits)",
        "config": config3_config(batch.B, batch.V, args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["config3", "config1", "config2", "config4", "config5", "cliff", "graphed",
                                           "nucleus"],
                    default="config3",
                    help="config3 (default) is the metric's configuration; the others print their own line")
    ap.add_argument("--bf16", action="store_true", help="config2: bf16 logits")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        out = run_reference(args, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        out = run_ours(args, rank, world, local_rank) if args.workload == "config3" else \
            run_workload(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
