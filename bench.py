#!/usr/bin/env python3
"""Benchmark of the paged-KV GQA decode operator (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

A step is one decode call over one batch: config 2 (Llama-3-8B-shaped,
B=64, L=4096, Hq=32, Hkv=8, D=128, page 256, bf16) unless --config says
otherwise.  Inputs are seeded synthetic tensors; the 1 GiB KV cache is larger
than the 126 MB L2, so no flush is needed between steps.

N > 1 (torchrun, one process per GPU): every rank decodes its own batch of
the same shape (batch sharding of a B*N batch, no data-path collective, weak
scaling); the time is the max over ranks of CUDA-event time.

--impl reference times the reference path's CPU restatement (the oracle;
the reference itself targets a MetaX GPU and has no CPU implementation) on
the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flashatte-hand_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "decode µs/call & KV HBM GB/s (% of B200 peak), B=64 L=4096 GQA-4 bf16"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="budget of the cpu_baseline leg (rank 0, N=1)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--shard", default="auto", choices=["auto", "heads"],
                    help="N>1: the config's default partition, or KV-head sharding")
    ap.add_argument("--kv", default="native", choices=["native", "fp8"],
                    help="K/V cache storage: the config's dtype, or e4m3 with per-head scales")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(workload: str):
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"decode_sm100_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """NVML SM clock / throttle-reason samples on a background thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], set()
        self.period = period_s
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # no NVML: report no samples
            self.max_mhz = None
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2] if s else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(s), "source": "nvml"}


def cpu_oracle_rate(case, tensors, budget_s: float, rows=None):
    """KV GB/s of the CPU oracle over whole sequences, within ~budget_s."""
    from oracle.decode_ref import decode_reference
    torch.set_num_threads(os.cpu_count() or 1)
    es = torch.empty((), dtype=case.dtype).element_size()
    order = rows if rows is not None else list(range(case.B))
    done_bytes, t0, n = 0, time.perf_counter(), 0
    while time.perf_counter() - t0 < budget_s:  # whole sequences, cycling over the batch
        b = order[n % len(order)]
        decode_reference(tensors["q"], tensors["k_cache"], tensors["v_cache"], tensors["cache_seqlens"],
                         tensors["block_table"], softmax_scale=case.softmax_scale, rows=[b])
        done_bytes += max(int(case.seqlens[b]), 0) * case.Hkv * case.D * 2 * es
        n += 1
    dt = time.perf_counter() - t0
    return done_bytes / dt / 1e9, n, dt


def run_reference(args, rank, world):
    """--impl reference: the CPU restatement on the host cores, rank 0 only."""
    if rank != 0:
        return
    from flashdecode import cases
    case = cases.config_case(args.config)
    tensors = cases.materialize(case, "cpu")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle.decode_ref import decode_reference
    es = torch.empty((), dtype=case.dtype).element_size()
    # Each step processes a bounded sample: the first `per_step` sequences,
    # sized so the whole run stays within about two minutes.
    t0 = time.perf_counter()
    decode_reference(tensors["q"], tensors["k_cache"], tensors["v_cache"], tensors["cache_seqlens"],
                     tensors["block_table"], softmax_scale=case.softmax_scale, rows=[0])
    one = time.perf_counter() - t0
    per_step = max(1, min(case.B, int(120.0 / max(one, 1e-6) / max(args.steps + args.warmup, 1))))
    rows = list(range(per_step))
    for _ in range(min(args.warmup, 3)):
        decode_reference(tensors["q"], tensors["k_cache"], tensors["v_cache"], tensors["cache_seqlens"],
                         tensors["block_table"], softmax_scale=case.softmax_scale, rows=rows)
    steps = args.steps
    t0 = time.perf_counter()
    deadline = t0 + 150.0
    done = 0
    for _ in range(steps):
        decode_reference(tensors["q"], tensors["k_cache"], tensors["v_cache"], tensors["cache_seqlens"],
                         tensors["block_table"], softmax_scale=case.softmax_scale, rows=rows)
        done += 1
        if time.perf_counter() > deadline:
            break
    dt = time.perf_counter() - t0
    kv = sum(max(int(case.seqlens[b]), 0) for b in rows) * case.Hkv * case.D * 2 * es
    gbs = kv * done / dt / 1e9
    sample = f"{per_step} of {case.B} sequences of {case.name} per step, {done} steps timed"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": world, "steps": done, "warmup": args.warmup,
        "ms_per_step": round(dt / done * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if case.dtype == torch.bfloat16 else "fp16",
        "data": "synthetic", "config": {"workload": case.name, "global_batch": case.B,
                                        "seq_len": int(case.seqlens.max()), "parallelism": "cpu"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import flashdecode
    from flashdecode import cases
    from flashdecode import dist as fdist

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    full = cases.config_case(args.config)
    lib = flashdecode.load_library()
    stream = torch.cuda.current_stream()
    splitter = None
    if world > 1 and args.shard == "heads":
        # every rank owns Hkv / N KV heads (and their query heads) of every sequence
        case, _qrange = fdist.head_shard(full, rank, world)
        scaling, parallel = "strong", f"kvheads{world}"
        total_kv = full.kv_bytes()
        t = cases.materialize(case, "cuda", seed=rank)
    elif world == 1 or args.config in (1, 2):
        # every rank decodes its own full batch: batch sharding of a B*N batch
        case, scaling, parallel = full, "weak", f"dp{world}"
        total_kv = full.kv_bytes() * world
        t = cases.materialize(case, "cuda", seed=rank)
    elif args.config in (3, 5):
        # the configured batch split over the ranks, longest sequences first
        case, _rows = fdist.batch_shard(full, rank, world)
        scaling, parallel = "strong", f"batch-shard{world}"
        total_kv = full.kv_bytes()
        t = cases.materialize(case, "cuda", seed=rank)
    else:
        # config 4: every rank holds a page range of each sequence; the decode
        # kernel pushes its partials to every rank over NVLink and a merge
        # kernel on each rank combines them
        case, _page_map = fdist.kv_split_case(full, rank, world)
        scaling, parallel = "strong", f"splitkv{world}-p2p"
        total_kv = full.kv_bytes()
        t = cases.materialize(case, "cuda", seed=0)  # same q on every rank
        splitter = fdist.PeerSplitKVDecode(case.B, case.Hq, case.D, case.dtype, "cuda")
    fp8 = args.kv == "fp8"
    if fp8:
        del t
        torch.cuda.empty_cache()
        # split-KV ranks share one query (seed 0), as above
        t = cases.materialize_e4m3(case, "cuda", seed=0 if splitter is not None else rank)
        total_kv //= 2
    kv_kw = dict(k_scale=t["k_scale"], v_scale=t["v_scale"]) if fp8 else {}
    max_len = max(int(case.seqlens.max()), 1)

    def decode(q, seqlens, bt):
        if splitter is not None:
            return splitter(q, t["k_cache"], t["v_cache"], seqlens, bt, case.softmax_scale, **kv_kw)
        return flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], seqlens, bt,
                                        softmax_scale=case.softmax_scale, return_softmax_lse=True,
                                        max_seqlen_k=max_len, **kv_kw)

    def step():
        decode(t["q"], t["cache_seqlens"], t["block_table"])

    launches_per_call = math.ceil(case.B / 512) + (1 if splitter is not None else 0)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist is not None:
        dist.barrier()
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    assert lib.fd_last_error() == 0

    # e2e: the public call with host buffers -- per-step inputs (q, seqlens,
    # block_table) copied from pinned host memory, output + LSE read back to
    # pinned host memory, every step inside the timed region.  As in a serving
    # loop the copies are double-buffered on two copy streams: step i+1's
    # inputs go in and step i-1's results come out while step i decodes.
    e2e = None
    if not args.no_e2e:
        hq = t["q"].cpu().pin_memory()
        hs = t["cache_seqlens"].cpu().pin_memory()
        hb = t["block_table"].cpu().pin_memory()
        ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]
        hl = [torch.empty((case.B, case.Hq), dtype=torch.float32).pin_memory() for _ in range(2)]
        dq = [torch.empty_like(t["q"]) for _ in range(2)]
        ds = [torch.empty_like(t["cache_seqlens"]) for _ in range(2)]
        db = [torch.empty_like(t["block_table"]) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer k landed
        ev_used = [torch.cuda.Event() for _ in range(2)]   # decode of buffer k done
        ev_out = [torch.cuda.Event() for _ in range(2)]    # results of buffer k read back
        for k in range(2):
            ev_used[k].record(stream)
            ev_out[k].record(stream)

        def e2e_step(i):
            k = i & 1
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_used[k])
                dq[k].copy_(hq, non_blocking=True)
                ds[k].copy_(hs, non_blocking=True)
                db[k].copy_(hb, non_blocking=True)
                ev_in[k].record(s_in)
            stream.wait_event(ev_in[k])
            stream.wait_event(ev_out[k])
            o, l = decode(dq[k], ds[k], db[k])
            ev_used[k].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_used[k])
                ho[k].copy_(o, non_blocking=True)
                hl[k].copy_(l, non_blocking=True)
                ev_out[k].record(s_out)
                o.record_stream(s_out)
                l.record_stream(s_out)

        for i in range(4):
            e2e_step(i)
        torch.cuda.synchronize()
        e_steps = max(10, min(args.steps, 500))
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        s_out.wait_event(e0)
        for i in range(e_steps):
            e2e_step(i)
        stream.wait_stream(s_out)
        stream.wait_stream(s_in)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / e_steps
        if dist is not None:
            tt = torch.tensor([e_ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        h2d = hq.numel() * hq.element_size() + hs.numel() * 4 + hb.numel() * 4
        d2h = ho[0].numel() * ho[0].element_size() + hl[0].numel() * 4
        e2e = {"value": round(total_kv / (e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "us_per_call": round(e_ms * 1e3, 2),
               "steps": e_steps, "copies": "double-buffered on two copy streams",
               "kv_cache": "resident in HBM (decode state, not a per-step input)"}

    if splitter is not None:
        splitter.close()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return

    per_call_s = ms * 1e-3 / args.steps
    kv_gbs = total_kv / per_call_s / 1e9
    alg_per_launch = case.algorithmic_bytes(with_lse=True) - (case.kv_bytes() // 2 if fp8 else 0)
    achieved = alg_per_launch / per_call_s / 1e9
    peak, peak_kind = peaks()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": (profile_traffic(f"cfg{args.config}" + ("_e4m3kv" if fp8 else ""))
                            if world == 1 else None),
                "peak_source": peak_kind, "kernel": "decode_sm100_kernel",
                "alg_bytes_per_launch": alg_per_launch}
    cpu = None
    if world == 1 and args.cpu_seconds > 0 and not fp8:
        ct = {k: v.cpu() for k, v in t.items()}
        rate, nseq, dt = cpu_oracle_rate(case, ct, args.cpu_seconds)
        cpu = {"value": round(rate, 4), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{nseq} sequence decodes (cycling over the {case.B} of {case.name}) "
                         f"in {dt:.1f}s, torch fp32 oracle"}
    line = {
        "metric": METRIC, "value": round(kv_gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_call_s * 1e3, 5),
        "us_per_call": round(per_call_s * 1e6, 2), "pct_of_peak": round(100 * kv_gbs / world / peak, 2),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": ("e4m3-kv/" if fp8 else "") + ("bf16" if case.dtype == torch.bfloat16 else "fp16"),
        "data": "synthetic",
        "config": {"workload": full.name + ("_e4m3kv" if fp8 else ""),
                   "global_batch": full.B * (world if scaling == "weak" else 1),
                   "seq_len": int(full.seqlens.max()), "parallelism": parallel,
                   "Hq": full.Hq, "Hkv": full.Hkv, "head_dim": full.D, "page": full.page,
                   "l2": "inputs larger than L2 (KV cache > 126 MB), no flush"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches_per_call * args.steps, "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
