"""Benchmark of the fused KV-append + GQA decode attention.

Workload: Llama-3-8B attention shape, F16, batch 1,
32 query / 8 KV heads, head_dim 128, 131072 cached positions with K,V ~ N(0,1) in a
16-token block-paged cache whose blocks are a seeded random permutation, one appended
token per step.  A step is one pass of the hot path: the new token's K/V written into its
paged slot and attention over all 131073 positions.  Lengths are not advanced between
steps, so every step appends at the same position and does identical work.  The 537 MB of
K/V read per step is larger than the 126 MB L2, so no flush is needed between steps.

At N > 1 GPUs the sequence is split along its positions (strong scaling: total work
fixed); each rank attends its share and the partial (O, lse) are exchanged and merged
inside the decode kernel itself over NVLink (``--exchange p2p``, the default: every rank's
final CTAs store their rows into the other ranks' buffers and merge what arrives), or
after one NCCL all-gather plus a merge kernel (``--exchange nccl``).

On one GPU consecutive steps are launched with programmatic dependent launch: a step's
block-table reads and first K/V copies may start while the previous step drains; it reads
q / k_new / v_new and writes anything only after the previous step has finished.

Other workloads are parity-test cases, not bench lines.

``--impl reference`` times the reference's algorithm on the host cores instead: the CPU
restatement of its Metal kernels (oracle/, faithful F16 chain, all cores), on the same
config, as many steps as fit a bounded time budget.
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
sys.path.insert(0, ROOT)

METRIC = ("decode tok/s; fused KV-append+GQA attn HBM GB/s vs B200 peak at 1/2/4/8 GPU")
HQ, HKV, D, CACHED, BS = 32, 8, 128, 131072, 16
ESIZE = 2
# The workload both arms report (the driver compares the two `config` dicts).
CFG4_CONFIG = {"workload": "cfg4 long-context decode attention op (Llama-3-8B attention "
                           "shape), 131072 cached + 1 appended, batch 1",
               "q_heads": HQ, "kv_heads": HKV, "head_dim": D, "cached": CACHED,
               "block_size": BS,
               "l2": "inputs larger than L2 (537 MB K/V per step vs 126 MB L2)"}
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one full-size launch of the
# tensor-core decode kernel, from one ncu capture of a 32768-position launch (reads scaled
# by the cached length, writes constant).  The figure belongs to the kernel source it was
# captured on: `roofline.traffic` is reported only while rustllm_b200/csrc/decode.cu still
# has that SHA-256.
NCU_TRAFFIC = {"bytes_per_launch": 537.5e6,
               "decode_cu_sha256": "7ceae295d2d81b3fba506620e6f933281e41c3f7b306a1bdbbc2e107034c7242"}
# Untimed steps run between the warm-up and the timed region so the GPU's clocks have left
# their idle state (the clock sampler's start-up pause idles the GPU for 0.4 s).
SETTLE_STEPS = 2000


def decode_cu_sha256() -> str:
    import hashlib
    with open(os.path.join(ROOT, "rustllm_b200", "csrc", "decode.cu"), "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def algorithmic_bytes(cached: int = CACHED, hq: int = HQ, hkv: int = HKV, d: int = D,
                      e: int = ESIZE, batch: int = 1) -> int:
    """Bytes one fused decode launch must move (the survey's per-call figure):
    K and V of all L = cached+1 positions, plus q, k_new, v_new read, the appended K/V
    written and the output written."""
    L = cached + 1
    return batch * (2 * hkv * L * d * e + hq * d * e + 2 * hkv * d * e + 2 * hkv * d * e
                    + hq * d * e)


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU while the timed loop runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.4)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self):
        return time.time()

    def stop(self, t0: float, t1: float) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            rows.append((ts, parts))
        inside = [r for ts, r in rows if t0 - 0.15 <= ts <= t1 + 0.15] or [r for _, r in rows]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in inside if num(r[1]) is not None]
        mx = [num(r[2]) for r in inside if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(inside),
                "power_w_max": max((num(r[3]) or 0.0) for r in inside)}


def profile_region(on: bool) -> None:
    """With TMLLM_PROFILE_REGION=1 the timed loop is bracketed by cudaProfilerStart/Stop, so
    a profiler started with --profile-from-start off sees only the timed steps."""
    if os.environ.get("TMLLM_PROFILE_REGION") == "1":
        import torch
        (torch.cuda.profiler.start if on else torch.cuda.profiler.stop)()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------
# CPU arm: the oracle (restatement of the reference's kernels) on the host cores
# ------------------------------------------------------------------------------------

def cpu_workload(seed: int = 1234):
    import numpy as np
    rng = np.random.default_rng(seed)
    L = CACHED + 1
    k = np.empty((1, HKV, L, D), np.float16)
    v = np.empty((1, HKV, L, D), np.float16)
    for h in range(HKV):
        k[0, h] = rng.standard_normal((L, D), dtype=np.float32)
        v[0, h] = rng.standard_normal((L, D), dtype=np.float32)
    q = rng.standard_normal((1, HQ, 1, D), dtype=np.float32).astype(np.float16)
    return q, k, v


def cpu_time(budget_s: float, max_steps: int, threads: int, data=None):
    """Runs the reference's chain (faithful F16) for the config-4 step until the budget or
    the step count is reached.  Returns (steps, seconds, threads)."""
    from oracle import oracle as orc
    orc.build()
    q, k, v = data if data is not None else cpu_workload()
    L = k.shape[2]
    steps, t0 = 0, time.perf_counter()
    while steps < max_steps:
        orc.attention_core(q, k, v, L, L - 1, threads=threads)
        steps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    return steps, time.perf_counter() - t0


def run_reference(args) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    data = cpu_workload()
    from oracle import oracle as orc
    orc.build()
    q, k, v = data
    for _ in range(min(args.warmup, 1)):
        orc.attention_core(q, k, v, k.shape[2], k.shape[2] - 1, threads=threads)
    steps, secs = cpu_time(args.ref_budget, args.steps, threads, data)
    tok_s = steps / secs
    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "impl": "reference",
        "n_gpus": world, "steps": steps, "warmup": min(args.warmup, 1),
        "ms_per_step": 1000.0 * secs / steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) K/V, q; random block permutation)",
        "config": dict(CFG4_CONFIG),
        "hbm_gbs_equiv": algorithmic_bytes() * tok_s / 1e9,
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{steps} full config-4 steps (all 32 query heads x 131073 "
                                   f"positions), time-boxed to {args.ref_budget:.0f} s"},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference is Rust + Apple Metal and cannot run on Linux; this arm runs "
                "the C restatement of its kernels (oracle/) on the host cores",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------

def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    import rustllm_b200 as rb
    from rustllm_b200.distributed import SequenceSplitAttention

    torch.manual_seed(1234 + rank)
    cached = args.cached
    overlap = (world == 1 or args.exchange == "p2p") and not args.no_overlap
    sp = SequenceSplitAttention(cached, HQ, HKV, D, dtype=torch.float16, block_size=BS,
                                shuffle_seed=77 + rank, device=dev, variant=args.variant,
                                num_splits=args.splits, exchange=args.exchange,
                                overlap=overlap)
    n_local = sp.hi - sp.lo
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    # fill in slabs to bound the temporary footprint
    slab = 16384
    k_hold = []
    for lo in range(0, n_local, slab):
        m = min(slab, n_local - lo)
        kk = torch.randn((HKV, m, D), generator=g, device=dev).half()
        vv = torch.randn((HKV, m, D), generator=g, device=dev).half()
        sp.cache.append(0, 0, kk, vv)
        sp.cache.advance(m, 0)
        del kk, vv
    q = torch.randn((1, HQ, D), generator=g, device=dev).half()
    kn = torch.randn((1, HKV, D), generator=g, device=dev).half()
    vn = torch.randn((1, HKV, D), generator=g, device=dev).half()
    out = torch.empty((1, HQ, D), dtype=torch.float16, device=dev)
    torch.cuda.synchronize()

    def step():
        sp.step(q, kn, vn, out)

    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()  # idles the GPU for 0.4 s: the warm-up and settle steps follow it
    for _ in range(args.warmup):
        step()
    # the same fixed count on every rank (the exchange pairs the ranks' calls step by step)
    for _ in range(args.settle):
        step()
    # (1) the timed steps: one fused launch each (plus the all-gather and merge with
    # --exchange nccl), no other host work inside the loop
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    profile_region(True)
    wall0 = time.time()
    h0 = time.perf_counter()
    t_start.record(stream)
    for _ in range(args.steps):
        sp.step(q, kn, vn, out)
    t_end.record(stream)
    host_us = (time.perf_counter() - h0) * 1e6 / args.steps  # host submission per step
    torch.cuda.synchronize()
    profile_region(False)
    wall1 = time.time()
    # (2) the decode kernel alone, per launch (CUDA events around each launch)
    n_k = min(args.steps, 1000)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_k)]
    if world > 1:
        dist.barrier()
    for i in range(n_k):
        kev[i][0].record(stream)
        if world == 1 or args.exchange == "p2p":
            sp.step(q, kn, vn, out)  # one launch: the fused kernel writes `out`
            kev[i][1].record(stream)
        else:
            sp.attend_local(q, kn, vn)
            kev[i][1].record(stream)
            sp.exchange_and_merge(out)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = t_start.elapsed_time(t_end)
    k_ms = sum(a.elapsed_time(b) for a, b in kev) / n_k
    # per-rank timeline (N > 1): this rank's share attended alone (the same fused kernel
    # without the exchange, consecutive launches overlapped), against the exchanged step
    local_ms = None
    if world > 1:
        lo = torch.empty((1, HQ, D), dtype=torch.float32, device=dev)
        ll = torch.empty((1, HQ), dtype=torch.float32, device=dev)
        kwl = dict(out=lo, lse=ll, overlap=not args.no_overlap, num_splits=args.splits,
                   variant=args.variant)
        for _ in range(20):
            sp.cache.decode(0, q, kn if sp.owner else None, vn if sp.owner else None, **kwl)
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_l = min(args.steps, 2000)
        l0.record(stream)
        for _ in range(n_l):
            sp.cache.decode(0, q, kn if sp.owner else None, vn if sp.owner else None, **kwl)
        l1.record(stream)
        torch.cuda.synchronize()
        local_ms = l0.elapsed_time(l1) / n_l
        dist.barrier()
    clocks = sampler.stop(wall0, wall1) if sampler else None
    per_rank = None
    if world > 1:
        mine = torch.tensor([ms_total / args.steps * 1e3, local_ms * 1e3, host_us],
                            dtype=torch.float64, device=dev)
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [{"rank": r, "step_us": float(x[0]), "local_attention_us": float(x[1]),
                     "host_submit_us": float(x[2])} for r, x in enumerate(allr)]
    t = torch.tensor([ms_total, k_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, k_ms = float(t[0]), float(t[1])
    ms_step = ms_total / args.steps
    tok_s = 1000.0 / ms_step
    k_ms_events = k_ms
    if world == 1 or args.exchange == "p2p":
        # a step is exactly one launch of the fused kernel: its average duration is the
        # timed region's device time per step (the per-launch events of loop (2) add the
        # host's event records between launches)
        k_ms = ms_step

    # e2e through the public API with host buffers: the step's q, k_new and v_new live in
    # one pinned host buffer (one host-to-device copy per step, views on the device side);
    # out comes back to pinned host memory.  Two forms, both with every copy inside the
    # timed region: serial (copy in, kernel, copy out on one stream) and pipelined, as a
    # serving loop runs it: two device buffer sets, the next step's input copy on a copy
    # stream while this step's kernel runs, this step's read-back on a third stream while
    # the next kernel runs.
    nq, nk = HQ * D, HKV * D
    hin = [torch.randn((nq + 2 * nk,)).half().pin_memory() for _ in range(2)]
    hout = [torch.empty((1, HQ, D), dtype=torch.float16).pin_memory() for _ in range(2)]
    din = [torch.empty((nq + 2 * nk,), dtype=torch.float16, device=dev) for _ in range(2)]
    dout = [out] + [torch.empty_like(out)]
    views = [(x[:nq].view(1, HQ, D), x[nq:nq + nk].view(1, HKV, D),
              x[nq + nk:].view(1, HKV, D)) for x in din]
    e_steps = max(1, min(args.steps, 2000))
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # input copy into set b done
    ev_k = [torch.cuda.Event() for _ in range(2)]     # kernel that read set b done
    ev_out = [torch.cuda.Event() for _ in range(2)]   # read-back of set b done
    for b in range(2):
        ev_k[b].record(stream)
        ev_out[b].record(stream)

    def e2e_serial():
        din[0].copy_(hin[0], non_blocking=True)
        sp.step(*views[0], dout[0])
        hout[0].copy_(dout[0], non_blocking=True)

    def e2e_pipelined(i):
        b = i & 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_k[b])             # the kernel that last read set b is done
            din[b].copy_(hin[b], non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])             # set b's previous result is on the host
        sp.step(*views[b], dout[b])
        ev_k[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_k[b])
            hout[b].copy_(dout[b], non_blocking=True)
            ev_out[b].record(s_out)

    def timed_e2e(fn, pipelined):
        for i in range(3):
            fn(i) if pipelined else fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(e_steps):
            fn(i) if pipelined else fn()
        if pipelined:
            stream.wait_event(ev_out[0])
            stream.wait_event(ev_out[1])
        e1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return 1000.0 * e_steps / float(te[0])

    e2e_serial_tok_s = timed_e2e(e2e_serial, False)
    e2e_tok_s = timed_e2e(e2e_pipelined, True)
    h2d = hin[0].numel() * 2
    d2h = hout[0].numel() * 2

    if rank == 0:
        peaks = load_peaks()
        launch_bytes = algorithmic_bytes(cached=n_local if world > 1 else cached)
        if world > 1 and not sp.owner:
            launch_bytes = 2 * HKV * n_local * D * ESIZE + 2 * HQ * D * ESIZE
        achieved = launch_bytes / (k_ms * 1e-3) / 1e9
        traffic, traffic_note = None, "no ncu capture of this kernel source"
        if args.traffic is not None:
            traffic, traffic_note = args.traffic, "given on the command line"
        elif (world == 1 and cached == CACHED and args.variant != 1
              and NCU_TRAFFIC["decode_cu_sha256"] == decode_cu_sha256()):
            traffic = NCU_TRAFFIC["bytes_per_launch"]
            traffic_note = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                            "32768-position launch, reads scaled to 131073 positions; "
                            "captured on this decode.cu (sha256 "
                            f"{NCU_TRAFFIC['decode_cu_sha256'][:12]})")
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) K/V, q; random block permutation)",
            "config": dict(CFG4_CONFIG),
            "parallelism": (f"seqsplit{world}-{args.exchange}" if world > 1 else "1gpu"),
            "settle_steps": args.settle,
            "overlapped_launches": overlap,
            "hbm_gbs": algorithmic_bytes(cached=cached) / (ms_step * 1e-3) / 1e9,
            "gpu_launches": args.steps * (2 if world > 1 and args.exchange == "nccl" else 1),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "peak_source": peaks["source"], "traffic": traffic,
                         "traffic_source": traffic_note,
                         "kernel": ("decode_split_kernel<__half,128,4,64,3>" if args.variant == 1
                                    else "decode_mma_kernel<128,3>"),
                         "kernel_ms": k_ms, "kernel_ms_single_launch_events": k_ms_events,
                         "bytes_per_launch": launch_bytes},
            "e2e": {"value": e2e_tok_s, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "form": "pipelined (2 buffer sets, 3 streams)",
                    "serial_value": e2e_serial_tok_s},
            "clocks": clocks,
        }
        if per_rank is not None:
            line["per_rank"] = per_rank
        if cached != CACHED:
            line["config"]["cached"] = cached
            line["config"]["workload"] += f" (reduced to {cached} cached for a capture)"
        if world == 1 and not args.no_cpu:
            import numpy as np
            kd, vd = sp.cache.gather(0, 0)
            L = cached + 1
            kc = np.empty((1, HKV, L, D), np.float16)
            vc = np.empty((1, HKV, L, D), np.float16)
            kc[0, :, :cached] = kd.cpu().numpy()
            vc[0, :, :cached] = vd.cpu().numpy()
            kc[0, :, cached] = kn[0].cpu().numpy()
            vc[0, :, cached] = vn[0].cpu().numpy()
            threads = os.cpu_count() or 1
            data = (q[:, :, None].cpu().numpy(), kc, vc)
            steps, secs = cpu_time(args.cpu_budget, 1000, threads, data)
            # the strict single-thread transcription: one full step
            s1, secs1 = cpu_time(0.0, 1, 1, data)
            line["cpu_baseline"] = {
                "value": steps / secs, "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{steps} full config-4 steps on the host (faithful F16 chain of "
                          f"the reference's kernels), time-boxed to {args.cpu_budget:.0f} s",
                "single_thread": {"value": s1 / secs1, "unit": "tok/s", "cores": 1,
                                  "sample": "1 full config-4 step, one thread"}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------
# Decoder workloads (3 and 5): decode tok/s of the whole model
# ------------------------------------------------------------------------------------

DECODER_WORKLOADS = {
    # name: (preset, sequences, prompt/context, decode tokens, description)
    "cfg2": ("smollm2-135m", 1, 32, 256,
             "cfg2 SmolLM2-135M decoder, batch 1, 32-token prompt then 256 greedy tokens"),
    "cfg3": ("smollm2-360m", 64, None, 128,
             "cfg3 SmolLM2-360M batched paged decode, 64 sequences with contexts U[256,2048], "
             "128 tokens each"),
    "cfg5": ("tinystories-110m", 16, 512, 64,
             "cfg5 TinyStories-110M, 16 prompts x 512 tokens then 64 decode tokens each"),
}


def decoder_cpu_time(cfg, weights, lens, budget_s: float, threads: int):
    """One decode token of the whole model on the host cores, per sequence, as the
    reference's CPU-side chain would compute it: numpy float32 products over the F16 weights
    with the reference's F16 storage points (normed rows, projections, residual sums, the
    SwiGLU product, logits), RoPE and the faithful attention chain of the C oracle over the
    sequence's cache (length from `lens`, random N(0,1) contents; `threads` host threads
    for the attention), greedy argmax.  Sequences are taken in turn until the budget is
    spent; returns (tokens, seconds, sample description)."""
    import numpy as np

    from oracle import oracle as orc
    orc.build()
    f32, f16 = np.float32, np.float16
    hkv, d = cfg.num_kv_heads, cfg.head_dim
    # the weights as host float32 (the conversion is not timed)
    emb = weights.embedding.float().cpu().numpy()
    layers = [{k: v.float().cpu().numpy() for k, v in L.items()} for L in weights.layers]
    fnorm = weights.final_norm.float().cpu().numpy()
    head = weights.lm_head.float().cpu().numpy()
    rng = np.random.default_rng(77)
    cos, sin = orc.rope_tables(d, max(lens) + 2, cfg.rope_theta)
    sample_lens = lens[:8]  # up to eight sequences, an equal share of the budget each
    tokens, t_total = 0, 0.0
    for si, L in enumerate(sample_lens):
        kc = [rng.standard_normal((1, hkv, L + 1, d), dtype=f32).astype(f16)
              for _ in range(cfg.num_layers)]
        vc = [rng.standard_normal((1, hkv, L + 1, d), dtype=f32).astype(f16)
              for _ in range(cfg.num_layers)]
        share_end = budget_s * (si + 1) / len(sample_lens)
        while True:
            t0 = time.perf_counter()
            decoder_cpu_token(cfg, emb, layers, fnorm, head, kc, vc, L, cos, sin, rng, threads)
            t_total += time.perf_counter() - t0
            tokens += 1
            if t_total >= share_end:
                break
    sample = (f"{tokens} decode tokens over {len(sample_lens)} sequence(s) of the workload's "
              f"context lengths, one token at a time, all {cfg.num_layers} layers, attention "
              f"on {threads} threads, time-boxed to {budget_s:.0f} s")
    return tokens, t_total, sample


def decoder_cpu_token(cfg, emb, layers, fnorm, head, kc, vc, L, cos, sin, rng, threads):
    """The body of decoder_cpu_time: one token of one sequence at position L."""
    import numpy as np

    from oracle import oracle as orc
    f32, f16 = np.float32, np.float16
    hq, hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    inter, eps = cfg.intermediate_size, cfg.rms_norm_eps

    def half(x):
        return x.astype(f16).astype(f32)

    def norm(x, w):
        return half(x / np.sqrt((x * x).mean() + eps) * w)

    x = half(emb[int(rng.integers(cfg.vocab_size))])
    for li, W in enumerate(layers):
        qkv = half(norm(x, W["attn_norm"]) @ W["wqkv"])
        q = qkv[:hq * d].reshape(1, hq, 1, d).astype(f16)
        kn = qkv[hq * d:(hq + hkv) * d].reshape(1, hkv, 1, d).astype(f16)
        vn = qkv[(hq + hkv) * d:].reshape(1, hkv, 1, d).astype(f16)
        q, kn = orc.rope(q, cos, sin, L), orc.rope(kn, cos, sin, L)
        kc[li][:, :, L:L + 1] = kn
        vc[li][:, :, L:L + 1] = vn
        att = orc.attention_core(q, kc[li], vc[li], L + 1, L, threads=threads)
        x = half(x + half(att.astype(f32).reshape(-1) @ W["wo"]))
        gu = half(norm(x, W["mlp_norm"]) @ W["wgu"])
        g, u = gu[:inter], gu[inter:]
        act = half(g / (1.0 + np.exp(-g)) * u)
        x = half(x + half(act @ W["wd"]))
    logits = half(norm(x, fnorm) @ head)
    return int(np.argmax(logits))


def run_decoder(args) -> None:
    import torch
    import torch.distributed as dist

    from rustllm_b200.decoder import PRESETS, Decoder, DecoderWeights, GraphedDecoder
    from rustllm_b200.distributed import shard_sequences

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    preset, total_seqs, prompt, steps, desc = DECODER_WORKLOADS[args.workload]
    steps = min(steps, args.steps)  # the config's token count unless fewer are asked for
    prefill_ms = None
    cfg = PRESETS[preset]
    gen = torch.Generator().manual_seed(1234)
    if args.workload == "cfg3":
        ctx = torch.randint(256, 2049, (total_seqs,), generator=gen).tolist()
        # batch sharding, no collective; --shard-of M runs rank 0's share of an M-way shard
        # on this one GPU (a rank's work alone, for exploring the per-rank step)
        ways = args.shard_of if (args.shard_of and world == 1) else world
        mine = shard_sequences(total_seqs, rank, ways)
        scaling = "strong"
    else:
        ctx = [prompt] * total_seqs
        mine = list(range(total_seqs))  # replicas: every GPU runs its own copy
        scaling = "weak"
    B = len(mine)
    need = max(ctx[s] for s in mine) + args.warmup + steps + 2
    w = DecoderWeights(cfg, device=dev, seed=7)
    dec = Decoder(cfg, w, B, device=dev, shuffle_seed=11 + rank, max_seq_len=need)
    if args.workload == "cfg3":
        # synthetic contexts: N(0,1) K/V written straight into every layer's paged cache
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        for i, s in enumerate(mine):
            for layer in range(cfg.num_layers):
                k = torch.randn((cfg.num_kv_heads, ctx[s], cfg.head_dim), generator=g,
                                device=dev).half()
                v = torch.randn((cfg.num_kv_heads, ctx[s], cfg.head_dim), generator=g,
                                device=dev).half()
                dec.cache.append(layer, i, k, v)
            dec.cache.advance(ctx[s], i)
        first = torch.randint(0, cfg.vocab_size, (B,), generator=gen).to(dev, torch.int32)
    else:
        prompts = torch.randint(0, cfg.vocab_size, (B, prompt), generator=gen).to(dev)
        first = dec.prefill(prompts)  # warm-up (library heuristics, allocations)
        torch.cuda.synchronize()
        dec.cache.reset()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        first = dec.prefill(prompts)  # whole-prompt prefill of every sequence, all layers
        p1.record()
        torch.cuda.synchronize()
        prefill_ms = p0.elapsed_time(p1)
    dec.ids.copy_(first)
    runner = GraphedDecoder(dec, args.warmup + steps)
    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    kv_before = sum(dec.cache.lens())
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region(True)
    wall0 = time.time()
    e0.record()
    for _ in range(steps):
        runner.step()
    e1.record()
    torch.cuda.synchronize()
    profile_region(False)
    wall1 = time.time()
    ms = e0.elapsed_time(e1)
    clocks = sampler.stop(wall0, wall1) if sampler else None
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    tokens = (total_seqs if args.workload == "cfg3" and not args.shard_of
              else B * world) * steps
    tok_s = tokens / (ms * 1e-3)
    # step bytes on this rank: every weight once + the K/V each sequence reads
    e = 2
    mean_len = kv_before / max(B, 1) + steps / 2
    kv_bytes = B * cfg.num_layers * 2 * cfg.num_kv_heads * cfg.head_dim * e * mean_len
    step_bytes = cfg.weight_params() * e + kv_bytes
    achieved = step_bytes / (ms * 1e-3 / steps) / 1e9
    if rank == 0:
        peaks = load_peaks()
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (random-init weights N(0,0.02), random token ids, seeded)",
            "config": {"workload": desc + (f" (rank 0's share of a {args.shard_of}-way "
                                           f"shard: {B} sequences)" if args.shard_of else ""),
                       "preset": preset, "sequences": total_seqs,
                       "parallelism": (f"batch-shard{world}" if args.workload == "cfg3"
                                       else f"replicas{world}") if world > 1 else "1gpu",
                       "graph": "one CUDA graph per decode step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "peak_source": peaks["source"], "traffic": None,
                         "scope": "whole decode step on rank 0: weights + K/V read per step",
                         "floor_ms_per_step": step_bytes / (peaks["hbm_gbs"] * 1e9) * 1e3,
                         "bytes_per_step": step_bytes},
            "clocks": clocks,
            # this package's kernels a step launches (cuBLAS GEMMs not counted): embedding;
            # a layer's projections + attention (fused: 4 + 1; else norm x2, SwiGLU,
            # attention); the head (fused: norm + head + argmax in one; else final norm,
            # argmax); the length advance outside the graph
            "gpu_launches": steps * (1 + cfg.num_layers * (5 if dec.fused else 4) +
                                     (1 if dec.head else 2) + 1),
        }
        if world == 1 and not args.no_cpu:
            threads = os.cpu_count() or 1
            lens = [ctx[s] + steps // 2 for s in mine]
            n_tok, secs, sample = decoder_cpu_time(cfg, w, lens, args.cpu_budget, threads)
            line["cpu_baseline"] = {"value": n_tok / secs, "unit": "tok/s", "cores": threads,
                                    "kind": "port", "sample": sample}
        if prefill_ms is not None:
            line["prefill"] = {"ms": prefill_ms, "tok_s": B * prompt / (prefill_ms * 1e-3),
                               "scope": f"{B} prompts x {prompt} tokens, whole model (GEMMs "
                                        f"+ fused prefill attention), one pass per layer"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------
# Config 3's attention op alone: batched paged decode over mixed lengths
# ------------------------------------------------------------------------------------

def run_cfg3_attention(args) -> None:
    import torch

    import rustllm_b200 as rb

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, hq, hkv, d, layers = 64, 15, 5, 64, 4
    gen = torch.Generator().manual_seed(1234)
    lens = torch.randint(256, 2049, (B,), generator=gen).tolist()  # config 3's contexts
    cache = rb.PagedKvCache(layers, B, max(lens) + 2, hkv, d, dtype=torch.float16,
                            block_size=16, shuffle_seed=11, device=dev)
    g = torch.Generator(device=dev).manual_seed(100)
    for layer in range(layers):
        for s, n in enumerate(lens):
            cache.append(layer, s, torch.randn((hkv, n, d), generator=g, device=dev).half(),
                         torch.randn((hkv, n, d), generator=g, device=dev).half())
    for s, n in enumerate(lens):
        cache.advance(n, s)
    q = torch.randn((B, hq, d), generator=g, device=dev).half()
    kn = torch.randn((B, hkv, d), generator=g, device=dev).half()
    vn = torch.randn((B, hkv, d), generator=g, device=dev).half()
    out = torch.empty((B, hq, d), dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev)
    # the C entry point with its arguments prepared once, consecutive launches overlapped
    # (programmatic dependent launch, as the decoder's step and config 4 use it): nothing
    # between two steps writes the cache, lengths stay put, every step is the same op
    import ctypes as C

    from rustllm_b200 import _lib
    fn = _lib.load().tmllm_cache_decode
    ov = 0 if args.no_overlap else _lib.DECODE_OVERLAP
    opts = [_lib.DecodeOpts(flags=ov, num_splits=args.splits),
            _lib.DecodeOpts(num_splits=args.splits)]
    argv = [[(cache.handle, li, q.data_ptr(), kn.data_ptr(), vn.data_ptr(), out.data_ptr(), None,
              hq, C.byref(o), stream.cuda_stream) for li in range(layers)] for o in opts]

    def launch(i, plain=False):
        rc = fn(*argv[1 if plain else 0][i % layers])
        if rc:
            _lib.check(rc)

    for i in range(max(args.warmup, 3)):
        launch(i)
    torch.cuda.synchronize()
    n = max(args.steps, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region(True)
    torch.cuda._sleep(2_000_000)  # the launches below queue up behind this
    e0.record(stream)
    for i in range(n):
        launch(i)
    e1.record(stream)
    torch.cuda.synchronize()
    profile_region(False)
    k_ms = e0.elapsed_time(e1) / n
    # each launch alone (CUDA events around it, no overlap), for comparison
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(min(n, 500))]
    torch.cuda._sleep(2_000_000)
    for i, (a, b) in enumerate(ev):
        a.record(stream)
        launch(i, plain=True)
        b.record(stream)
    torch.cuda.synchronize()
    k_ms_alone = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    L = [x + 1 for x in lens]
    launch_bytes = sum(2 * hkv * x * d * 2 for x in L) + B * (2 * hq * d + 4 * hkv * d) * 2
    peaks = load_peaks()
    achieved = launch_bytes / (k_ms * 1e-3) / 1e9
    line = {
        "metric": "batched decode attention tok/s (fused append + paged GQA attention)",
        "value": B / (k_ms * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": n,
        "warmup": max(args.warmup, 3), "ms_per_step": k_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) K/V, q; random block permutation)",
        "config": {"workload": "cfg3 attention op: 64 sequences, contexts U[256,2048] (seeded), "
                               "Hq 15 / Hkv 5 / D 64, 16-token pages, one appended token each",
                   "l2": f"{layers} layers cycled: {layers * launch_bytes / 1e6:.0f} MB of K/V "
                         f"per cycle vs 126 MB L2"},
        "gpu_launches": n,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": peaks["source"], "traffic": None,
                     "kernel": "decode_mma_kernel<64,2,PT>", "kernel_ms": k_ms,
                     "kernel_ms_single_launch_events": k_ms_alone,
                     "bytes_per_launch": launch_bytes},
        "overlapped_launches": not args.no_overlap,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# Config 1: the reference's own CPU-runnable case, a latency figure (no roofline claim)
# ------------------------------------------------------------------------------------

def run_cfg1(args) -> None:
    import numpy as np
    import torch

    import rustllm_b200 as rb

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    hq, hkv, d, cached, theta = 9, 3, 64, 128, 100000.0
    rng = np.random.default_rng(1234)
    k = rng.standard_normal((hkv, cached, d)).astype(np.float32)
    v = rng.standard_normal((hkv, cached, d)).astype(np.float32)
    q = rng.standard_normal((1, hq, d)).astype(np.float32)
    kn = rng.standard_normal((1, hkv, d)).astype(np.float32)
    vn = rng.standard_normal((1, hkv, d)).astype(np.float32)
    # the reference's layout: one [1, Hkv, max, D] buffer (block size = capacity)
    cache = rb.PagedKvCache(1, 1, cached + 1, hkv, d, dtype=torch.float32,
                            block_size=cached + 1, device=dev)
    cache.append(0, 0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
    cache.advance(cached, 0)
    cache.reserve(0, 1)
    rope = rb.rope_tables(d, cached + 2, theta, device=dev)
    gq, gkn, gvn = (torch.from_numpy(x).to(dev) for x in (q, kn, vn))
    out = torch.empty((1, hq, d), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    n = max(args.steps, 1)
    for _ in range(max(args.warmup, 3)):
        cache.decode(0, gq, gkn, gvn, out=out, rope=rope, scale=0.125)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n)]
    for a, b in ev:  # lengths are not advanced: every step appends at position 128
        a.record(stream)
        cache.decode(0, gq, gkn, gvn, out=out, rope=rope, scale=0.125)
        b.record(stream)
    torch.cuda.synchronize()
    lat = sorted(a.elapsed_time(b) * 1e3 for a, b in ev)
    med = lat[len(lat) // 2]
    # end to end: pinned host q, k, v in, out back to the host, every step
    hq_, hk_, hv_ = (torch.from_numpy(x).pin_memory() for x in (q, kn, vn))
    hout = torch.empty((1, hq, d), dtype=torch.float32).pin_memory()
    e_lat = []
    for i in range(min(n, 1000) + 3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        gq.copy_(hq_, non_blocking=True)
        gkn.copy_(hk_, non_blocking=True)
        gvn.copy_(hv_, non_blocking=True)
        cache.decode(0, gq, gkn, gvn, out=out, rope=rope, scale=0.125)
        hout.copy_(out, non_blocking=True)
        b.record(stream)
        b.synchronize()
        if i >= 3:
            e_lat.append(a.elapsed_time(b) * 1e3)
    e_lat.sort()
    line = {
        "metric": "config 1 decode step latency (fused append + attention, F32)",
        "value": med, "unit": "us", "n_gpus": 1, "steps": n, "warmup": max(args.warmup, 3),
        "ms_per_step": med / 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) cache of 128 positions, q, k, v)",
        "config": {"workload": "cfg1 TinyLlama-like layer: Hq=9, Hkv=3, D=64, 128 cached + 1 "
                               "appended, RoPE theta 1e5, scale 1/8, contiguous cache",
                   "statistic": "median over steps of per-launch CUDA-event time"},
        "p90_us": lat[int(len(lat) * 0.9)], "gpu_launches": n,
        "e2e": {"value": e_lat[len(e_lat) // 2], "unit": "us",
                "h2d_bytes_per_step": (q.size + kn.size + vn.size) * 4,
                "d2h_bytes_per_step": hq * d * 4},
        "roofline": None,
    }
    if not args.no_cpu:
        from oracle import oracle as orc
        orc.build()
        cos, sin = orc.rope_tables(d, cached + 2, theta)
        kc = np.zeros((1, hkv, cached + 1, d), np.float32)
        vc = np.zeros_like(kc)
        kc[0, :, :cached], vc[0, :, :cached] = k, v
        cnt, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.cpu_budget, 5.0) and cnt < 20000:
            orc.decode_step(q[:, :, None], kn[:, :, None], vn[:, :, None], kc, vc, cached,
                            cos, sin, threads=1)
            cnt += 1
        secs = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 1e6 * secs / cnt, "unit": "us", "cores": 1,
                                "kind": "port",
                                "sample": f"{cnt} config-1 steps of the single-thread oracle "
                                          f"(RoPE, append, faithful F32 chain)"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# Prefill workload (BASELINE config 5's prompt phase): the tensor-core prefill attention
# ------------------------------------------------------------------------------------

P_SEQS, P_LEN, P_HEADS, P_D, P_LAYERS = 16, 512, 12, 64, 12


def prefill_flops(seqs: int = P_SEQS, n: int = P_LEN, heads: int = P_HEADS, d: int = P_D,
                  cached: int = 0) -> float:
    """Algorithmic FLOPs of one causal prefill launch: query row i attends cached + i + 1
    keys; each (query, key) pair costs 2*D for Q.K and 2*D for P.V."""
    pairs = n * cached + n * (n + 1) // 2
    return 4.0 * d * pairs * heads * seqs


def run_prefill(args) -> None:
    import torch
    import torch.distributed as dist

    import rustllm_b200 as rb

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    B, S, H, d, NL = P_SEQS, P_LEN, P_HEADS, P_D, P_LAYERS
    T = B * S
    cache = rb.PagedKvCache(NL, B, S, H, d, dtype=torch.float16, block_size=16,
                            shuffle_seed=31 + rank, device=dev)
    for s in range(B):
        cache.reserve(s, S)
    rope = rb.rope_tables(d, S + 1, 10000.0, device=dev)
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    # per-layer inputs (3 x 12.6 MB each, 453 MB over the 12 layers: larger than L2)
    qs = [torch.randn((T, H, d), generator=g, device=dev).half() for _ in range(NL)]
    ks = [torch.randn((T, H, d), generator=g, device=dev).half() for _ in range(NL)]
    vs = [torch.randn((T, H, d), generator=g, device=dev).half() for _ in range(NL)]
    outs = [torch.empty((T, H, d), dtype=torch.float16, device=dev) for _ in range(NL)]
    views = [cache.view(li) for li in range(NL)]
    stream = torch.cuda.current_stream(dev)
    # the C entry point with arguments prepared once (the Python wrapper's checks would
    # otherwise keep the GPU waiting on the host between these ~10 us launches)
    import ctypes as C

    from rustllm_b200 import _lib
    lib = _lib.load()
    opts = _lib.DecodeOpts(rope_cos=rope[0].data_ptr(), rope_sin=rope[1].data_ptr(),
                           rope_len=rope[0].shape[0], q_seq_stride=H * d, kv_seq_stride=H * d)
    sp = stream.cuda_stream
    calls = [(C.byref(views[li]), qs[li].data_ptr(), ks[li].data_ptr(), vs[li].data_ptr(),
              outs[li].data_ptr()) for li in range(NL)]
    fn = lib.tmllm_gqa_prefill

    # RoPE off: the call is the attention kernel alone (with RoPE and an F16 output the
    # query rotation runs in the append kernel first), used to time that kernel by itself
    opts_plain = _lib.DecodeOpts(q_seq_stride=H * d, kv_seq_stride=H * d)

    def launch(li, append=True, rope_on=True):
        kv, q, k, v, o = calls[li]
        rc = fn(kv, q, k if append else None, v if append else None, None, S, 0, 0, o, H,
                C.byref(opts if rope_on else opts_plain), sp)
        if rc:
            _lib.check(rc)

    def step(append=True):  # lengths stay 0: every step rewrites the same positions
        for li in range(NL):
            launch(li, append)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if rb.prefill_status() != 0:
        raise SystemExit("prefill kernel reported an expired wait")
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
    # (1) the hot path as a step: append + attention for all 12 layers
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    profile_region(True)
    wall0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    profile_region(False)
    # (2) the attention kernel alone, per launch (attend-only calls without RoPE: the same
    # kernel and work, and no other launch inside the events)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps * NL)]
    i = 0
    for _ in range(args.steps):
        for li in range(NL):
            kev[i][0].record(stream)
            launch(li, append=False, rope_on=False)
            kev[i][1].record(stream)
            i += 1
    torch.cuda.synchronize()
    wall1 = time.time()
    clocks = sampler.stop(wall0, wall1) if sampler else None
    ms = e0.elapsed_time(e1)
    k_ms = sum(a.elapsed_time(b) for a, b in kev) / len(kev)
    t = torch.tensor([ms, k_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, k_ms = float(t[0]), float(t[1])
    ms_step = ms / args.steps
    step_flops = prefill_flops() * NL
    value = step_flops * world / (ms_step * 1e-3) / 1e12
    achieved = prefill_flops() / (k_ms * 1e-3) / 1e12

    # e2e: per-layer q/k/v from pinned host memory, outputs back to the host
    hq = [x.cpu().pin_memory() for x in qs[:2]]
    hk = [x.cpu().pin_memory() for x in ks[:2]]
    hv = [x.cpu().pin_memory() for x in vs[:2]]
    ho = torch.empty((T, H, d), dtype=torch.float16).pin_memory()
    dq, dk, dv = torch.empty_like(qs[0]), torch.empty_like(ks[0]), torch.empty_like(vs[0])

    def e2e_step():
        for li in range(NL):
            dq.copy_(hq[li % 2], non_blocking=True)
            dk.copy_(hk[li % 2], non_blocking=True)
            dv.copy_(hv[li % 2], non_blocking=True)
            rb.gqa_prefill(views[li], dq, dk, dv, rows_per_seq=S, out=outs[li], rope=rope)
            ho.copy_(outs[li], non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e_steps = max(1, min(args.steps, 20))
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(e_steps):
        e2e_step()
    f1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = step_flops * world * e_steps / (float(te[0]) * 1e-3) / 1e12
    if rb.prefill_status() != 0:
        raise SystemExit("prefill kernel reported an expired wait")

    if rank == 0:
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        peak, src = 1590.0, "fallback"
        if os.path.exists(peaks_path):
            with open(peaks_path) as f:
                peak, src = float(json.load(f)["bf16_tflops"]), "measured (burst)"
        line = {
            "metric": "prefill attention TFLOP/s (fused append + causal tcgen05 attention)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) q, k, v per layer)",
            "config": {"workload": "cfg5 prompt phase: TinyStories-110M attention shape, 16 "
                                   "prompts x 512 tokens, 12 layers (MHA 12 heads, D=64), "
                                   "16-token pages",
                       "tokens_per_step": T, "layers": NL,
                       "parallelism": f"replicas{world}" if world > 1 else "1gpu",
                       "l2": "per-layer inputs, 453 MB per step: larger than L2"},
            "prefill_tok_s": T * world / (ms_step * 1e-3),
            "gpu_launches": args.steps * NL * 2,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": src,
                         "traffic": None, "kernel": "prefill_tc_kernel<64>",
                         "kernel_ms": k_ms, "flops_per_launch": prefill_flops()},
            "e2e": {"value": e2e, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": NL * 3 * T * H * d * 2,
                    "d2h_bytes_per_step": NL * T * H * d * 2},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu:
            from oracle import oracle as orc
            orc.build()
            threads = os.cpu_count() or 1
            qn = qs[0][:S].float().cpu().numpy().transpose(1, 0, 2)[None].astype("float16")
            kn = ks[0][:S].float().cpu().numpy().transpose(1, 0, 2)[None].astype("float16")
            vn = vs[0][:S].float().cpu().numpy().transpose(1, 0, 2)[None].astype("float16")
            import numpy as np
            qn, kn, vn = (np.ascontiguousarray(x) for x in (qn, kn, vn))
            n_done, c0 = 0, time.perf_counter()
            while time.perf_counter() - c0 < args.cpu_budget:
                orc.attention_core(qn, kn, vn, S, 0, threads=threads)
                n_done += 1
            secs = time.perf_counter() - c0
            cpu_tflops = prefill_flops(seqs=1) * n_done / secs / 1e12
            line["cpu_baseline"] = {
                "value": cpu_tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{n_done} one-sequence one-layer prefills (12 heads x 512 rows, the "
                          f"reference's faithful F16 op chain), time-boxed to "
                          f"{args.cpu_budget:.0f} s"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------------
# Kernel survey: every kernel of the library, timed alone on a moderate case
# ------------------------------------------------------------------------------------

def run_kernel_survey(args) -> None:
    """Launches each kernel of libtmllm_b200.so on a case sized so its algorithmic traffic
    exceeds L2 where the kernel streams HBM, times the launches with CUDA events on the
    launching stream (queued behind a GPU sleep, so the launches run back to back without
    host gaps) and reports algorithmic GB/s (TFLOP/s for the tensor-core prefill and the
    batched matmul) against the measured peaks.  Under ncu the same command gives each
    kernel's DRAM counters."""
    import torch

    import rustllm_b200 as rb
    from rustllm_b200 import _lib
    from rustllm_b200.decoder import head_workspace, linear, lm_head

    world, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    peaks = load_peaks()
    tc_peak = 1590.0
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            tc_peak = float(json.load(f)["bf16_tflops"])
    g = torch.Generator(device=dev).manual_seed(7)
    H = torch.float16

    def rnd(*shape, dtype=H):
        return torch.randn(shape, generator=g, device=dev).to(dtype)

    results = []

    def timed(name, kernel, fn, work, unit="GB/s", reps=None):
        reps = reps or args.steps
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        torch.cuda._sleep(3_000_000)  # the launches below queue up behind this
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(reps)]
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        us = sum(a.elapsed_time(b) for a, b in ev) / reps * 1e3
        if unit == "GB/s":
            ach = work / (us * 1e-6) / 1e9
            frac = ach / peaks["hbm_gbs"]
        else:
            ach = work / (us * 1e-6) / 1e12
            frac = ach / tc_peak
        results.append({"case": name, "kernel": kernel, "us": round(us, 3), "work": work,
                        "achieved": round(ach, 1), "unit": unit, "frac": round(frac, 4)})
        print(f"# {name:42s} {kernel:36s} {us:9.2f} us {ach:9.1f} {unit} {frac:6.3f}",
              file=sys.stderr, flush=True)

    # ---- paged cache runtime (cache.cu)
    hkv, d, n = 8, 128, 65536
    cache = rb.PagedKvCache(1, 1, n + 64, hkv, d, dtype=H, block_size=16, shuffle_seed=3,
                            device=dev)
    k, v = rnd(hkv, n, d), rnd(hkv, n, d)
    cache.append(0, 0, k, v)  # reserves the blocks once
    nb = 4 * hkv * n * d * 2
    timed("append 65536 positions, Hkv 8, D 128", "paged_rows_kernel",
          lambda: cache.append(0, 0, k, v), nb)
    cache.advance(n, 0)
    ko, vo = torch.empty_like(k), torch.empty_like(v)
    timed("gather 65536 positions, Hkv 8, D 128", "paged_rows_kernel",
          lambda: _lib.call("tmllm_cache_gather", cache.handle, 0, 0, ko.data_ptr(),
                            vo.data_ptr(), sp), nb)
    # the table / length kernels move a few bytes each: launch latency, no roofline claim
    timed("reset + reserve 16 + advance 16", "fill_i32 x2 + set_entries + add_lens",
          lambda: (cache.reset(0), cache.reserve(0, 16), cache.advance(16, 0)), 16, reps=20)
    del cache, k, v, ko, vo
    torch.cuda.empty_cache()

    # ---- fused decode (decode.cu)
    def decode_case(name, kernel, dtype, hq, hkv, d, lens, variant):
        c = rb.PagedKvCache(1, len(lens), max(lens) + 2, hkv, d, dtype=dtype, block_size=16,
                            shuffle_seed=5, device=dev)
        for s_, L in enumerate(lens):
            c.append(0, s_, rnd(hkv, L, d, dtype=dtype), rnd(hkv, L, d, dtype=dtype))
            c.advance(L, s_)
        B = len(lens)
        q = rnd(B, hq, d, dtype=dtype)
        kn, vn = rnd(B, hkv, d, dtype=dtype), rnd(B, hkv, d, dtype=dtype)
        out = torch.empty((B, hq, d), dtype=dtype, device=dev)
        e = 2 if dtype == H else 4
        work = sum(2 * hkv * (L + 1) * d * e for L in lens) + B * (2 * hq + 4 * hkv) * d * e
        timed(name, kernel, lambda: c.decode(0, q, kn, vn, out=out, variant=variant), work)

    lens3 = torch.randint(256, 2049, (64,), generator=torch.Generator().manual_seed(1234)).tolist()
    decode_case("decode F16 32768 pos, Hq 32/Hkv 8, D 128", "decode_mma_kernel<128,3>",
                H, 32, 8, 128, [32768], 0)
    decode_case("decode F16 cfg3 batch, Hq 15/Hkv 5, D 64", "decode_mma_kernel<64,3,PT>",
                H, 15, 5, 64, lens3, 0)
    decode_case("decode F16 16 seqs, Hq 32/Hkv 2, D 64", "decode_mma_kernel<64,3>",
                H, 32, 2, 64, lens3[:16], 0)
    decode_case("decode F32 32768 pos, Hq 32/Hkv 8, D 128", "decode_split_kernel<f32,128>",
                torch.float32, 32, 8, 128, [32768], 1)
    decode_case("decode F16 CUDA cores, 32768 pos, D 128", "decode_split_kernel<f16,128>",
                H, 32, 8, 128, [32768], 1)
    decode_case("decode F16 D 96 (any even head_dim)", "decode_generic_kernel",
                H, 8, 2, 96, [8192], 0)
    torch.cuda.empty_cache()
    parts, rows = 8, 32768
    po, pl = rnd(parts, rows, 128, dtype=torch.float32), rnd(parts, rows, dtype=torch.float32)
    mo = torch.empty((rows, 128), dtype=H, device=dev)
    timed("merge 8 parts x 32768 rows x 128", "merge_lse_kernel",
          lambda: rb.merge_lse(po, pl, out=mo), parts * rows * (128 + 1) * 4 + rows * 128 * 2)
    del po, pl, mo

    # ---- prefill (prefill.cu): config 5's layer
    B, S, Hh, dd = 16, 512, 12, 64
    pc = rb.PagedKvCache(1, B, S, Hh, dd, dtype=H, block_size=16, shuffle_seed=31, device=dev)
    for s_ in range(B):
        pc.reserve(s_, S)
    rope = rb.rope_tables(dd, S + 1, 10000.0, device=dev)
    pq, pk, pv = rnd(B * S, Hh, dd), rnd(B * S, Hh, dd), rnd(B * S, Hh, dd)
    po_ = torch.empty_like(pq)
    view = pc.view(0)
    timed("prefill append + attention, cfg5 layer", "prefill_append_vec + prefill_tc<64>",
          lambda: rb.gqa_prefill(view, pq, pk, pv, rows_per_seq=S, out=po_, rope=rope),
          prefill_flops(), unit="TFLOP/s")
    timed("prefill attention alone, cfg5 layer", "prefill_tc_kernel<64>",
          lambda: rb.gqa_prefill(view, pq, None, None, rows_per_seq=S, out=po_),
          prefill_flops(), unit="TFLOP/s")
    # the append alone: its bytes (q, k, v read; k, v, rotated q written) over the
    # difference of the two launches above
    pair, alone = results[-2]["us"], results[-1]["us"]
    if pair > alone:
        ab = 6 * B * S * Hh * dd * 2
        results.append({"case": "prefill append alone (pair - attention)",
                        "kernel": "prefill_append_vec_kernel", "us": round(pair - alone, 3),
                        "work": ab, "achieved": round(ab / ((pair - alone) * 1e-6) / 1e9, 1),
                        "unit": "GB/s",
                        "frac": round(ab / ((pair - alone) * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)})
    del pc, pq, pk, pv, po_
    pc32 = rb.PagedKvCache(1, 2, 256, 4, 64, dtype=torch.float32, block_size=16, device=dev)
    for s_ in range(2):
        pc32.reserve(s_, 256)
    view32 = pc32.view(0)
    q32, k32, v32 = (rnd(512, 4, 64, dtype=torch.float32) for _ in range(3))
    o32 = torch.empty_like(q32)
    timed("prefill F32 (CUDA cores), 2 x 256 rows", "prefill_append + prefill_generic",
          lambda: rb.gqa_prefill(view32, q32, k32, v32, rows_per_seq=256, out=o32),
          prefill_flops(seqs=2, n=256, heads=4, d=64), unit="TFLOP/s")
    del pc32
    torch.cuda.empty_cache()

    # ---- decoder element-wise kernels and projections (decoder.cu)
    hid, voc, nid = 960, 49152, 65536
    table = rnd(voc, hid)
    ids = torch.randint(0, voc, (nid,), generator=torch.Generator().manual_seed(3)).to(
        dev, torch.int32)
    emb = torch.empty((nid, hid), dtype=H, device=dev)
    timed("embedding 65536 ids x 960", "embedding_kernel",
          lambda: _lib.call("tmllm_embedding", 1, table.data_ptr(), ids.data_ptr(),
                            emb.data_ptr(), nid, hid, voc, None, sp), 2 * nid * hid * 2)
    res, nw = rnd(nid, hid), (1 + 0.1 * rnd(hid, dtype=torch.float32)).to(H)
    outn, sumo = torch.empty_like(emb), torch.empty_like(emb)
    timed("add + RMSNorm 65536 x 960 (warp per row)", "add_rmsnorm_warp_kernel",
          lambda: _lib.call("tmllm_add_rmsnorm", 1, emb.data_ptr(), res.data_ptr(),
                            nw.data_ptr(), outn.data_ptr(), sumo.data_ptr(), nid, hid, 1e-5,
                            sp), 4 * nid * hid * 2)
    e32, r32 = emb[:16384].float(), res[:16384].float()
    n32, o32b, s32 = nw.float(), torch.empty_like(e32), torch.empty_like(e32)
    timed("add + RMSNorm F32 16384 x 960", "add_rmsnorm_kernel<f32>",
          lambda: _lib.call("tmllm_add_rmsnorm", 0, e32.data_ptr(), r32.data_ptr(),
                            n32.data_ptr(), o32b.data_ptr(), s32.data_ptr(), 16384, hid, 1e-5,
                            sp), 4 * 16384 * hid * 4)
    del table, emb, res, outn, sumo, e32, r32, o32b, s32
    inter, rws = 2560, 16384
    gu = rnd(rws, 2 * inter)
    act = torch.empty((rws, inter), dtype=H, device=dev)
    timed("SwiGLU 16384 x 2560", "swiglu_vec_kernel",
          lambda: _lib.call("tmllm_swiglu", 1, gu.data_ptr(), act.data_ptr(), rws, inter, sp),
          3 * rws * inter * 2)
    gu32, act32 = gu[:8192].float(), act[:8192].float()
    timed("SwiGLU F32 8192 x 2560", "swiglu_kernel<f32>",
          lambda: _lib.call("tmllm_swiglu", 0, gu32.data_ptr(), act32.data_ptr(), 8192, inter,
                            sp), 3 * 8192 * inter * 4)
    del gu, act, gu32, act32
    lg = rnd(1024, voc)
    am = torch.empty(1024, dtype=torch.int32, device=dev)
    timed("argmax 1024 x 49152", "argmax_kernel<f16>",
          lambda: _lib.call("tmllm_argmax", 1, lg.data_ptr(), am.data_ptr(), 1024, voc, sp),
          1024 * voc * 2)
    del lg
    # the decode-step head (final norm + lm_head + argmax): three weight copies in turn, so
    # the weight is read from HBM as in a decode step
    for rows, kk, nn, what in ((1, 576, 49152, "cfg2"), (16, 768, 32000, "cfg5")):
        hw = [(rnd(kk, nn) / 30).to(H) for _ in range(3)]
        hx, hnw = rnd(rows, kk), rnd(kk)
        hlg = torch.empty((rows, nn), dtype=H, device=dev)
        hid_ = torch.empty(rows, dtype=torch.int32, device=dev)
        hws = head_workspace(device=dev)
        turn = [0]

        def head_call(hw=hw, hx=hx, hnw=hnw, hlg=hlg, hid_=hid_, hws=hws, turn=turn):
            turn[0] += 1
            lm_head(hx, hw[turn[0] % 3], norm_weight=hnw, logits=hlg, ids=hid_, workspace=hws)
        timed(f"head {rows} rows, {kk}x{nn} ({what})", "head_kernel<1>", head_call,
              kk * nn * 2 + rows * (kk + nn) * 2)
        del hw
    for kk, nn, sw, what in [(hid, 1600, False, "QKV 960x1600"), (960, 960, False, "O 960x960"),
                             (hid, 2560, True, "gate/up + SwiGLU 960x5120"),
                             (2560, 960, False, "down 2560x960")]:
        w = (rnd(kk, 2 * nn if sw else nn) / 30).to(H)
        for rows, kern in ((8, "linear_kernel"), (64, "linear_kernel")):
            xin = rnd(rows, kk)
            outl = torch.empty((rows, nn), dtype=H, device=dev)
            timed(f"projection {rows} rows, {what}", kern,
                  lambda w=w, xin=xin, outl=outl, sw=sw: linear(xin, w, out=outl, swiglu=sw),
                  w.numel() * 2 + rows * (kk + nn) * 2)
    torch.cuda.empty_cache()

    # ---- op-level API kernels (ops.cu)
    cbuf, src = rnd(1, 8, 65536, 128), rnd(1, 8, 65536, 128)
    timed("kv_cache_write [1,8,65536,128]", "gather_rows_kernel",
          lambda: rb.kv_cache_write(cbuf, src, 0), 2 * src.numel() * 2)
    left, right = rnd(1, 8, 32768, 128), rnd(1, 8, 32768, 128)
    timed("concat_sequence 2 x [1,8,32768,128]", "gather_rows_kernel",
          lambda: rb.concat_sequence(left, right), 4 * left.numel() * 2)
    kvr = rnd(1, 8, 16384, 128)
    timed("repeat_kv [1,8,16384,128] x 4", "gather_rows_kernel",
          lambda: rb.repeat_kv(kvr, 4), 5 * kvr.numel() * 2)
    del cbuf, src, left, right
    qo, ko_ = rnd(1, 32, 1, 128), rnd(1, 8, 32768, 128)
    timed("gqa_qk Hq 32 / Hkv 8, 32768 keys", "gqa_qk_kernel<f16>",
          lambda: rb.gqa_qk_matmul(qo, ko_), ko_.numel() * 2 + 32 * 32768 * 2)
    sc = rnd(1, 32, 1, 32768)
    timed("gqa_pv Hq 32 / Hkv 8, 32768 keys", "gqa_pv_kernel<f16>",
          lambda: rb.gqa_pv_matmul(sc, ko_), ko_.numel() * 2 + sc.numel() * 2)
    big = rnd(32, 64, 32768)
    timed("attention_scale_mask 32 x 64 x 32768", "scale_mask_kernel<f16>",
          lambda: rb.attention_scale_mask(big, 0.125, 32768 - 64), 2 * big.numel() * 2)
    timed("softmax_last_dim 2048 rows x 32768", "softmax_kernel<f16>",
          lambda: rb.softmax_last_dim(big), 2 * big.numel() * 2)
    del big, sc, ko_
    ba, bb = rnd(64, 128, 128), rnd(64, 128, 128)
    timed("batched_matmul 64 x 128^3", "bmm_kernel<f16>",
          lambda: rb.batched_matmul(ba, bb), 2 * 64 * 128 ** 3, unit="TFLOP/s")
    cos, sin = rb.rope_tables(128, 4096, 10000.0, device=dev)
    xr = rnd(32, 4096, 128)
    timed("rope [32,4096,128]", "rope_kernel<f16>",
          lambda: rb.rope(xr, cos, sin, 0), 2 * xr.numel() * 2)
    torch.cuda.synchronize()
    fr = [r["frac"] for r in results if r["unit"] == "GB/s" and r["work"] > 1e8]
    line = {
        "metric": "kernel survey: achieved fraction of the measured peak, per kernel",
        "value": statistics.median(fr), "unit": "median fraction (HBM-streaming cases)",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16/f32",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "every kernel of libtmllm_b200.so on a moderate case",
                   "l2": "streaming cases move 100-500 MB per launch (more than L2)"},
        "gpu_launches": args.steps * len(results),
        "peaks": {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": tc_peak},
        "kernels": results,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--ref-budget", type=float, default=60.0)
    ap.add_argument("--workload",
                    choices=["cfg4", "cfg1", "cfg2", "cfg3", "cfg3a", "cfg5", "cfg5p",
                             "kernels"],
                    default="cfg4",
                    help="cfg4 (default): the fused attention op; cfg2/3/5: whole-model "
                         "decode; cfg3a: config 3's attention op; cfg5p: config 5's prefill "
                         "attention; cfg1: latency")
    ap.add_argument("--variant", type=int, default=0,
                    help="decode kernel: 0 auto (tensor-core for F16), 1 CUDA-core, 2 tensor-core")
    ap.add_argument("--splits", type=int, default=0, help="split count (0 = automatic)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: exchange inside the decode kernel (p2p) or NCCL all-gather")
    ap.add_argument("--cached", type=int, default=CACHED,
                    help="cached positions (smaller values only for profiling captures)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu DRAM bytes per launch of the decode kernel, if measured anew")
    ap.add_argument("--settle", type=int, default=SETTLE_STEPS,
                    help="untimed steps after the warm-up, before the timed region")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="cfg3 on one GPU: run only rank 0's share of this many batch shards")
    ap.add_argument("--no-overlap", action="store_true",
                    help="config 4 on one GPU: launch consecutive steps without "
                         "programmatic dependent launch")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg5p":
        run_prefill(args)
    elif args.workload == "cfg1":
        run_cfg1(args)
    elif args.workload == "cfg3a":
        run_cfg3_attention(args)
    elif args.workload == "kernels":
        run_kernel_survey(args)
    elif args.workload != "cfg4":
        run_decoder(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
