"""Benchmark of the paged decode hot path (BASELINE config 2 at N=1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (per GPU, weak scaling): BASELINE.json configs[1] — paged fp16
decode, batch 32, 32 heads x 128, 4096 cached tokens per sequence in 16-token
pages with seeded random-permuted block tables, one query token per
sequence, Q/K/V ~ N(0,1) fp16, retain_ratio 1.0, synthetic data.  A step is
one dynamic_sparse_attention over the whole batch; the pool (2.1 GB of K/V)
is larger than L2, so every step streams it from HBM.

Metric: algorithmic HBM GB/s of the step (K+V pages + q/out + tables),
with decode tokens/s beside it.  `e2e` is the same metric through the public
API (memopt_C.write_cache of each new token + dynamic_sparse_attention) with
pinned host buffers copied in and the output copied back inside the timed
region.  `--impl reference` times the reference's CPU paged attention
(_sdpa_fallback, restated in oracle/sdpa_port.py) on whole configs[1] steps
with all host threads, and adds the reference's own CUDA kernel (built from
its sources into oracle/_ref) on the same inputs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "memopt-transformer-runtime_b200"))

B, H, D, BS, CTX = 32, 32, 128, 16, 4096
MB = CTX // BS
NB = B * MB  # 8192 pages
INT4_B, INT4_CTX = 16, 16384
LONG_B, LONG_CTX = 64, 131072  # BASELINE configs[4] decode (sharded over the ranks)
METRIC = "paged decode attention HBM GB/s (% of peak) & decode tokens/s at 1/2/4/8 B200"


def step_bytes(batch: int, ctx: int, fmt: str = "fp16") -> int:
    """Algorithmic bytes of one decode step (each byte the step must move once)."""
    if fmt == "fp16":
        kv = 2 * batch * ctx * H * D * 2
    else:
        kv = 2 * batch * ctx * H * (D // 2) + 2 * batch * ctx * H * (D // 64) * 2
    qo = 2 * batch * H * D * 2
    tables = batch * (ctx // BS) * 4 + batch * 4
    return kv + qo + tables


def peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


_CLOCK_SAMPLER = r"""
import sys, time, pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByPciBusId(sys.argv[1].encode()) if sys.argv[1] else \
    pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[2]))
bits = [pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
        pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap]
mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
out = open(sys.argv[3], "w") if len(sys.argv) > 3 else sys.stdout
pause = float(sys.argv[4]) if len(sys.argv) > 4 else 0.0
print("ready", mx, flush=True)
while True:
    t = time.time()
    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    print(t, pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), "".join("1" if r & b else "0" for b in bits),
          file=out, flush=True)
    if pause:
        time.sleep(pause)
"""


class Clocks:
    """SM clock and clock-event reasons sampled during the timed region.

    A separate process polls NVML back to back (a decode step lasts a
    fraction of a millisecond, so nvidia-smi's 100 ms loop sees nothing, and
    a thread of this process would contend for the interpreter lock with the
    launches being timed); entering the block waits until it samples.
    nvidia-smi is the fallback when NVML cannot be used.  Read-only."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int, log_path: str = ""):
        self.index = index
        self.log_path = log_path  # samples go to this file, one per millisecond (long blocks)
        self.samples = []  # (time, SM MHz, reason bits) of every NVML sample
        self.proc = None
        self.sm, self.mx, self.reasons = [], 0.0, set()
        self.source = "none"
        self.nvml = False
        self.t0 = self.t1 = 0.0
        self.near = []  # every NVML sample, the block's and those around it

    def __enter__(self):
        bus = ""
        try:
            import torch

            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        except Exception:  # noqa: BLE001
            pass
        try:
            extra = [self.log_path, "0.001"] if self.log_path else []
            self.proc = subprocess.Popen([sys.executable, "-c", _CLOCK_SAMPLER, bus, str(self.index)] + extra,
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline().split()
            if first and first[0] == "ready":
                self.mx = float(first[1])
                self.nvml = True
                self.source = "nvml"
                self.t0 = time.time()
                return self
            self.proc.kill()
            self.proc.wait()
        except Exception:  # noqa: BLE001
            self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"
        except Exception:  # noqa: BLE001
            self.proc = None
        return self

    def __exit__(self, *a):
        out = ""
        self.t1 = time.time()
        if self.proc is not None and self.nvml:
            time.sleep(0.02)  # let samples taken inside the block reach the pipe
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
        if self.nvml and self.log_path:
            try:
                with open(self.log_path) as f:
                    out = f.read()
                os.remove(self.log_path)
            except OSError:
                out = ""
        for line in (out or "").splitlines():
            if self.nvml:
                f = line.split()
                if len(f) != 3:
                    continue
                try:
                    ts, mhz = float(f[0]), float(f[1])
                except ValueError:
                    continue
                self.near.append(mhz)
                self.samples.append((ts, mhz, f[2]))
                if not self.t0 <= ts <= self.t1:  # taken outside the block
                    continue
                self.sm.append(mhz)
                for n, bit in zip(self.NAMES, f[2]):
                    if bit == "1":
                        self.reasons.add(n)
                continue
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                self.sm.append(float(f[1]))
                self.mx = max(self.mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(self.NAMES, f[5:9]):
                if v.lower().startswith("active"):
                    self.reasons.add(n)

    def windows_summary(self, windows) -> dict:
        """SM clock and reasons over the samples inside any of `windows`
        ((start, end) wall times): the timed loops of one group of legs."""
        sm, reasons = [], set()
        for ts, mhz, bits in self.samples:
            if any(a <= ts <= b for a, b in windows):
                sm.append(mhz)
                reasons.update(n for n, bit in zip(self.NAMES, bits) if bit == "1")
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}

    def summary(self) -> dict:
        sm = self.sm
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.mx or None,
                "reasons": sorted(self.reasons), "samples": len(sm), "source": self.source,
                "window_ms": round((self.t1 - self.t0) * 1e3, 2),
                "sm_mhz_around": statistics.median(self.near) if self.near else None}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def make_fp16_workload(torch, seed: int, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    kp = torch.randn(NB, BS, H, D, device=dev, dtype=torch.float16, generator=g)
    vp = torch.randn(NB, BS, H, D, device=dev, dtype=torch.float16, generator=g)
    gc = torch.Generator().manual_seed(seed + 1)
    bt = torch.randperm(NB, generator=gc)[: B * MB].reshape(B, MB).to(torch.int32).to(dev)
    q = torch.randn(B, 1, H, D, device=dev, dtype=torch.float16, generator=g)
    ctx = torch.full((B,), CTX, dtype=torch.int32, device=dev)
    return kp, vp, bt, q, ctx


PREFILL_B, PREFILL_QL = 4, 8192  # BASELINE configs[4] prefill


def make_prefill_workload(torch, dev, rank: int = 0, batch: int = PREFILL_B):
    """configs[4] prefill inputs: `batch` sequences x 8192 query tokens over
    their own 8192 cached tokens (seeded N(0,1) fp16, permuted tables)."""
    pql = PREFILL_QL
    mb = pql // BS
    nb = batch * mb
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    kp = torch.randn(nb, BS, H, D, device=dev, dtype=torch.float16, generator=g)
    vp = torch.randn(nb, BS, H, D, device=dev, dtype=torch.float16, generator=g)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(5 + rank))[: batch * mb].reshape(batch, mb)
    bt = bt.to(torch.int32).to(dev)
    q = torch.randn(batch, pql, H, D, device=dev, dtype=torch.float16, generator=g)
    ctx = torch.full((batch,), pql, dtype=torch.int32, device=dev)
    return kp, vp, bt, q, ctx


def time_e2e(torch, loop, steps: int, warmup: int, barrier, stream, copy_stream):
    """time_loop for the pipelined end-to-end step: the copy stream starts
    after the start event, and the end event follows the last step's
    device->host copy."""
    loop(warmup)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_stream.wait_stream(stream)
    loop(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


TIMED_WINDOWS = []  # wall-clock (start, end) of every timed loop, for the clock record


def time_loop(torch, fn, steps: int, warmup: int, barrier, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    TIMED_WINDOWS.append((w0, time.time()))
    barrier()
    return e0.elapsed_time(e1) / steps  # ms per step


def cpu_sample(torch, kp, vp, bt, q, ctx, rows_budget_s: float, max_rows: int):
    """Times the oracle (CPU restatement of the reference kernel) on whole
    (sequence, head) rows; returns (GB/s, tokens/s-equivalent, rows, seconds)."""
    import numpy as np

    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    pages = bt[0].cpu().numpy()
    kp0 = kp[torch.from_numpy(pages).long().to(kp.device)].cpu().numpy()
    vp0 = vp[torch.from_numpy(pages).long().to(kp.device)].cpu().numpy()
    bt0 = np.arange(MB, dtype=np.int32)[None, :]
    q0 = q[0:1].cpu().numpy()
    ctx0 = np.array([CTX], np.int32)
    O.paged_attention_f16(q0[:, :, :1], kp0[:, :, :1].copy(), vp0[:, :, :1].copy(), bt0, ctx0, CTX, CTX)
    t = time.perf_counter()
    O.paged_attention_f16(q0, kp0, vp0, bt0, ctx0, CTX, CTX)  # one sequence, all heads
    t_seq = time.perf_counter() - t
    t_row = t_seq / H
    rows = int(max(1, min(max_rows, rows_budget_s / max(t_row, 1e-9))))
    nseq = max(1, rows // H)
    reps = max(1, rows // (nseq * H)) if rows >= H else 0
    if rows >= H:
        t = time.perf_counter()
        for _ in range(reps):
            O.paged_attention_f16(np.repeat(q0, nseq, 0), kp0, vp0, np.repeat(bt0, nseq, 0),
                                  np.repeat(ctx0, nseq), CTX, CTX)
        el = time.perf_counter() - t
        rows = reps * nseq * H
    else:
        t = time.perf_counter()
        O.paged_attention_f16(q0[:, :, :rows], kp0[:, :, :rows].copy(), vp0[:, :, :rows].copy(), bt0, ctx0,
                              CTX, CTX)
        el = time.perf_counter() - t
    row_bytes = step_bytes(B, CTX) / (B * H)
    return rows * row_bytes / el / 1e9, rows / H / el, rows, el


def cpu_sdpa_sample(torch, kp, vp, bt, q, ctx, nseq: int):
    """The reference's CPU paged attention (its _sdpa_fallback,
    triton_attention.py:473-550, restated in oracle/sdpa_port.py and checked
    bit for bit against its recorded outputs) on the first `nseq` sequences,
    all host threads.  Returns (GB/s, tokens/s, seconds) with the configs[1]
    algorithmic bytes of those sequences."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    from sdpa_port import paged_sdpa

    torch.set_num_threads(os.cpu_count())
    pages = bt[:nseq].reshape(-1).long().to(kp.device)
    ck = kp.index_select(0, pages).cpu()
    cv = vp.index_select(0, pages).cpu()
    cbt = torch.arange(nseq * MB, dtype=torch.int32).reshape(nseq, MB)
    cq, cctx = q[:nseq].cpu(), ctx[:nseq].cpu()
    with torch.no_grad():
        t = time.perf_counter()
        paged_sdpa(cq, ck, cv, cbt, cctx, CTX, CTX)
        el = time.perf_counter() - t
    return step_bytes(nseq, CTX) / el / 1e9, nseq / el, el


def run_reference(args) -> None:
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import torch

    kp, vp, bt, q, ctx = make_fp16_workload(torch, 1234, "cpu")
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, toks, el = cpu_sdpa_sample(torch, kp, vp, bt, q, ctx, B)  # the whole configs[1] step
        if i >= args.warmup:
            vals.append((gbs, toks, el))
    gbs = statistics.median(v[0] for v in vals)
    toks = statistics.median(v[1] for v in vals)
    cores = os.cpu_count()
    # The C restatement of the reference CUDA kernel's arithmetic (fp64,
    # OpenMP), the reference arm of earlier runs, as a second labelled number.
    c_gbs, c_toks, c_rows, c_el = cpu_sample(torch, kp, vp, bt, q, ctx, 10.0, B * H)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.median(v[2] for v in vals) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "decode_tokens_per_s": round(toks, 3),
        "config": config_dict(args.gpus),
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": "one whole configs[1] step per timed step (32 sequences x 32 heads x 4096 "
                                   "tokens): the reference's CPU paged attention (_sdpa_fallback: page gather + "
                                   "torch SDPA in fp32) restated in oracle/sdpa_port.py, bit-identical to its "
                                   "recorded outputs, all host threads"},
        "c_port": {"value": round(c_gbs, 4), "unit": "GB/s", "cores": cores,
                   "sample": f"{c_rows} (sequence, head) rows, oracle/memopt_oracle.c (the reference CUDA "
                             "kernel's arithmetic in fp64, OpenMP)"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    line["reference_gpu_kernel"] = reference_gpu_kernel(args)
    print(json.dumps(line), flush=True)


def reference_gpu_kernel(args) -> dict:
    """The reference's own CUDA dynamic_sparse_attention (attention.cu:371-521,
    compiled unmodified from its sources into oracle/_ref by
    oracle/build_ref.py) on the configs[1] workload, for comparison with this
    build's kernel.  The reference op synchronises the device after its
    launch (its debug-sync macro), so each call is timed alone with CUDA
    events on the default stream it launches on.  configs[1] is within its
    limits (8192 pages x 65536 elements < 2^31)."""
    try:
        import torch

        if not torch.cuda.is_available():
            return {"unavailable": "no CUDA device"}
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        from build_ref import load

        ref = load()
        if ref is None:
            return {"unavailable": "oracle/_ref/memopt_ref_C.so was not built (no reference checkout at build time)"}
        dev = torch.device("cuda", 0)
        kp, vp, bt, q, ctx = make_fp16_workload(torch, 1234, dev)
        stream = torch.cuda.default_stream(dev)
        with torch.cuda.stream(stream):
            ref.dynamic_sparse_attention(q, kp, vp, bt, ctx, CTX, CTX)
            torch.cuda.synchronize()
            ms = time_each(torch, lambda: ref.dynamic_sparse_attention(q, kp, vp, bt, ctx, CTX, CTX),
                           max(3, min(args.steps, 10)), stream)
        sbytes = step_bytes(B, CTX)
        peak, kind = peaks()
        return {"workload": "BASELINE configs[1] (the same seeded inputs as this build's headline)",
                "value": round(sbytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
                "frac_of_hbm_peak": round(sbytes / ms / 1e6 / peak, 4), "peak_kind": kind,
                "decode_tokens_per_s": round(B / (ms * 1e-3), 1),
                "kernel": "reference sparse_flash_attention_kernel<16,128> (one CTA per (sequence, head, query))"}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def config_dict(n: int) -> dict:
    return {"workload": "BASELINE configs[1]: paged fp16 decode, batch 32/GPU, 32 heads x 128, ctx 4096, "
                        "16-token pages, permuted block tables",
            "batch_per_gpu": B, "global_batch": B * n, "seq_len": CTX, "heads": H, "head_dim": D,
            "block_size": BS, "pages_per_gpu": NB,
            "l2": "inputs larger than L2: 2.15 GB of K/V per GPU streamed every step",
            "parallelism": f"dp{n} (sequences sharded, one pool per GPU, no data-path collective)"}


def run_ours(args) -> None:
    import torch

    from memopt.sharding import RankGroup, dist_env, job_rate

    ws_n, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # One process, one GPU and one pool per rank; sequences are sharded (each
    # rank runs the per-GPU workload on its own sequences: weak scaling).
    group = RankGroup.init("nccl", dev)
    barrier = group.barrier
    max_over_ranks = group.max

    import memopt_C
    from memopt import _capi

    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    kp, vp, bt, q, ctx = make_fp16_workload(torch, 1234 + rank, dev)
    out = torch.empty_like(q)
    wsb = _capi.workspace_size(B, 1, H, D, MB, BS, CTX, CTX)
    wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)

    def step():
        _capi.paged_attention_f16(q, kp, vp, bt, ctx, out, CTX, CTX, wsp, wsb, sp)

    # ---- device-resident decode (value) --------------------------------------
    with Clocks(local) as clk:
        ms = time_loop(torch, step, args.steps, args.warmup, barrier, stream)
    ms = max_over_ranks(ms)
    sbytes = step_bytes(B, CTX)
    value = job_rate(sbytes, ms, ws_n) / 1e9
    tokens = job_rate(B, ms, ws_n)
    peak, peak_kind = peaks()
    kernel_gbs = sbytes / (ms * 1e-3) / 1e9  # one kernel launch per step

    # ---- end to end through the public API (host buffers) --------------------
    hq = torch.randn(B, 1, H, D, dtype=torch.float16).pin_memory()
    hk = torch.randn(B, H, D, dtype=torch.float16).pin_memory()
    hv = torch.randn(B, H, D, dtype=torch.float16).pin_memory()
    bt_cpu = bt.cpu()
    hslots = (bt_cpu[:, MB - 1] * BS + (BS - 1)).to(torch.int32).pin_memory()  # token CTX-1 of each seq
    hbt = bt_cpu.pin_memory()
    hctx = ctx.cpu().pin_memory()
    hout = torch.empty(B, 1, H, D, dtype=torch.float16).pin_memory()
    memopt_C.init_pool(NB, BS, H, D)
    pk, pv = memopt_C.get_pool_tensors()
    pk.copy_(kp)
    pv.copy_(vp)
    del kp, vp
    dq = torch.empty_like(hq, device=dev)
    dk = torch.empty_like(hk, device=dev)
    dv = torch.empty_like(hv, device=dev)
    ds = torch.empty_like(hslots, device=dev)
    dbt = torch.empty_like(hbt, device=dev)
    dctx = torch.empty_like(hctx, device=dev)

    # Serving-style pipeline: the step's host->device copies run on a copy
    # stream into one of two device buffer sets while the previous step's
    # attention runs, and its output goes back on a second copy stream; the
    # compute stream waits for the step's inputs.  Every copy of every step
    # is inside the timed region.
    dq, dk, dv, ds, dbt, dctx = [[x, torch.empty_like(x)] for x in (dq, dk, dv, ds, dbt, dctx)]
    houts = [hout, torch.empty_like(hout).pin_memory()]
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    freed = [torch.cuda.Event(), torch.cuda.Event()]  # buffer set i no longer read by compute
    for e in freed:
        e.record(stream)
    it = [0]

    def e2e_step():
        i = it[0] & 1
        it[0] += 1
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(freed[i])
            for d_, h_ in ((dq, hq), (dk, hk), (dv, hv), (ds, hslots), (dbt, hbt), (dctx, hctx)):
                d_[i].copy_(h_, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(h2d_s)
        stream.wait_event(ready)
        memopt_C.write_cache(dk[i], dv[i], dbt[i], ds[i])
        o = memopt_C.dynamic_sparse_attention(dq[i], pk, pv, dbt[i], dctx[i], CTX, CTX)
        done = torch.cuda.Event()
        done.record(stream)
        freed[i].record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(done)
            houts[i].copy_(o, non_blocking=True)
            o.record_stream(d2h_s)

    def e2e_loop(n):
        for _ in range(n):
            e2e_step()
        stream.wait_stream(d2h_s)  # the last outputs are on the host before the end event

    e2e_steps = max(1, min(args.steps, 500))
    ms_e2e = max_over_ranks(time_e2e(torch, e2e_loop, e2e_steps, args.warmup, barrier, stream, h2d_s))
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hslots, hbt, hctx))
    d2h = hout.numel() * hout.element_size()
    e2e = job_rate(sbytes, ms_e2e, ws_n) / 1e9

    # ---- INT4 decode as a secondary line ---------------
    extra = {}
    if not args.no_int4:
        # Each leg starts from an empty allocator cache, so its buffers are
        # fresh allocations rather than pieces of an earlier leg's segments.
        legs = [lambda: int4_extra(torch, memopt_C, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank),
                lambda: prefill_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank),
                lambda: evict_extra(torch, memopt_C, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n,
                                    rank),
                lambda: long_decode_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank),
                lambda: multi_query_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank),
                lambda: ops_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank)]
        # SM clocks over each group's timed loops (the later legs run with the
        # GPU warm, often under sw_power_cap), recorded with its legs.
        groups = []
        lclk = Clocks(local, log_path=os.path.join(tempfile.gettempdir(), f"memopt_leg_clocks_{os.getpid()}.log"))
        with lclk:
            for leg in legs:
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
                n0 = len(TIMED_WINDOWS)
                r = leg()
                groups.append((r, TIMED_WINDOWS[n0:]))
        for r, wins in groups:
            cs = lclk.windows_summary(wins)
            for v in r.values():
                if isinstance(v, dict):
                    v["clocks"] = cs
            extra.update(r)
        if ws_n > 1:
            extra.update(evict_head_sharded_extra(torch, memopt_C, dev, stream, group, ws_n))

    # ---- CPU baseline (rank 0, N=1 only) --------------------------------------
    cpu = None
    if ws_n == 1 and not args.no_cpu:
        # whole configs[1] steps (all 32 sequences) until about 8 s of CPU
        # work (at least 3, at most 25 steps); the median step is reported
        nseq = B
        sdpa, spent = [], 0.0
        while len(sdpa) < 3 or (spent < 8.0 and len(sdpa) < 25):
            sdpa.append(cpu_sdpa_sample(torch, pk, pv, bt, q, ctx, nseq))
            spent += sdpa[-1][2]
        gbs, toks, el = sorted(sdpa)[len(sdpa) // 2]
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"whole configs[1] steps ({nseq} sequences, all heads, 4096 tokens), median of "
                         f"{len(sdpa)} steps ({el:.2f} s each, {spent:.1f} s in all): the reference's CPU paged "
                         "attention (_sdpa_fallback) restated in oracle/sdpa_port.py, all host threads",
               "decode_tokens_per_s": round(toks, 3)}

    if rank != 0:
        group.destroy()
        return
    traffic = None
    tpath = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("paged_decode_f16_cfg2_bytes_per_launch")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws_n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded N(0,1) K/V/q, permuted block tables)",
        "decode_tokens_per_s": round(tokens, 1),
        "pct_of_hbm_peak": round(100 * kernel_gbs / peak, 2),
        "config": config_dict(ws_n),
        "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(kernel_gbs / peak, 4), "traffic": traffic,
                     "kernel": "paged_decode_kernel<128,16,false>", "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": sbytes},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(ms_e2e, 5), "steps": e2e_steps,
                "path": "memopt_C.write_cache + memopt_C.dynamic_sparse_attention, pinned host buffers; each step's "
                        "copies overlap the previous step's attention (two buffer sets, two copy streams)"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
        "extra": extra,
    }
    print(json.dumps(line), flush=True)
    print_leg_summary(extra, ws_n)
    group.destroy()


# Order of the one-line summaries printed after the JSON line: the north-star
# legs come last, so that a reader of the last lines of the output sees them.
LEG_ORDER = ["evict_tokens", "evict_tokens_l2_flushed", "evict_tokens_no_sinks_l2_flushed", "evict_cache",
             "evict_topk_compact", "evict_topk_compact_int4",
             "evict_topk_head_sharded", "window_decode", "quantize_int4", "dequantize_int4", "write_cache_f16",
             "multi_row_decode_f16", "gqa_decode_f16", "gqa_decode_int4", "long_context_decode_retain_0.75",
             "long_context_decode", "int4_prefill", "prefill", "int4_write_cache", "int4_decode"]


def print_leg_summary(extra: dict, n: int) -> None:
    """One short text line per secondary leg (not JSON: the JSON line above is
    the bench result): value, unit, fraction of the measured peak, time."""
    names = [k for k in LEG_ORDER if k in extra] + [k for k in extra if k not in LEG_ORDER]
    for k in names:
        v = extra[k]
        frac = next((v[f] for f in ("frac_of_hbm_peak", "frac_of_hbm_peak_per_gpu", "frac_of_tensor_peak")
                     if f in v), None)
        ms = next((v[f] for f in ("ms_per_step", "ms_per_call", "ms_per_launch") if f in v), None)
        fs = f" frac {frac:.3f}" if frac is not None else ""
        c = v.get("clocks") or {}
        cs = f" sm {c['sm_mhz']:.0f} MHz {','.join(c['reasons']) or '-'}" if c.get("sm_mhz") else ""
        print(f"leg {k} N={n}: {v['value']} {v['unit']}{fs} {ms} ms{cs}", flush=True)


def int4_extra(torch, memopt_C, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """INT4 pool written by the fused write_cache, then
    decode with fused dequant.  Reported as secondary numbers."""
    b, ctx_len = INT4_B, INT4_CTX
    mb = ctx_len // BS
    nb = b * mb
    memopt_C.init_pool(nb, BS, H, D, kv_format="int4")
    pages = memopt_C.get_int4_pages()
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(7 + rank)).to(torch.int32)
    bt = perm[: b * mb].reshape(b, mb).to(dev)
    # Token t of sequence s goes to page bt[s, t // BS], slot t % BS.
    chunk = 32768
    T = b * ctx_len
    slots_all = (bt.reshape(-1).repeat_interleave(BS) * BS +
                 torch.arange(BS, device=dev, dtype=torch.int32).repeat(b * mb)).to(torch.int32)
    kbuf = torch.empty(chunk, H, D, dtype=torch.float16, device=dev)
    vbuf = torch.empty_like(kbuf)
    write_ms = []
    for c0 in range(0, T, chunk):
        kbuf.normal_(generator=g)
        vbuf.normal_(generator=g)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        memopt_C.write_cache(kbuf, vbuf, bt, slots_all[c0:c0 + chunk])
        e1.record(stream)
        torch.cuda.synchronize()
        write_ms.append(e0.elapsed_time(e1))
    wms = max_over_ranks(statistics.median(write_ms[1:] if len(write_ms) > 1 else write_ms))
    wbytes_chunk = 2 * chunk * H * D * 2 + 2 * chunk * H * (D // 2) + 2 * chunk * H * (D // 64) * 2 + chunk * 4
    q = torch.randn(b, 1, H, D, dtype=torch.float16, device=dev, generator=g)
    ctx = torch.full((b,), ctx_len, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    wsb = _capi.workspace_size(b, 1, H, D, mb, BS, ctx_len, ctx_len)
    wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)

    def step():
        _capi.paged_attention_int4(q, pages, BS, bt, ctx, out, ctx_len, ctx_len, wsp, wsb, sp)

    ms = max_over_ranks(time_loop(torch, step, max(args.steps, 20), args.warmup, barrier, stream))
    sbytes = step_bytes(b, ctx_len, "int4")
    peak, _ = peaks()
    return {"int4_decode": {"workload": "BASELINE configs[2]: batch 16/GPU, ctx 16384, INT4 g64 pages",
                            "value": round(sbytes * ws_n / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                            "ms_per_step": round(ms, 5),
                            "frac_of_hbm_peak": round(sbytes / (ms * 1e-3) / 1e9 / peak, 4),
                            "decode_tokens_per_s": round(b * ws_n / (ms * 1e-3), 1),
                            "algorithmic_bytes_per_launch": sbytes},
            "int4_write_cache": {"value": round(wbytes_chunk * ws_n / (wms * 1e-3) / 1e9, 2), "unit": "GB/s",
                                 "frac_of_hbm_peak": round(wbytes_chunk / (wms * 1e-3) / 1e9 / peak, 4),
                                 "tokens_per_launch": chunk, "ms_per_launch": round(wms, 5)}}


def run_only(args) -> None:
    """One kernel family in isolation (for ncu captures and quick timing)."""
    import torch

    import memopt_C
    from memopt import _capi

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    if args.only == "fp16":
        kp, vp, bt, q, ctx = make_fp16_workload(torch, 1234, dev)
        out = torch.empty_like(q)
        wsb = _capi.workspace_size(B, 1, H, D, MB, BS, CTX, CTX)
        wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)
        ms = time_loop(torch, lambda: _capi.paged_attention_f16(q, kp, vp, bt, ctx, out, CTX, CTX, wsp, wsb, sp),
                       args.steps, args.warmup, lambda: None, stream)
        res = {"kernel": "paged_decode f16 cfg2", "ms": ms, "GB/s": step_bytes(B, CTX) / ms / 1e6}
    elif args.only == "evict":
        res = evict_extra(torch, memopt_C, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    elif args.only == "prefill":
        res = prefill_extra(torch, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    elif args.only == "mq":
        res = multi_query_extra(torch, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    elif args.only == "ops":
        res = ops_extra(torch, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    elif args.only == "long":
        res = long_decode_extra(torch, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    else:
        res = int4_extra(torch, memopt_C, _capi, dev, sp, stream, args, lambda: None, lambda x: x, 1, 0)
    print(json.dumps(res), flush=True)


def time_each(torch, fn, n: int, stream, flush=None) -> float:
    """Median device time (ms) of n calls timed one by one with CUDA events on
    `stream`; `flush` (untimed) runs before each call."""
    evs = []
    w0 = time.time()
    for _ in range(n):
        if flush is not None:
            flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        evs.append((e0, e1))
    torch.cuda.synchronize()
    TIMED_WINDOWS.append((w0, time.time()))
    return statistics.median(a.elapsed_time(b) for a, b in evs)


def l2_flusher(torch, dev):
    """A write of 256 MB (twice the 126 MB L2) that evicts earlier data."""
    buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    return lambda: buf.zero_()


def ops_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """The data-plane operators besides decode, each on inputs larger than L2,
    median of >= 20 calls timed one by one:
    * quantize / dequantize (quantization.cu:104-270) of a 1.07 GB fp16 cache
      [16, 32, 8192, 128]: bytes = fp16 elements x 2 + codes (1/2 B per
      element) + fp32 scales (4 B per 64 elements);
    * fp16 write_cache (kv_cache.cu:228-348) of 131072 tokens x 32 heads x 128
      at configs[1] into an 8192-page pool: K and V read and written once plus
      the int32 slots;
    * evict_cache (kv_cache.cu:379-559) over a configs[3]-sized pool (16384
      pages x 16 x 32 heads x 128), retain 0.75: per (block, head) 12 rows
      kept, 4 zeroed; bytes = fp32 scores read + zeroed rows written."""
    peak, _ = peaks()
    res = {}
    n = max(20, min(args.steps, 50))
    g = torch.Generator(device=dev).manual_seed(71 + rank)
    # quantize / dequantize
    x = torch.randn(16, 32, 8192, 128, dtype=torch.float16, device=dev, generator=g)
    ne = x.numel()
    packed = torch.empty(16, 32, 8192, 64, dtype=torch.uint8, device=dev)
    scales = torch.empty(ne // 64, dtype=torch.float32, device=dev)
    qbytes = ne * 2 + ne // 2 + (ne // 64) * 4
    ms_q = max_over_ranks(time_each(torch, lambda: _capi.quantize_int4(x, packed, scales, sp), n, stream))
    y = torch.empty_like(x)
    ms_d = max_over_ranks(time_each(torch, lambda: _capi.dequantize_int4(packed, scales, y, sp), n, stream))
    res["quantize_int4"] = {"workload": "fp16 cache [16, 32, 8192, 128] (1.07 GB), group 64",
                            "value": round(qbytes * ws_n / (ms_q * 1e-3) / 1e9, 2), "unit": "GB/s",
                            "ms_per_call": round(ms_q, 5), "frac_of_hbm_peak": round(qbytes / ms_q / 1e6 / peak, 4),
                            "algorithmic_bytes_per_call": qbytes}
    res["dequantize_int4"] = {"workload": "packed codes + fp32 scales of the same cache -> fp16",
                              "value": round(qbytes * ws_n / (ms_d * 1e-3) / 1e9, 2), "unit": "GB/s",
                              "ms_per_call": round(ms_d, 5), "frac_of_hbm_peak": round(qbytes / ms_d / 1e6 / peak, 4),
                              "algorithmic_bytes_per_call": qbytes}
    del x, y, packed, scales
    # fp16 write_cache, 131072 tokens
    T = B * CTX
    keys = torch.randn(T, H, D, dtype=torch.float16, device=dev, generator=g)
    vals = torch.randn(T, H, D, dtype=torch.float16, device=dev, generator=g)
    kp = torch.empty(NB, BS, H, D, dtype=torch.float16, device=dev)
    vp = torch.empty_like(kp)
    slots = (torch.randperm(NB, generator=torch.Generator().manual_seed(9 + rank)).to(torch.int32)
             .repeat_interleave(BS) * BS + torch.arange(BS, dtype=torch.int32).repeat(NB)).to(dev)
    wbytes = 2 * (2 * T * H * D * 2) + T * 4
    ms_w = max_over_ranks(time_each(torch, lambda: _capi.write_cache_f16(keys, vals, slots, kp, vp, sp), n, stream))
    res["write_cache_f16"] = {"workload": "configs[1]: 131072 tokens x 32 heads x 128 fp16 into 8192 permuted pages",
                              "value": round(wbytes * ws_n / (ms_w * 1e-3) / 1e9, 2), "unit": "GB/s",
                              "ms_per_call": round(ms_w, 5), "frac_of_hbm_peak": round(wbytes / ms_w / 1e6 / peak, 4),
                              "tokens_per_s": round(T * ws_n / (ms_w * 1e-3), 1), "algorithmic_bytes_per_call": wbytes}
    del keys, vals, kp, vp, slots
    # evict_cache over a configs[3]-sized pool
    enb = 16384
    kp = torch.randn(enb, BS, H, D, dtype=torch.float16, device=dev, generator=g)
    vp = torch.randn_like(kp)
    sc = torch.empty(enb, BS, H, device=dev).log_normal_(0.0, 1.0, generator=g)
    keep = max(1, int(0.75 * BS))
    ebytes = sc.numel() * 4 + 2 * enb * H * (BS - keep) * D * 2
    ms_e = max_over_ranks(time_each(torch, lambda: _capi.evict_cache(sc, kp, vp, 0.75, sp), n, stream))
    res["evict_cache"] = {"workload": "configs[3] pool: 16384 pages x 16 x 32 heads x 128, lognormal scores, "
                                      "retain 0.75 (12 of 16 rows kept per block and head)",
                          "value": round(ebytes * ws_n / (ms_e * 1e-3) / 1e9, 2), "unit": "GB/s",
                          "ms_per_call": round(ms_e, 5), "frac_of_hbm_peak": round(ebytes / ms_e / 1e6 / peak, 4),
                          "algorithmic_bytes_per_call": ebytes}
    del kp, vp, sc
    torch.cuda.empty_cache()
    return res


def long_decode_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """BASELINE configs[4] decode: 64 sequences x 131072 cached tokens in INT4
    pages, the sequences sharded over the ranks (64 / N per GPU: strong
    scaling for this line; 36.5 GB of pages on one GPU).  The pages hold
    seeded random codes and fp16 scales in [0.05, 0.55) (the fused writer that
    produces real pages is timed in the int4 line); decode reads every byte
    of them either way."""
    from memopt.sharding import shard_range

    lo, hi = shard_range(LONG_B, ws_n, rank)
    b = hi - lo
    mb = LONG_CTX // BS
    nb = b * mb
    pbytes = BS * D + BS * (D // 64) * 4
    g = torch.Generator(device=dev).manual_seed(31 + rank)
    pages = torch.empty(nb, H, pbytes, dtype=torch.uint8, device=dev)
    pages.random_(0, 256, generator=g)
    sb = BS * (D // 64) * 2  # fp16 scale bytes per (page, head) for K, and again for V
    step_pages = 65536
    for p0 in range(0, nb, step_pages):
        p1 = min(nb, p0 + step_pages)
        sc = (torch.rand(p1 - p0, H, sb, device=dev, generator=g) * 0.5 + 0.05).half()
        pages[p0:p1, :, BS * D:] = sc.view(torch.uint8).view(p1 - p0, H, 2 * sb)
        del sc
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(41 + rank)).to(torch.int32).reshape(b, mb).to(dev)
    q = torch.randn(b, 1, H, D, dtype=torch.float16, device=dev, generator=g)
    ctx = torch.full((b,), LONG_CTX, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    wsb = _capi.workspace_size(b, 1, H, D, mb, BS, LONG_CTX, LONG_CTX)
    wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)

    def step():
        _capi.paged_attention_int4(q, pages, BS, bt, ctx, out, LONG_CTX, LONG_CTX, wsp, wsb, sp)

    steps = min(max(args.steps // 50, 10), 40)
    ms = max_over_ranks(time_loop(torch, step, steps, min(args.warmup, 5), barrier, stream))
    sbytes_rank = step_bytes(b, LONG_CTX, "int4")
    total = step_bytes(LONG_B, LONG_CTX, "int4")
    peak, _ = peaks()

    # configs[4] names retain_ratio 0.75: exact top-k eviction (this build's
    # operator; with sinks the reference's bisection keeps every token) on the
    # same pages, lognormal(0,1) scores, then decode over the compacted
    # contexts.  Eviction is destructive, so it is timed once (outputs and
    # workspace allocated beforehand).
    scores = torch.empty(b, H, LONG_CTX, device=dev).log_normal_(0.0, 1.0, generator=g)
    kept = torch.empty(b, LONG_CTX, dtype=torch.int32, device=dev)
    kcnt = torch.empty(b, dtype=torch.int32, device=dev)
    freed = torch.empty(b, mb, dtype=torch.int32, device=dev)
    fcnt = torch.empty(b, dtype=torch.int32, device=dev)
    ewsb = _capi.evict_topk_workspace_size(b, LONG_CTX, H, D)
    ews = torch.empty(ewsb, dtype=torch.uint8, device=dev)
    bt_c, ctx_c = bt.clone(), ctx.clone()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    _capi.evict_topk_compact_int4(scores, bt_c, ctx_c, pages, BS, D, 0.75, 4, kept, kcnt, freed, fcnt, ews, ewsb, sp)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_ev = max_over_ranks(e0.elapsed_time(e1))
    kept_ctx = int(ctx_c.max().item())
    moved = int(kcnt.sum().item())
    del scores, ews

    def step_c():
        _capi.paged_attention_int4(q, pages, BS, bt_c, ctx_c, out, LONG_CTX, LONG_CTX, wsp, wsb, sp)

    ms_c = max_over_ranks(time_loop(torch, step_c, steps, min(args.warmup, 5), barrier, stream))
    sbytes_c_rank = step_bytes(b, kept_ctx, "int4")
    total_c = step_bytes(LONG_B, kept_ctx, "int4")
    del pages
    torch.cuda.empty_cache()
    return {"long_context_decode_retain_0.75": {
        "workload": f"BASELINE configs[4] decode at retain_ratio 0.75: exact top-k eviction (4 sinks, lognormal "
                    f"scores) compacts each of {b} sequences on this GPU from 131072 to {kept_ctx} tokens, then "
                    f"decode over the compacted pages",
        "value": round(total_c / (ms_c * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms_c, 4),
        "frac_of_hbm_peak_per_gpu": round(sbytes_c_rank / (ms_c * 1e-3) / 1e9 / peak, 4),
        "decode_tokens_per_s": round(LONG_B / (ms_c * 1e-3), 1), "steps": steps, "scaling": "strong",
        "evict_ms": round(ms_ev, 3), "evict_kept_rows": moved,
        "evict_note": "one call (destructive); moves each kept token's codes and scales in every head's page"},
            "long_context_decode": {
        "workload": f"BASELINE configs[4] decode: 64 x 131072 tokens INT4, {b} sequences on this GPU "
                    f"(sequences sharded over {ws_n} GPU(s): strong scaling)",
        "value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
        "frac_of_hbm_peak_per_gpu": round(sbytes_rank / (ms * 1e-3) / 1e9 / peak, 4),
        "decode_tokens_per_s": round(LONG_B / (ms * 1e-3), 1), "steps": steps,
        "scaling": "strong", "bytes_per_step_whole_job": total,
        "data": "seeded random INT4 codes and fp16 scales in [0.05, 0.55)"}}


def prefill_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """BASELINE configs[4] prefill: 4 sequences x 8192 query tokens over their
    own 8192 cached tokens, 32 heads x 128, fp16, non-causal (reference
    semantics), on the tcgen05 path.  FLOPs = 4 * B * H * QL * ctx * D."""
    pb, pql = PREFILL_B, PREFILL_QL
    kp, vp, bt, q, ctx = make_prefill_workload(torch, dev, rank)
    out = torch.empty_like(q)

    def step():
        _capi.paged_attention_f16(q, kp, vp, bt, ctx, out, pql, pql, None, 0, sp)

    steps = max(3, min(args.steps, 20))
    ms = max_over_ranks(time_loop(torch, step, steps, args.warmup, barrier, stream))
    flops = 4.0 * pb * H * pql * pql * D
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        tpk, kind = float(pk["bf16_tflops"]), "measured"
        tpk_s = float(pk.get("bf16_tflops_sustained") or 0) or None
    except Exception:  # noqa: BLE001
        tpk, kind, tpk_s = 1590.0, "fallback", 1400.0
    tf = flops / (ms * 1e-3) / 1e12
    # The same prefill over an INT4 pool holding those K/V rows: the call
    # dequantises the sequences' pages into an fp16 scratch in its workspace,
    # then runs the same kernel (the reference dequantises an INT4 cache before
    # fp16 attention).  Same FLOPs; the dequantisation is inside the time.
    nb = kp.shape[0]
    pbytes = BS * D + BS * (D // 64) * 4
    pages = torch.zeros(nb, H, pbytes, dtype=torch.uint8, device=dev)
    slots = torch.arange(nb * BS, dtype=torch.int32, device=dev)
    _capi.write_cache_int4(kp.view(-1, H, D), vp.view(-1, H, D), slots, pages, BS, sp)
    del kp, vp, slots
    mb = bt.shape[1]
    wsb4 = _capi.int4_workspace_size_ex(pb, pql, H, H, D, mb, BS, pql, pql)
    ws4 = torch.zeros(max(wsb4, 1), dtype=torch.uint8, device=dev)

    def step4():
        _capi.paged_attention_int4(q, pages, BS, bt, ctx, out, pql, pql, ws4, wsb4, sp)

    ms4 = max_over_ranks(time_loop(torch, step4, steps, args.warmup, barrier, stream))
    tf4 = flops / (ms4 * 1e-3) / 1e12
    del pages, ws4
    int4_leg = {"workload": "BASELINE configs[4] prefill over an INT4 pool (the same K/V rows written by the fused "
                            "INT4 write_cache): 4 x 8192 tokens, 32 heads x 128, non-causal",
                "value": round(tf4 * ws_n, 2), "unit": "TFLOP/s", "ms_per_step": round(ms4, 4),
                "frac_of_tensor_peak": round(tf4 / tpk, 4), "peak_kind": kind,
                "workspace_bytes": wsb4,
                "kernel": "int4_pages_to_f16_kernel (pages -> fp16 scratch) + prefill_kernel<128,16> (tcgen05)"}
    return {"int4_prefill": int4_leg,
            "prefill": {"workload": "BASELINE configs[4] prefill: 4 x 8192 tokens, 32 heads x 128, fp16, "
                                    "non-causal over context_lens=8192",
                        "value": round(tf * ws_n, 2), "unit": "TFLOP/s", "ms_per_step": round(ms, 4),
                        "frac_of_tensor_peak": round(tf / tpk, 4), "peak_kind": kind, "flops_per_launch": flops,
                        "frac_of_sustained_tensor_peak": round(tf / tpk_s, 4) if tpk_s else None,
                        "note": "peak: the measured bf16 burst figure (a launch of ~4 ms timed alone); the "
                                "sustained figure is the same GEMM under the power cap for seconds",
                        "kernel": "prefill_kernel<128,16> (tcgen05)"}}


def evict_extra(torch, memopt_C, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """Ada-KV eviction (8 sequences x 32 heads x 32768
    tokens, lognormal(0,1) scores, 4 sinks, retain 0.75, with compaction of
    the kept indices) followed by block-skipping decode with window 4096."""
    eb, ectx, win = 8, 32768, 4096
    mb = ectx // BS
    nb = eb * mb
    memopt_C.init_pool(nb, BS, H, D)
    kp, vp = memopt_C.get_pool_tensors()
    g = torch.Generator(device=dev).manual_seed(21 + rank)
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(3 + rank))[: eb * mb].reshape(eb, mb)
    bt = bt.to(torch.int32).to(dev)
    scores = torch.empty(eb, H, ectx, device=dev).log_normal_(0.0, 1.0, generator=g)
    ibf = torch.zeros(nb, dtype=torch.int32, device=dev)

    idx_buf = torch.empty(eb, H, ectx, dtype=torch.int32, device=dev)
    cnt_buf = torch.empty(eb, H, dtype=torch.int32, device=dev)

    def evict():  # the kernel through the C-ABI, outputs preallocated
        _capi.evict_tokens(scores, bt, ibf, kp, vp, 0.75, 4, idx_buf, cnt_buf, sp)

    ev_steps = max(3, min(args.steps, 50))
    ms_ev = max_over_ranks(time_loop(torch, evict, ev_steps, args.warmup, barrier, stream))
    # the same calls with the L2 flushed before each (scores streamed from HBM)
    ms_ev_cold = max_over_ranks(time_each(torch, evict, max(20, ev_steps), stream, l2_flusher(torch, dev)))
    # Without sinks the threshold falls among the scores: the exact select of
    # the keep-th largest score runs and a quarter of the tokens are evicted
    # (their partial rows zeroed in K and V).  The pool is refilled below
    # before anything reads it.
    def evict_no_sinks():
        _capi.evict_tokens(scores, bt, ibf, kp, vp, 0.75, 0, idx_buf, cnt_buf, sp)

    ms_ev0 = max_over_ranks(time_each(torch, evict_no_sinks, max(20, ev_steps), stream, l2_flusher(torch, dev)))
    evicted0 = int((ectx - cnt_buf).sum().item())
    # scores read, index list written, D/32 halves zeroed per evicted token, head and pool
    ev0_bytes = 2 * eb * H * ectx * 4 + evicted0 * 2 * (D // 32) * 2
    idx, cnt = memopt_C.evict_tokens(scores, bt, ibf, 0.75, 4, return_retained=True)
    kept = float(cnt.float().mean().item()) / ectx
    ev_bytes = 2 * eb * H * ectx * 4  # scores read + kept-index list written (no row is evicted with sinks)
    # Exact top-k eviction with compaction (this build's operator), one call
    # on the same scores: head sums, select, and the kept rows moved.
    # (an untimed first call takes the workspace allocation; every call works
    # on fresh copies of the tables and lengths: the same work each time)
    topk_ms = []
    for it in range(4):
        bt_c = bt.clone()
        ctx_c = torch.full((eb,), ectx, dtype=torch.int32, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        _, kcnt, _, _ = memopt_C.evict_topk_compact(scores, bt_c, ctx_c, 0.75, 4)
        e1.record(stream)
        torch.cuda.synchronize()
        if it > 0:
            topk_ms.append(e0.elapsed_time(e1))
    ms_topk = max_over_ranks(statistics.median(topk_ms))
    kept_rows = int(kcnt.sum().item())
    topk_bytes = eb * H * ectx * 4 + 2 * 2 * kept_rows * H * D * 2  # scores + K/V rows read and written once
    # The same eviction on an INT4 pool of the same sequences (seeded random
    # codes and scales): each kept token moves 2 x D/2 code bytes and
    # 2 x D/64 fp16 scales per head.
    q4_ms = []
    memopt_C.init_pool(nb, BS, H, D, kv_format="int4")
    pages4 = memopt_C.get_int4_pages()
    pages4.random_(0, 256, generator=g)
    pages4[:, :, BS * D:].view(torch.float16).uniform_(0.05, 0.55, generator=g)
    for it in range(4):
        bt_c = bt.clone()
        ctx_c = torch.full((eb,), ectx, dtype=torch.int32, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        _, kcnt4, _, _ = memopt_C.evict_topk_compact(scores, bt_c, ctx_c, 0.75, 4)
        e1.record(stream)
        torch.cuda.synchronize()
        if it > 0:
            q4_ms.append(e0.elapsed_time(e1))
    ms_topk4 = max_over_ranks(statistics.median(q4_ms))
    topk4_bytes = eb * H * ectx * 4 + 2 * int(kcnt4.sum().item()) * H * (D + 4 * (D // 64))
    del pages4
    memopt_C.init_pool(nb, BS, H, D)
    kp, vp = memopt_C.get_pool_tensors()
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    q = torch.randn(eb, 1, H, D, dtype=torch.float16, device=dev, generator=g)
    ctx = torch.full((eb,), ectx, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    wsb = _capi.workspace_size(eb, 1, H, D, mb, BS, ectx, win)
    wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)

    def step():
        _capi.paged_attention_f16(q, kp, vp, bt, ctx, out, ectx, win, wsp, wsb, sp)

    ms = max_over_ranks(time_loop(torch, step, max(args.steps, 20), args.warmup, barrier, stream))
    dbytes = 2 * eb * win * H * D * 2 + 2 * eb * H * D * 2 + eb * (win // BS + 1) * 4
    peak, _ = peaks()
    return {"evict_tokens": {"workload": "BASELINE configs[3]: 8 x 32 heads x 32768 tokens, lognormal(0,1), "
                                         "4 sinks, retain 0.75, kept indices compacted",
                             "value": round(ev_bytes * ws_n / (ms_ev * 1e-3) / 1e9, 2), "unit": "GB/s",
                             "ms_per_call": round(ms_ev, 5), "kept_fraction": round(kept, 4),
                             "note": "reference semantics: with sinks the 32-step bisection keeps every token",
                             "l2": "the 33.5 MB of scores fit in L2 and stay resident between calls"},
            "evict_tokens_l2_flushed": {"workload": "the same evict_tokens calls with a 256 MB write between them "
                                                    "(scores read from HBM)",
                                        "value": round(ev_bytes * ws_n / (ms_ev_cold * 1e-3) / 1e9, 2), "unit": "GB/s",
                                        "ms_per_call": round(ms_ev_cold, 5),
                                        "frac_of_hbm_peak": round(ev_bytes / ms_ev_cold / 1e6 / peaks()[0], 4)},
            "evict_tokens_no_sinks_l2_flushed": {
                "workload": "the same scores without sink tokens (the threshold falls among them: exact select, "
                            "25% of tokens evicted, their partial rows zeroed), L2 flushed before each call",
                "value": round(ev0_bytes * ws_n / (ms_ev0 * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_call": round(ms_ev0, 5), "evicted_tokens": evicted0,
                "note": "bound by the reference's partial-row zeroing: 2-byte stores at d = t % 32 + 32k, so each "
                        "evicted (token, head) dirties 2 x D/32 separate 32-byte sectors that L2 must fill from "
                        "and write back to HBM (about 64 B of DRAM traffic per zeroed element)",
                "frac_of_hbm_peak": round(ev0_bytes / ms_ev0 / 1e6 / peaks()[0], 4)},
            "evict_topk_compact": {"workload": "BASELINE configs[3] scores, exact top-k shared across heads "
                                               "(retain 0.75, 4 sinks), kept K/V rows compacted, pages released",
                                   "value": round(topk_bytes * ws_n / (ms_topk * 1e-3) / 1e9, 2), "unit": "GB/s",
                                   "ms_per_call": round(ms_topk, 4), "kept_rows": kept_rows,
                                   "note": "median of 3 calls after an untimed one; kept rows move in place (each "
                                           "read and written once)"},
            "evict_topk_compact_int4": {"workload": "the same eviction on an INT4 pool of the same 8 x 32768 tokens "
                                                    "(32 heads x 128, seeded random codes and scales)",
                                        "value": round(topk4_bytes * ws_n / (ms_topk4 * 1e-3) / 1e9, 2), "unit": "GB/s",
                                        "ms_per_call": round(ms_topk4, 4),
                                        "note": "median of 3 calls after an untimed one; each kept token's codes "
                                                "and scales read and written once"},
            "window_decode": {"workload": "BASELINE configs[3]: decode batch 8, ctx 32768, window 4096",
                              "value": round(dbytes * ws_n / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                              "ms_per_step": round(ms, 5),
                              "frac_of_hbm_peak": round(dbytes / (ms * 1e-3) / 1e9 / peak, 4),
                              "decode_tokens_per_s": round(eb * ws_n / (ms * 1e-3), 1)}}


def multi_query_extra(torch, _capi, dev, sp, stream, args, barrier, max_over_ranks, ws_n, rank):
    """Decode shapes where several query rows read each KV head (the
    multi-query kernel): grouped-query attention with 32 query heads over 8 KV
    heads (batch 128, ctx 4096; fp16 and INT4 pools) and the configs[1] shape
    with 4 query rows per sequence (speculative decoding).  Bytes are the
    pool pages read once per (sequence, KV head) plus q/out; every sequence
    has its own pages (inputs larger than L2)."""
    peak, _ = peaks()
    res = {}
    g = torch.Generator(device=dev).manual_seed(61 + rank)
    cases = [("gqa_decode_f16", 128, 1, 32, 8, "f16"), ("gqa_decode_int4", 128, 1, 32, 8, "int4"),
             ("multi_row_decode_f16", 32, 4, 32, 32, "f16")]
    ctx_len = CTX
    mb = ctx_len // BS
    for name, b, ql, h, kvh, fmt in cases:
        nb = b * mb
        bt = torch.randperm(nb, generator=torch.Generator().manual_seed(5 + rank)).to(torch.int32)
        bt = bt.reshape(b, mb).to(dev)
        q = torch.randn(b, ql, h, D, dtype=torch.float16, device=dev, generator=g)
        ctx = torch.full((b,), ctx_len, dtype=torch.int32, device=dev)
        out = torch.empty_like(q)
        wsb = _capi.workspace_size_ex(b, ql, h, kvh, D, mb, BS, ctx_len, ctx_len)
        wsp = torch.zeros(max(wsb, 1), dtype=torch.uint8, device=dev)
        if fmt == "f16":
            kp = torch.randn(nb, BS, kvh, D, dtype=torch.float16, device=dev, generator=g)
            vp = torch.randn_like(kp)
            pool_bytes = 2 * b * ctx_len * kvh * D * 2

            def step():
                _capi.paged_attention_f16_ex(q, kp, vp, bt, ctx, out, ctx_len, ctx_len, False, wsp, wsb, sp)
        else:
            pb = BS * D + 2 * BS * (D // 64) * 2
            pages = torch.randint(0, 256, (nb, kvh, pb), dtype=torch.uint8, device=dev, generator=g)
            sc = pages[:, :, BS * D:].view(torch.float16)
            sc.uniform_(0.05, 0.55, generator=g)
            pool_bytes = b * mb * kvh * pb

            def step():
                _capi.paged_attention_int4_ex(q, pages, BS, bt, ctx, out, ctx_len, ctx_len, False, wsp, wsb, sp)
        ms = max_over_ranks(time_loop(torch, step, max(args.steps // 4, 20), args.warmup, barrier, stream))
        sbytes = pool_bytes + 2 * b * ql * h * D * 2 + b * mb * 4
        res[name] = {"workload": f"batch {b}/GPU, {ql} query row(s), {h} query heads over {kvh} KV heads x {D}, "
                                 f"ctx {ctx_len}, {fmt} pool",
                     "value": round(sbytes * ws_n / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                     "ms_per_step": round(ms, 5), "frac_of_hbm_peak": round(sbytes / (ms * 1e-3) / 1e9 / peak, 4),
                     "decode_tokens_per_s": round(b * ql * ws_n / (ms * 1e-3), 1),
                     "kernel": "paged_decode_mq_kernel"}
        del bt, q, out, wsp
        if fmt == "f16":
            del kp, vp
        else:
            del pages, sc
    return res


def evict_head_sharded_extra(torch, memopt_C, dev, stream, group, ws_n):
    """configs[3] eviction with the HEADS sharded (N > 1): every rank holds
    32/N heads of all 8 sequences (same block tables on every rank), sums its
    heads' scores, the partial rows are all-gathered over NCCL, and each rank
    compacts its own pool on the shared decision.  Timed per call, exchange
    included; the value counts every rank's scores and moved rows once."""
    from memopt.sharding import evict_exact_head_sharded

    eb, ectx = 8, 32768
    hl = H // ws_n
    mb = ectx // BS
    nb = eb * mb
    memopt_C.init_pool(nb, BS, hl, D)
    kp, vp = memopt_C.get_pool_tensors()
    g = torch.Generator(device=dev).manual_seed(41 + group.rank)
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(3)).reshape(eb, mb).to(torch.int32).to(dev)
    scores = torch.empty(eb, hl, ectx, device=dev).log_normal_(0.0, 1.0, generator=g)
    times = []
    for it in range(4):
        bt_c = bt.clone()
        ctx_c = torch.full((eb,), ectx, dtype=torch.int32, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        group.barrier()
        e0.record(stream)
        _, kcnt, _, _ = evict_exact_head_sharded(group, scores, bt_c, ctx_c, 0.75, 4, memopt_C)
        e1.record(stream)
        torch.cuda.synchronize()
        if it > 0:
            times.append(e0.elapsed_time(e1))
    ms = group.max(statistics.median(times))
    kept_rows = int(kcnt.sum().item())
    rank_bytes = eb * hl * ectx * 4 + 2 * 2 * kept_rows * hl * D * 2
    return {"evict_topk_head_sharded": {
        "workload": f"BASELINE configs[3] scores, heads sharded: {hl} heads of all {eb} sequences per GPU, "
                    "exact top-k shared across heads (retain 0.75, 4 sinks), rows compacted in place",
        "value": round(rank_bytes * ws_n / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_call": round(ms, 4),
        "kept_rows": kept_rows, "exchange_bytes_per_rank": eb * ectx * 4 * ws_n,
        "collective": "NCCL all-gather of the fp32 partial token scores (one row per sequence and rank)",
        "note": "median of 3 calls after an untimed one, max over ranks"}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-int4", action="store_true", help="skip the INT4 secondary line")
    ap.add_argument("--only", choices=["fp16", "int4", "prefill", "evict", "long", "mq", "ops"], help="time one kernel family alone (profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
