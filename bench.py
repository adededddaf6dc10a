"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

Default workload (the headline): gated delta-rule recurrent decode, batch 64,
H_qk=16, H_v=32, d_k=d_v=128, fp32 state [64,32,128,128] (128 MiB) updated in
place, bf16 q/k/v, 256 distinct token inputs cycled.  One step = one decode
step of the whole batch = one kernel launch.  Weak scaling: every rank owns
its own batch of 64 sequences; no collective on the data path.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config gdn_decode|gdn_prefill|kv_attention|gdn_layer|cache_ops|stack]

Without ``--config`` the decode line also carries, as secondary lines, the
chunked prefill (8 x 32768 tokens, the tensor-core kernel), the KV-cache
attention pass (causal and with a 512-token window), the gated delta-rule layer
(512-token prefill + 64 decode steps) and the 24-layer hybrid stack (128 x
(1024 + 256) tokens), each with its own roofline, e2e leg and CPU baseline.
``--config X`` prints X's line alone.

``--impl reference`` times the CPU oracle of the same path on the host cores
(the reference has no GPU implementation of this path), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """Polls NVML (read-only) every few ms while the timed region runs."""

    def __init__(self, device_index=0, period_s=0.005):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._idx = device_index
        self._thread = None
        self._nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            try:
                pr = torch.cuda.get_device_properties(self._idx)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(self._idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self):
        nv = self._nvml
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for n, bit in names.items():
                    if r & bit:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(self._period)

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# --------------------------------------------------------------- dist utils --
def init_dist(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return ws, rank, local  # host-only arm: rank 0 works, the others exit
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(x, ws, device):
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------- GDN decode ---
DECODE_B, DECODE_STEPS = 64, 256
H_QK, H_V, DK, DV = 16, 32, 128, 128


def cudart():
    """The CUDA runtime that torch has loaded, for the e2e legs' stream-ordered copies and events:
    cudaMemcpyAsync, cudaEventRecord and cudaStreamWaitEvent called directly (one C call each)."""
    import ctypes
    rt = ctypes.CDLL("libcudart.so.12")
    vp, sz, ci = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    rt.cudaMemcpyAsync.argtypes = [vp, vp, sz, ci, vp]
    rt.cudaEventRecord.argtypes = [vp, vp]
    rt.cudaStreamWaitEvent.argtypes = [vp, vp, ctypes.c_uint]
    rt.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(vp), ctypes.c_uint]
    rt.cudaEventDestroy.argtypes = [vp]
    for f in ("cudaMemcpyAsync", "cudaEventRecord", "cudaStreamWaitEvent", "cudaEventCreateWithFlags",
              "cudaEventDestroy"):
        getattr(rt, f).restype = ci
    return rt


def decode_bytes_per_step(B=DECODE_B):
    state = 2 * B * H_V * DK * DV * 4
    qk = 2 * B * H_QK * DK * 2
    v = B * H_V * DV * 2
    out = B * H_V * DV * 2
    gb = 2 * B * H_V * 4
    return state + qk + v + out + gb


def cpu_decode_sample(n_steps, threads):
    """Oracle decode steps at the full batch on the host cores; returns steps/s."""
    from anemll_b200 import inputs
    from oracle import gdn as og
    torch.set_num_threads(threads)
    w = inputs.gdn_decode(B=DECODE_B, steps=min(n_steps, DECODE_STEPS))
    S = w["state"]
    # warm one step
    og.recurrent_gated_delta_rule(w["q"][0], w["k"][0], w["v"][0], w["g"][0], w["beta"][0], S)
    t0 = time.perf_counter()
    for i in range(n_steps):
        t = i % w["q"].shape[0]
        _, S = og.recurrent_gated_delta_rule(w["q"][t], w["k"][t], w["v"][t], w["g"][t], w["beta"][t], S)
    dt = time.perf_counter() - t0
    return n_steps / dt


def decode_config(ws):
    return {"workload": "gdn_recurrent_decode", "batch_per_gpu": DECODE_B, "H_qk": H_QK, "H_v": H_V,
            "d_k": DK, "d_v": DV, "state_bytes": DECODE_B * H_V * DK * DV * 4, "tokens_cycled": DECODE_STEPS,
            "l2": "no flush: two batch-64 states (2 x 128 MiB) alternate step by step, so no step reads "
                  "state the previous one left in the 126 MB L2",
            "parallelism": f"weak, {ws} independent batch shards"}


def bench_gdn_decode(args, ws, rank, local):
    from anemll_b200 import _lib, gdn, inputs
    dev = torch.device("cuda", local)
    from anemll_b200 import shard
    w = inputs.gdn_decode(seed=shard.decode_seed(1, rank), B=DECODE_B, steps=DECODE_STEPS)
    # two batches' states alternate step by step, so no step reads state that the previous step left in
    # the 126 MB L2 (one state is 128 MiB, but L2 still holds the tail the previous step wrote)
    states = [w["state"].to(dev), w["state"].to(dev)]
    q, k, v, g, beta = (w[n].to(dev) for n in ("q", "k", "v", "g", "beta"))
    out = torch.empty(DECODE_B, 1, H_V, DV, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    sp = _lib.stream_ptr(dev)
    # pre-resolved raw pointers: the timed loop is one C call per step
    ptrs = [(_lib.ptr(q[t]), _lib.ptr(k[t]), _lib.ptr(v[t]), _lib.ptr(g[t]), _lib.ptr(beta[t]))
            for t in range(DECODE_STEPS)]
    sptrs, optr = [_lib.ptr(x) for x in states], _lib.ptr(out)

    def step(i):
        pq, pk, pv, pg, pb = ptrs[i % DECODE_STEPS]
        rc = lib.anemll_gdn_recurrent(pq, pk, pv, _lib.BF16, pg, pb, sptrs[i & 1], optr, _lib.BF16,
                                      DECODE_B, 1, H_QK, H_V, DK, DV, 0.0, 0, sp)
        if rc:
            _lib.check(rc, "anemll_gdn_recurrent")

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    barrier(ws)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(ws)
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, ws, dev)

    # End to end through the public op with host buffers.  Serial form: every step copies its five
    # inputs from pinned memory, runs the op and reads its output back, all on one stream.
    hq, hk, hv, hg, hb = (w[n].pin_memory() for n in ("q", "k", "v", "g", "beta"))
    dq, dk_, dv_, dg, db = (torch.empty_like(x[0], device=dev) for x in (hq, hk, hv, hg, hb))
    hout = torch.empty(DECODE_B, 1, H_V, DV, dtype=torch.bfloat16).pin_memory()
    h2d = sum(x[0].numel() * x.element_size() for x in (hq, hk, hv, hg, hb))
    d2h = hout.numel() * hout.element_size()

    def e2e_serial_step(i):
        t = i % DECODE_STEPS
        dq.copy_(hq[t], non_blocking=True)
        dk_.copy_(hk[t], non_blocking=True)
        dv_.copy_(hv[t], non_blocking=True)
        dg.copy_(hg[t], non_blocking=True)
        db.copy_(hb[t], non_blocking=True)
        gdn.recurrent_gated_delta_rule_(dq, dk_, dv_, dg, db, states[i & 1], out=out)
        hout.copy_(out, non_blocking=True)

    def timed_e2e(step_fn, streams=()):
        for i in range(args.warmup):
            step_fn(i)
        torch.cuda.synchronize(dev)
        barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for s2 in streams:  # the copy streams start with the timed region ...
            s2.wait_event(e0)
        for i in range(args.steps):
            step_fn(i)
        for s2 in streams:  # ... and it ends after their last copy
            stream.wait_stream(s2)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return max_over_ranks(e0.elapsed_time(e1), ws, dev)

    e2e_serial_ms = timed_e2e(e2e_serial_step)

    # Pipelined form (the headline e2e): a serving loop that keeps the kernel busy, driving the C-ABI
    # entry point (anemll_gdn_recurrent) and the CUDA runtime directly, so that the host issues a step
    # in a few microseconds.  Each step's inputs sit in one pinned host buffer and go to the device in
    # one copy on a copy stream, a step ahead of the kernel; the output comes back on a third stream
    # while the next step computes.  Device input and output buffers are double-buffered, guarded by
    # events.
    names = ("q", "k", "v", "g", "beta")
    sizes = [w[n][0].numel() * w[n].element_size() for n in names]
    offs, o = [], 0
    for sz in sizes:
        offs.append(o)
        o += (sz + 255) // 256 * 256
    step_bytes = o
    hin = torch.empty(DECODE_STEPS, step_bytes, dtype=torch.uint8).pin_memory()
    for t in range(DECODE_STEPS):
        for n, off, sz in zip(names, offs, sizes):
            hin[t, off:off + sz].copy_(w[n][t].contiguous().view(-1).view(torch.uint8))
    din = [torch.empty(step_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    vptrs = [tuple(din[b].data_ptr() + off for off in offs) for b in range(2)]
    douts = [torch.empty(DECODE_B, 1, H_V, DV, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    houts = torch.empty(2, DECODE_B, 1, H_V, DV, dtype=torch.bfloat16).pin_memory()
    hin_p = [hin[t].data_ptr() for t in range(DECODE_STEPS)]
    din_p, dout_p, hout_p = [x.data_ptr() for x in din], [x.data_ptr() for x in douts], [houts[b].data_ptr()
                                                                                          for b in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    rt = cudart()
    h_in, h_out, h_cmp = s_in.cuda_stream, s_out.cuda_stream, stream.cuda_stream

    def new_event():
        import ctypes
        ev = ctypes.c_void_p()
        if rt.cudaEventCreateWithFlags(ctypes.byref(ev), 2):  # cudaEventDisableTiming
            raise RuntimeError("cudaEventCreateWithFlags failed")
        return ev.value

    ev_in, ev_k, ev_out = ([new_event() for _ in range(2)] for _ in range(3))

    def cu(rc, what):
        if rc:
            raise RuntimeError(f"e2e: {what} failed (CUDA error {rc})")

    def e2e_step(i):
        b = i & 1
        if i >= 2:
            cu(rt.cudaStreamWaitEvent(h_in, ev_k[b], 0), "cudaStreamWaitEvent")  # kernel i - 2 read din[b]
        cu(rt.cudaMemcpyAsync(din_p[b], hin_p[i % DECODE_STEPS], step_bytes, 1, h_in), "cudaMemcpyAsync")
        cu(rt.cudaEventRecord(ev_in[b], h_in), "cudaEventRecord")
        cu(rt.cudaStreamWaitEvent(h_cmp, ev_in[b], 0), "cudaStreamWaitEvent")
        if i >= 2:
            cu(rt.cudaStreamWaitEvent(h_cmp, ev_out[b], 0), "cudaStreamWaitEvent")  # step i - 2 read douts[b]
        pq, pk, pv, pg, pb = vptrs[b]
        rc = lib.anemll_gdn_recurrent(pq, pk, pv, _lib.BF16, pg, pb, sptrs[i & 1], dout_p[b], _lib.BF16,
                                      DECODE_B, 1, H_QK, H_V, DK, DV, 0.0, 0, h_cmp)
        if rc:
            _lib.check(rc, "anemll_gdn_recurrent")
        cu(rt.cudaEventRecord(ev_k[b], h_cmp), "cudaEventRecord")
        cu(rt.cudaStreamWaitEvent(h_out, ev_k[b], 0), "cudaStreamWaitEvent")
        cu(rt.cudaMemcpyAsync(hout_p[b], dout_p[b], d2h, 2, h_out), "cudaMemcpyAsync")
        cu(rt.cudaEventRecord(ev_out[b], h_out), "cudaEventRecord")

    e2e_ms = timed_e2e(e2e_step, (s_in, s_out))
    if not torch.equal(houts[(args.steps - 1) & 1].to(dev), douts[(args.steps - 1) & 1]):
        raise RuntimeError("e2e: the last step's output read back does not match the device copy")
    # the same copies without the kernel: how long a step's H2D and D2H take on their own (they hide
    # under the neighbouring steps' kernels when the pipelined leg approaches the device-timed value)
    def copy_step(i):
        b = i & 1
        cu(rt.cudaMemcpyAsync(din_p[b], hin_p[i % DECODE_STEPS], step_bytes, 1, h_cmp), "cudaMemcpyAsync")
        cu(rt.cudaMemcpyAsync(hout_p[b], dout_p[b], d2h, 2, h_cmp), "cudaMemcpyAsync")

    copies_ms = timed_e2e(copy_step)
    for ev in ev_in + ev_k + ev_out:
        rt.cudaEventDestroy(ev)

    pk, how = peaks()
    per_launch_s = ms / 1e3 / args.steps
    achieved = decode_bytes_per_step() / per_launch_s / 1e9
    res = {
        "metric": "gdn_decode_steps_per_s",
        "value": ws * args.steps / (ms_max / 1e3),
        "unit": "steps/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 state, bf16 q/k/v/out",
        "data": "synthetic (seeded; state ~N(0,0.01), q/k l2-normalised N(0,1), v ~N(0,1))",
        "config": decode_config(ws),
        "tokens_per_s": ws * args.steps * DECODE_B / (ms_max / 1e3),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / pk["hbm_gbs"], "peak_source": how,
                     "algorithmic_bytes_per_launch": decode_bytes_per_step(),
                     # ncu DRAM bytes (read + write) per launch in steady state (consecutive launches,
                     # caches not flushed: each launch's window carries the write-back of the previous
                     # launch's dirty state lines), and the fraction of the peak those bytes reach
                     "traffic": traffic_from_profiles("gdn_recurrent_decode"),
                     "dram_frac": dram_frac(traffic_from_profiles("gdn_recurrent_decode"), per_launch_s,
                                            pk["hbm_gbs"])},
        "e2e": {"value": ws * args.steps / (e2e_ms / 1e3), "unit": "steps/s", "h2d_bytes_per_step": step_bytes,
                "d2h_bytes_per_step": d2h,
                "form": "pipelined: one H2D copy of the step's packed inputs on a copy stream a step ahead, "
                        "the C-ABI call anemll_gdn_recurrent, the output's D2H on a third stream "
                        "(double-buffered, events; copies and events through the CUDA runtime)",
                "copies_alone_us_per_step": copies_ms / args.steps * 1e3},
        "e2e_serial": {"value": ws * args.steps / (e2e_serial_ms / 1e3), "unit": "steps/s",
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                       "form": "five H2D copies, the public op and the D2H copy on one stream"},
        "gpu_launches": args.steps,
    }
    res["clocks"] = clk.summary()
    return res


PREFILL_B, PREFILL_T, CHUNK = 8, 32768, 64
PREFILL_FLOP_PER_TOKEN_HEAD = (2 * CHUNK * CHUNK * (3 * DK + 2 * DV) + 6 * CHUNK * DK * DV) // CHUNK  # 180,224


def prefill_config(ws, nseq=PREFILL_B, seqlen=PREFILL_T):
    return {"workload": "gdn_chunked_prefill", "batch": nseq, "seq_len": seqlen, "chunk": CHUNK,
            "H_qk": H_QK, "H_v": H_V, "d_k": DK, "d_v": DV,
            "l2": "no flush: 4.3 GB of inputs per step exceed the 126 MB L2",
            "parallelism": f"{ws} ranks, sequences x value heads, no collective"}


def bench_gdn_prefill(args, ws, rank, local):
    """Chunked prefill, B=8 x 32768 tokens, H_qk=16, H_v=32, d=128, bf16 in, bf16 out.

    Sharding: the 8 sequences are split over the ranks (one launch per rank per
    step); with more ranks than sequences the value heads are split too (the
    head pairs that share a key head stay together).  One step = one prefill of
    this rank's shard; value = all tokens of the job / max-over-ranks time."""
    from anemll_b200 import gdn, inputs, shard
    dev = torch.device("cuda", local)
    nseq, seqlen = args.prefill_seqs, args.prefill_len
    sh = shard.prefill_shard(ws, rank, nseq, H_QK, H_V)
    b_loc, hv_loc, hqk_loc = sh.seq_count, sh.v_head_count, sh.k_head_count
    w = inputs.gdn_prefill_device(seed=3 + 1000 * rank, B=b_loc, T=seqlen, device=dev, Hqk=hqk_loc, Hv=hv_loc)
    state = torch.zeros(b_loc, hv_loc, DK, DV, device=dev)
    out = torch.empty(b_loc, seqlen, hv_loc, DV, dtype=torch.bfloat16, device=dev)

    def step():
        gdn.chunk_gated_delta_rule_(w["q"], w["k"], w["v"], w["g"], w["beta"], state, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(ws)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(ws)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, ws, dev)
    if gdn.chunked_device_error(reset=True):
        raise RuntimeError("chunked prefill reported a device-side wait timeout")

    # End to end through the public op with host buffers (a few steps: the PCIe copies dominate).
    # Sequence by sequence: the H2D of its q/k/v/g/beta from pinned memory on a copy stream, its
    # prefill on the compute stream, the D2H of its output on a third stream, so that the copies in
    # and out of neighbouring sequences overlap each other and the kernels.
    host = {n: w[n].cpu().pin_memory() for n in ("q", "k", "v", "g", "beta")}
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in host.values())
    d2h = hout.numel() * hout.element_size()
    e2e_steps = min(args.steps, 3)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(b_loc)]
    ev_k = [torch.cuda.Event() for _ in range(b_loc)]

    def e2e_step():
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        for sq in range(b_loc):
            with torch.cuda.stream(s_in):
                for n, x in host.items():
                    w[n][sq].copy_(x[sq], non_blocking=True)
            ev_in[sq].record(s_in)
            stream.wait_event(ev_in[sq])
            sl = slice(sq, sq + 1)
            gdn.chunk_gated_delta_rule_(w["q"][sl], w["k"][sl], w["v"][sl], w["g"][sl], w["beta"][sl], state[sl],
                                        out=out[sl])
            ev_k[sq].record(stream)
            s_out.wait_event(ev_k[sq])
            with torch.cuda.stream(s_out):
                hout[sq].copy_(out[sq], non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)

    e2e_step()
    torch.cuda.synchronize(dev)
    if not torch.equal(hout[-1].to(dev), out[-1]):
        raise RuntimeError("e2e: the last sequence's output read back does not match the device copy")
    barrier(ws)
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1), ws, dev)
    tokens_local = b_loc * seqlen
    tokens_job = nseq * seqlen
    flop_launch = tokens_local * hv_loc * PREFILL_FLOP_PER_TOKEN_HEAD
    per_launch_s = ms / 1e3 / args.steps
    pk, how = peaks()
    achieved = flop_launch / per_launch_s / 1e12
    return {
        "metric": "gdn_prefill_tokens_per_s",
        "value": tokens_job * args.steps / (ms_max / 1e3),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 (inputs as tensor-core operands; derived operands split hi+lo), f32 accumulate/state, bf16 in/out",
        "data": "synthetic (seeded on device; q/k l2-normalised N(0,1), v ~N(0,1))",
        "config": prefill_config(ws, nseq, seqlen),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["bf16_tflops"], "peak_source": how,
                     "algorithmic_flop_per_launch": flop_launch,
                     # ncu DRAM bytes of one 8 x 4096 launch, scaled by the tokens to the 8 x 32768 launch
                     "traffic": (traffic_from_profiles("gdn_chunked_prefill_8x32768")
                                 if (ws, nseq, seqlen) == (1, 8, 32768) else None)},
        "e2e": {"value": tokens_job * e2e_steps / (e2e_ms / 1e3), "unit": "tokens/s", "steps": e2e_steps,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "form": "per sequence: H2D of its inputs (copy stream), the public op, D2H of its output "
                        "(third stream); neighbouring sequences overlap"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }


def kv_config(ws, window):
    return {"workload": "kv_cache_attention", "H_q": 16, "H_kv": 2, "head_dim": 256, "ctx": 4096,
            "prefill_chunks": 31, "chunk": 64, "decode_steps": 64, "window": window,
            "l2": "flushed (256 MB write) before the prefill chunks and before the decode steps of every timed "
                  "pass; within a pass the one-layer cache (8 MiB) stays L2-resident",
            "parallelism": f"{ws} ranks: kv heads split over up to 2, replicas beyond"}


def bench_kv_attention(args, ws, rank, local):
    """Fixed-shape KV-cache attention, H_q=16, H_kv=2, hd=256, ctx 4096, fp16.

    One step = one pass of the layer's attention over the workload: 31 prefill
    chunks of 64 tokens at positions 2048..4031 then 64 decode steps at
    4032..4095 (cache write fused in every call).  `--window 512` selects the
    sliding-window variant.  Ranks beyond the two kv heads are replicas."""
    from anemll_b200 import attention, inputs, shard
    dev = torch.device("cuda", local)
    d = inputs.kv_attention()
    kv0, nkv = shard.kv_head_shard(ws, rank, 2)
    hq0, nq = kv0 * 8, nkv * 8
    cache = d["cache"][:, kv0:kv0 + nkv].contiguous().to(dev)
    q = d["q"][:, hq0:hq0 + nq].contiguous().to(dev)
    k = d["k"][:, kv0:kv0 + nkv].contiguous().to(dev)
    v = d["v"][:, kv0:kv0 + nkv].contiguous().to(dev)
    gate = d["gate"].view(1, -1, 16, 256)[:, :, hq0:hq0 + nq].reshape(1, -1, nq * 256).contiguous().to(dev)
    K, V = cache[0], cache[1]
    pos0, pos1 = d["prefill_from"], d["prefill_to"]
    calls = []
    for p in range(pos0, pos1, 64):
        j = p - pos0
        calls.append((p, q[:, :, j:j + 64].contiguous(), k[:, :, j:j + 64].contiguous(), v[:, :, j:j + 64].contiguous(),
                      gate[:, j:j + 64].contiguous()))
    dec = []
    for p in range(pos1, 4096):
        j = p - pos0
        dec.append((p, q[:, :, j:j + 1].contiguous(), k[:, :, j:j + 1].contiguous(), v[:, :, j:j + 1].contiguous(),
                    gate[:, j:j + 1].contiguous()))
    outs = [torch.empty(1, c[1].shape[2], nq * 256, dtype=torch.half, device=dev) for c in calls + dec]
    ws_buf = torch.empty(attention.kv_attention_workspace_size(1, 64, nq, nkv, 256, 4096), dtype=torch.uint8,
                         device=dev)
    window = args.window

    def run(seq):
        for (p, qq, kk, vv, gg), o in seq:
            attention.kv_attention(qq, K, V, p, k_new=kk, v_new=vv, gate=gg, window=window, out=o, workspace=ws_buf)

    pre = list(zip(calls, outs[:len(calls)]))
    dcd = list(zip(dec, outs[len(calls):]))
    from anemll_b200 import _lib
    for _ in range(args.warmup):
        c0 = _lib.launch_count()
        run(pre)
        run(dcd)
        launches_pass = _lib.launch_count() - c0  # the library's kernels of one pass (counted on the host)
    torch.cuda.synchronize(dev)
    # the 31 prefill calls and the 64 decode calls replay as CUDA graphs (as a serving loop would)
    g_pre, g_dec = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_pre):
        run(pre)
    with torch.cuda.graph(g_dec):
        run(dcd)
    g_pre.replay()
    g_dec.replay()
    torch.cuda.synchronize(dev)
    barrier(ws)
    stream = torch.cuda.current_stream(dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # larger than the 126 MB L2
    pre_ms = dec_ms = 0.0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            # L2 flushed (outside the timed regions) before the prefill chunks and before the decode steps
            flush.zero_()
            e[0].record(stream)
            g_pre.replay()
            e[1].record(stream)
            flush.zero_()
            e[2].record(stream)
            g_dec.replay()
            e[3].record(stream)
            torch.cuda.synchronize(dev)
            pre_ms += e[0].elapsed_time(e[1])
            dec_ms += e[2].elapsed_time(e[3])
    barrier(ws)
    tot_ms = max_over_ranks(pre_ms + dec_ms, ws, dev)

    # End to end through the public op with host buffers: per call, one H2D copy of its packed
    # q | k_new | v_new | gate from pinned memory on a copy stream, the call on the compute stream, and
    # the D2H of its output on a third stream, so that the copies of neighbouring calls overlap the
    # kernels.  The pass, copies included, is captured once as a CUDA graph and replayed (as a
    # serving loop would).
    hbufs, dbufs, dviews = [], [], []
    for c in calls + dec:
        parts = c[1:]
        sizes = [x.numel() * x.element_size() for x in parts]
        offs, o_ = [], 0
        for sz in sizes:
            offs.append(o_)
            o_ += (sz + 255) // 256 * 256
        hb = torch.empty(o_, dtype=torch.uint8).pin_memory()
        for x, off, sz in zip(parts, offs, sizes):
            hb[off:off + sz].copy_(x.cpu().contiguous().view(-1).view(torch.uint8))
        db = torch.empty(o_, dtype=torch.uint8, device=dev)
        hbufs.append(hb)
        dbufs.append(db)
        dviews.append(tuple(db[off:off + sz].view(x.dtype).view(x.shape) for x, off, sz in zip(parts, offs, sizes)))
    houts = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
    h2d = sum(hb.numel() for hb in hbufs)
    d2h = sum(o.numel() * o.element_size() for o in houts)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    n_calls = len(calls) + len(dec)
    ev_in = [torch.cuda.Event() for _ in range(n_calls)]
    ev_k = [torch.cuda.Event() for _ in range(n_calls)]

    def e2e_pass():
        cur = torch.cuda.current_stream(dev)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        for i, ((p, *_), o, hb, db, vw, ho) in enumerate(zip(calls + dec, outs, hbufs, dbufs, dviews, houts)):
            with torch.cuda.stream(s_in):
                db.copy_(hb, non_blocking=True)
            ev_in[i].record(s_in)
            cur.wait_event(ev_in[i])
            qq, kk, vv, gg = vw
            attention.kv_attention(qq, K, V, p, k_new=kk, v_new=vv, gate=gg, window=window, out=o, workspace=ws_buf)
            ev_k[i].record(cur)
            s_out.wait_event(ev_k[i])
            with torch.cuda.stream(s_out):
                ho.copy_(o, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    e2e_pass()
    torch.cuda.synchronize(dev)
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e):
        e2e_pass()
    g_e2e.replay()
    torch.cuda.synchronize(dev)
    if not torch.equal(houts[-1].to(dev), outs[-1]):
        raise RuntimeError("e2e: the last call's output read back does not match the device copy")
    barrier(ws)
    e2e_passes = min(args.steps, 3)
    e2e_ms = 0.0
    for _ in range(e2e_passes):
        flush.zero_()
        e[0].record(stream)
        g_e2e.replay()
        e[1].record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms += e[0].elapsed_time(e[1])
    e2e_ms = max_over_ranks(e2e_ms, ws, dev)
    pre_ms_max = max_over_ranks(pre_ms, ws, dev)
    dec_ms_max = max_over_ranks(dec_ms, ws, dev)
    # algorithmic work: 4*hd*H_q FLOP per visible (query, key) pair in prefill; K+V bytes of visible keys in decode
    vis_pre = sum(min(p + i + 1, window) if window else p + i + 1 for p in range(pos0, pos1, 64) for i in range(64))
    flop_pre = 4 * 256 * nq * vis_pre
    bytes_dec = sum((min(p + 1, window) if window else p + 1) * nkv * 256 * 2 * 2 + 3 * nq * 256 * 2 + 2 * nkv * 256 * 2
                    for p in range(pos1, 4096))
    pk, how = peaks()
    tflops = flop_pre / (pre_ms / args.steps / 1e3) / 1e12
    gbs = bytes_dec / (dec_ms / args.steps / 1e3) / 1e9
    n_tok = (pos1 - pos0) + (4096 - pos1)
    return {
        "metric": "kv_attention_tokens_per_s",
        "value": n_tok * args.steps / (tot_ms / 1e3) * (1 if ws <= 2 else ws / 2),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if ws <= 2 else "strong up to 2 (kv heads), replicas beyond",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded; cache prefilled N(0,1) at 0..2047)",
        "config": kv_config(ws, window),
        "prefill_us_per_chunk": pre_ms_max / args.steps / len(calls) * 1e3,
        "decode_us_per_step": dec_ms_max / args.steps / len(dec) * 1e3,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / pk["bf16_tflops"], "peak_source": how,
                     "algorithmic_flop_per_pass": flop_pre, "traffic": None,
                     "decode": {"bound": "hbm", "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"],
                                "algorithmic_bytes_per_pass": bytes_dec,
                                # ncu DRAM bytes of one causal decode-step launch (position 4032)
                                "traffic_per_step": traffic_from_profiles("kv_decode_step") if not window else None}},
        "e2e": {"value": n_tok * e2e_passes / (e2e_ms / 1e3) * (1 if ws <= 2 else ws / 2), "unit": "tokens/s",
                "passes": e2e_passes, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "form": "per call one H2D copy of its packed inputs (copy stream), the public op, the output's "
                        "D2H (third stream); the pass captured once as a CUDA graph and replayed"},
        "gpu_launches": args.steps * launches_pass,
        "clocks": clk.summary(),
    }


# ------------------------------------------------------------- GDN layer ----
LAYER_PREFILL, LAYER_DECODE, HIDDEN = 512, 64, 2048


def layer_config(ws):
    return {"workload": "gdn_layer", "batch_per_gpu": 1, "prefill": LAYER_PREFILL, "decode_steps": LAYER_DECODE,
            "hidden": HIDDEN, "H_qk": H_QK, "H_v": H_V, "d_k": DK, "d_v": DV, "chunk": CHUNK,
            "l2": "flushed (256 MB write) before the prefill and before the decode steps of every timed pass",
            "parallelism": f"weak, {ws} independent sequences"}


CACHE_NL, CACHE_H, CACHE_SW, CACHE_HD = 18, 1, 512, 256


def cache_ops_config(ws):
    return {"workload": "kv_cache_ops", "local_layers": CACHE_NL, "window": CACHE_SW, "H_kv": CACHE_H,
            "head_dim": CACHE_HD, "mask_tokens": 64, "resize": "36x1x1024x256 -> 4096 rows, position 1000",
            "calls_per_step": 4 * CACHE_NL + 1,
            "l2": "flushed (256 MB write) before every timed step",
            "parallelism": f"weak, {ws} replicas"}


def stack_config(ws, seqs=None, prefill=None, decode=None):
    from anemll_b200.stack import StackConfig
    cfg = StackConfig()
    seqs = STACK_B if seqs is None else seqs
    prefill = STACK_PREFILL if prefill is None else prefill
    decode = STACK_DECODE if decode is None else decode
    n_att = sum(cfg.is_attention(i) for i in range(cfg.n_layers))
    return {"workload": "hybrid_stack", "sequences": seqs, "sequences_per_gpu": seqs // ws,
            "prefill": prefill, "decode_steps": decode, "layers": cfg.n_layers,
            "attention_layers": n_att, "hidden": cfg.hidden, "ffn": cfg.ffn, "vocab": cfg.vocab,
            "ctx": cfg.ctx, "gdn": f"H_qk {cfg.H_qk}, H_v {cfg.H_v}, d {cfg.d_k}",
            "attention": f"H_q {cfg.H_q}, H_kv {cfg.H_kv}, hd {cfg.head_dim}",
            "l2": "flushed (256 MB write) before every timed pass; weights and states exceed L2",
            "parallelism": f"sequences split over {ws} GPUs, NCCL all-gather of next-token ids"}
LAYER_PROJ = 2 * H_QK * DK + 2 * H_V * DV + 2 * H_V  # in_proj_qkv | in_proj_z | in_proj_b | in_proj_a rows


def layer_flop_per_token():
    return 2 * HIDDEN * LAYER_PROJ + 2 * H_V * DV * HIDDEN + H_V * PREFILL_FLOP_PER_TOKEN_HEAD


def layer_decode_bytes():
    return 2 * (HIDDEN * LAYER_PROJ + H_V * DV * HIDDEN) + 2 * H_V * DK * DV * 4  # bf16 weights, state r+w


def _load_layer(layer, w):
    with torch.no_grad():
        for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            getattr(layer, n).weight.copy_(w[n])
        layer.conv_weight.copy_(w["conv_w"])
        layer.A_log.copy_(w["A_log"])
        layer.dt_bias.copy_(w["dt_bias"])
        layer.norm_weight.copy_(w["norm_w"])


def bench_gdn_layer(args, ws, rank, local):
    """One Qwen3.5 gated delta-rule layer through the drop-in module.

    B=1 per rank, a 512-token prefill then 64 decode steps, hidden 2048, bf16,
    random-init weights.  The input/output projections are torch GEMMs.  The
    core runs the library's kernels: prologue, chunked prefill or recurrent
    decode, gated RMSNorm.  One step = one pass (prefill + 64 decode steps),
    replayed as two CUDA graphs.  Weak scaling: every rank runs its own
    sequence."""
    from anemll_b200 import gdn, inputs
    dev = torch.device("cuda", local)
    w, hidden = inputs.gdn_layer(seed=1000 * rank)
    layer = gdn.GatedDeltaNet(dtype=torch.bfloat16, device=dev)
    _load_layer(layer, w)
    conv, rec = layer.new_states(1)
    h = hidden.to(dev)
    x_pre = h[:, :LAYER_PREFILL].contiguous()
    x_dec = [h[:, LAYER_PREFILL + i:LAYER_PREFILL + i + 1].contiguous() for i in range(LAYER_DECODE)]

    def run_pre():
        return layer(x_pre, 0, conv, rec)

    def run_dec():
        return [layer(x, LAYER_PREFILL + i, conv, rec) for i, x in enumerate(x_dec)]

    from anemll_b200 import _lib
    with torch.no_grad():
        for _ in range(args.warmup):
            c0 = _lib.launch_count()
            run_pre()
            run_dec()
            launches_pass = _lib.launch_count() - c0  # the library's kernels of one pass (counted on the host)
        torch.cuda.synchronize(dev)
        g_pre, g_dec = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_pre):
            y_pre = run_pre()
        with torch.cuda.graph(g_dec):
            y_dec = run_dec()
        g_pre.replay()
        g_dec.replay()
        torch.cuda.synchronize(dev)
    barrier(ws)
    stream = torch.cuda.current_stream(dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # larger than the 126 MB L2
    pre_ms = dec_ms = 0.0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            flush.zero_()  # outside the timed regions
            e[0].record(stream)
            g_pre.replay()
            e[1].record(stream)
            flush.zero_()
            e[2].record(stream)
            g_dec.replay()
            e[3].record(stream)
            torch.cuda.synchronize(dev)
            pre_ms += e[0].elapsed_time(e[1])
            dec_ms += e[2].elapsed_time(e[3])
    barrier(ws)
    if gdn.chunked_device_error(reset=True):
        raise RuntimeError("chunked prefill reported a device-side wait timeout")
    tot_ms = max_over_ranks(pre_ms + dec_ms, ws, dev)

    # End to end through the module with host buffers: the prompt's hidden states and then each decode
    # token's come from pinned memory by H2D copies on a copy stream, each call's output goes back by a
    # D2H copy on a third stream, so that the copies overlap the neighbouring calls; the pass (copies
    # included) is captured once as a CUDA graph and replayed, as a serving loop would run it.
    hx = hidden.pin_memory()
    hy = torch.empty(1, LAYER_PREFILL + LAYER_DECODE, HIDDEN, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty_like(h)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    spans = [(0, LAYER_PREFILL)] + [(LAYER_PREFILL + i, LAYER_PREFILL + i + 1) for i in range(LAYER_DECODE)]
    ev_in = [torch.cuda.Event() for _ in spans]
    ev_k = [torch.cuda.Event() for _ in spans]

    def e2e_pass():
        cur = torch.cuda.current_stream(dev)
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)
        for i, (a, b_) in enumerate(spans):
            with torch.cuda.stream(s_in):
                dx[:, a:b_].copy_(hx[:, a:b_], non_blocking=True)
            ev_in[i].record(s_in)
            cur.wait_event(ev_in[i])
            y = layer(dx[:, a:b_], a, conv, rec)
            ev_k[i].record(cur)
            s_out.wait_event(ev_k[i])
            with torch.cuda.stream(s_out):
                hy[:, a:b_].copy_(y, non_blocking=True)
        cur.wait_stream(s_in)
        cur.wait_stream(s_out)

    with torch.no_grad():
        e2e_pass()
        torch.cuda.synchronize(dev)
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e):
            e2e_pass()
        g_e2e.replay()
        torch.cuda.synchronize(dev)
        e2e_passes = min(args.steps, 3)
        e2e_ms = 0.0
        for _ in range(e2e_passes):
            flush.zero_()
            e[0].record(stream)
            g_e2e.replay()
            e[1].record(stream)
            torch.cuda.synchronize(dev)
            e2e_ms += e[0].elapsed_time(e[1])
        if not torch.isfinite(hy.float()).all():
            raise RuntimeError("e2e: non-finite layer output read back")
    e2e_ms = max_over_ranks(e2e_ms, ws, dev)
    n_tok = LAYER_PREFILL + LAYER_DECODE
    pk, how = peaks()
    tflops = LAYER_PREFILL * layer_flop_per_token() / (pre_ms / args.steps / 1e3) / 1e12
    gbs = layer_decode_bytes() * LAYER_DECODE / (dec_ms / args.steps / 1e3) / 1e9
    return {
        "metric": "gdn_layer_tokens_per_s",
        "value": ws * n_tok * args.steps / (tot_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations and weights, f32 state",
        "data": "synthetic (seeded; hidden ~N(0,1), weights ~N(0,0.02), conv ~N(0,0.1), A_log ~U(0, log 16))",
        "config": layer_config(ws),
        "prefill_ms": pre_ms / args.steps,
        "decode_us_per_step": dec_ms / args.steps / LAYER_DECODE * 1e3,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / pk["bf16_tflops"], "peak_source": how,
                     "algorithmic_flop_per_prefill": LAYER_PREFILL * layer_flop_per_token(), "traffic": None,
                     "decode": {"bound": "hbm", "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"],
                                "algorithmic_bytes_per_step": layer_decode_bytes()}},
        "e2e": {"value": ws * n_tok * e2e_passes / (e2e_ms / 1e3), "unit": "tokens/s", "passes": e2e_passes,
                "h2d_bytes_per_step": hx.numel() * hx.element_size(),
                "d2h_bytes_per_step": hy.numel() * hy.element_size(),
                "form": "per call the H2D of its hidden states (copy stream), the module, the D2H of its output "
                        "(third stream); the pass captured once as a CUDA graph and replayed"},
        "gpu_launches": args.steps * launches_pass,
        "clocks": clk.summary(),
    }


# ------------------------------------------------------------- cache ops ----
def bench_cache_ops(args, ws, rank, local):
    """Cache-management ops on a Gemma3-style split cache (HBM-bound copies).

    One step = one decode-step's rotating update of all 18 local layers (window 512, 1 kv head,
    hd 256, fp16; key and value slots, one call per layer), one 64-token update-mask write into
    every local layer, and one resize of a 36-layer state [36, 1, 1024, 256] to 4096 rows
    (current position 1000).  Calls replay as one CUDA graph; L2 flushed between steps.
    Weak scaling (replicas)."""
    from anemll_b200 import _lib as lib, cache_ops
    dev = torch.device("cuda", local)
    g = torch.Generator().manual_seed(6 + rank)
    nl, H, sw, hd = CACHE_NL, CACHE_H, CACHE_SW, CACHE_HD
    kv = torch.randn(2 * nl, H, sw, hd, generator=g).half().to(dev)
    key = torch.randn(1, H, 1, hd, generator=g).half().to(dev)
    val = torch.randn(1, H, 1, hd, generator=g).half().to(dev)
    new = torch.randn(2, H, 64, hd, generator=g).half().to(dev)
    mask = torch.zeros(1, 1, sw, 64, dtype=torch.half)
    for t in range(64):
        mask[0, 0, 200 + t, t] = 1
    mask = mask.to(dev)
    st = torch.randn(36, 1, 1024, 256, generator=g).half().to(dev)
    out = torch.empty(36, 1, 4096, 256, dtype=torch.half, device=dev)

    def step():
        for i in range(nl):
            cache_ops.update_kv_local_(kv, i, nl, key, val, 1)
        for i in range(nl):
            cache_ops.apply_update_mask_(kv[i:i + 1], new[0:1], mask)
            cache_ops.apply_update_mask_(kv[i + nl:i + nl + 1], new[1:2], mask)
        rc = lib.load().anemll_kv_state_transition(lib.ptr(st), lib.F16, lib.ptr(out), lib.F16, 36, 1024, 4096, 256,
                                                   1000, 0.0, lib.stream_ptr(dev))
        lib.check(rc, "anemll_kv_state_transition")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize(dev)
    barrier(ws)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ms = 0.0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            flush.zero_()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms += e0.elapsed_time(e1)
    barrier(ws)
    ms_max = max_over_ranks(ms, ws, dev)

    # end to end through the public ops: the step's new rows (key, value, the 64-token chunk) and
    # the mask copied in from pinned host memory, the calls (eager), and the rows the step wrote into
    # the local cache (its newest row and the mask-written rows of every slot) read back
    h_in = [t.cpu().pin_memory() for t in (key, val, new, mask)]
    d_in = (key, val, new, mask)
    h_out = torch.empty(2 * nl, H, 65, hd, dtype=torch.half).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step():
        for d, h in zip(d_in, h_in):
            d.copy_(h, non_blocking=True)
        step()
        h_out[:, :, :64].copy_(kv[:, :, 200:264], non_blocking=True)
        h_out[:, :, 64:].copy_(kv[:, :, sw - 1:], non_blocking=True)

    e2e_step()
    torch.cuda.synchronize(dev)
    e2e_steps = min(args.steps, 50)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws, dev)
    es = 2
    b_rot = nl * 2 * H * 2 * sw * hd * es            # every slot read and written once
    b_mask = nl * 2 * H * 3 * 64 * hd * es            # new rows read, touched rows read and written
    b_tr = 36 * (1000 * 256 + 4096 * 256) * es        # valid rows read, the whole target written
    bytes_step = b_rot + b_mask + b_tr
    pk, how = peaks()
    gbs = bytes_step / (ms / args.steps / 1e3) / 1e9
    return {
        "metric": "kv_cache_ops_bytes_per_s",
        "value": ws * bytes_step * args.steps / (ms_max / 1e3) / 1e9,
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded N(0,1))",
        "config": cache_ops_config(ws),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / pk["hbm_gbs"], "peak_source": how, "algorithmic_bytes_per_step": bytes_step,
                     "traffic": None,
                     "bytes": {"rotate": b_rot, "update_mask": b_mask, "transition": b_tr}},
        "e2e": {"value": ws * bytes_step * e2e_steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s", "steps": e2e_steps,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (2 * nl + 2 * nl + 1),
        "clocks": clk.summary(),
    }


# ------------------------------------------------------------- hybrid stack --
STACK_B, STACK_PREFILL, STACK_DECODE, STACK_SEED = 128, 1024, 256, 4


def stack_linear_params(cfg):
    """Weights one token's pass multiplies (every layer's projections and MLP; LM head separate)."""
    gdn = cfg.hidden * (2 * cfg.H_qk * cfg.d_k + 2 * cfg.H_v * cfg.d_v + 2 * cfg.H_v) + cfg.H_v * cfg.d_v * cfg.hidden
    att = cfg.hidden * (2 * cfg.H_q * cfg.head_dim + 2 * cfg.H_kv * cfg.head_dim) + cfg.H_q * cfg.head_dim * cfg.hidden
    mlp = 3 * cfg.hidden * cfg.ffn
    n_att = sum(cfg.is_attention(i) for i in range(cfg.n_layers))
    return (cfg.n_layers - n_att) * gdn + n_att * att + cfg.n_layers * mlp, n_att


def stack_prefill_flop(cfg, B, T):
    """Algorithmic FLOPs of the prefill: projections/MLP per token, the GDN core per token and head,
    causal attention (4*hd per visible key per query head), the LM head once per sequence."""
    lin, n_att = stack_linear_params(cfg)
    n_gdn = cfg.n_layers - n_att
    attn = n_att * 4 * cfg.head_dim * cfg.H_q * (T * (T + 1) // 2)
    return B * (T * (2 * lin + n_gdn * cfg.H_v * PREFILL_FLOP_PER_TOKEN_HEAD) + attn + 2 * cfg.hidden * cfg.vocab)


def stack_decode_bytes(cfg, B, pos):
    """Algorithmic HBM bytes of one decode step at position ``pos``: bf16 weights (LM head included)
    once, every GDN layer's f32 state read and written, every attention layer's K and V rows [0, pos]
    read and row pos written, conv states read and written."""
    lin, n_att = stack_linear_params(cfg)
    n_gdn = cfg.n_layers - n_att
    conv_dim = 2 * cfg.H_qk * cfg.d_k + cfg.H_v * cfg.d_v
    w = 2 * (lin + cfg.hidden * cfg.vocab)
    st = n_gdn * B * (2 * cfg.H_v * cfg.d_k * cfg.d_v * 4 + 2 * conv_dim * 4 * 2)
    kv = n_att * B * 2 * cfg.H_kv * (pos + 2) * cfg.head_dim * 2
    return w + st + kv


def bench_stack(args, ws, rank, local):
    """The hybrid decoder stack end to end: 24 layers (18 gated-DeltaNet, 6 gated full attention),
    hidden 2048, SwiGLU 6144, vocab 151936, bf16, random N(0, 0.02) weights (seed 4).  Job: 128
    sequences of 1024 uniform random prompt tokens, prefill, then 256 greedy decode steps.  The
    sequences are split evenly over the ranks; after every step the ranks all-gather the next-token
    ids (NCCL).  One step = one whole pass (prefill + 256 decode steps); the decode steps replay one
    CUDA graph per position.  Strong scaling (the job is fixed)."""
    from anemll_b200 import gdn
    from anemll_b200.stack import GreedyDecoder, HybridStack, StackConfig, nccl_id_gather, shard
    dev = torch.device("cuda", local)
    cfg = StackConfig()
    # the job (128 x (1024 + 256)) unless a smaller profiling case is asked for
    STACK_B, STACK_PREFILL, STACK_DECODE = args.stack_seqs, args.stack_prefill, args.stack_decode
    model = HybridStack(cfg, device=dev).init_weights(STACK_SEED)
    g = torch.Generator().manual_seed(STACK_SEED)
    prompt_job = torch.randint(0, cfg.vocab, (STACK_B, STACK_PREFILL), generator=g)
    lo, hi = shard(STACK_B, rank, ws)
    B = hi - lo
    prompt = prompt_job[lo:hi].to(dev)
    gather = nccl_id_gather() if ws > 1 else None
    dec = GreedyDecoder(model, B, graphs=True)
    for _ in range(args.warmup):  # the first pass runs every position eagerly and captures its graph
        dec(prompt, STACK_DECODE, gather)
    torch.cuda.synchronize(dev)
    barrier(ws)
    stream = torch.cuda.current_stream(dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pre_ms = dec_ms = 0.0
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            flush.zero_()  # outside the timed region
            e[0].record(stream)
            first = dec.prefill(prompt)
            if gather:
                gather(first)
            e[1].record(stream)
            dec.decode(STACK_PREFILL, STACK_DECODE, gather)
            e[2].record(stream)
            torch.cuda.synchronize(dev)
            pre_ms += e[0].elapsed_time(e[1])
            dec_ms += e[1].elapsed_time(e[2])
    barrier(ws)
    if gdn.chunked_device_error(reset=True):
        raise RuntimeError("chunked prefill reported a device-side wait timeout")
    tot_ms = max_over_ranks(pre_ms + dec_ms, ws, dev)
    pre_max = max_over_ranks(pre_ms, ws, dev)
    dec_max = max_over_ranks(dec_ms, ws, dev)

    # end to end through the decoder: the prompt shard copied in from pinned host memory, the job's
    # generated ids copied back, inside the timed region
    h_prompt = prompt_job[lo:hi].clone().pin_memory()
    h_out = torch.empty(STACK_B if gather else B, STACK_DECODE + 1, dtype=torch.long).pin_memory()
    d_prompt = torch.empty_like(prompt)
    e2e_passes = min(args.steps, 2)
    e2e_ms = 0.0
    for _ in range(e2e_passes):
        flush.zero_()
        e[0].record(stream)
        d_prompt.copy_(h_prompt, non_blocking=True)
        ids = dec(d_prompt, STACK_DECODE, gather)
        h_out.copy_(ids, non_blocking=True)
        e[1].record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms += e[0].elapsed_time(e[1])
    e2e_ms = max_over_ranks(e2e_ms, ws, dev)

    n_tok = STACK_B * (STACK_PREFILL + STACK_DECODE)
    pk, how = peaks()
    # the prefill is a long run of back-to-back GEMMs under the power cap: the sustained bf16 figure
    tc_peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    flop = stack_prefill_flop(cfg, B, STACK_PREFILL)
    tflops = flop / (pre_ms / args.steps / 1e3) / 1e12
    dbytes = sum(stack_decode_bytes(cfg, B, STACK_PREFILL + s) for s in range(STACK_DECODE))
    gbs = dbytes / (dec_ms / args.steps / 1e3) / 1e9
    n_att = sum(cfg.is_attention(i) for i in range(cfg.n_layers))
    return {
        "metric": "stack_tokens_per_s",
        "value": n_tok * args.steps / (tot_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 activations and weights, f32 GDN states",
        "data": "synthetic (uniform random prompt ids, seed 4; weights ~N(0,0.02), conv ~N(0,0.1), "
                "A_log ~U(0, log 16))",
        "config": stack_config(ws, STACK_B, STACK_PREFILL, STACK_DECODE),
        "prefill_tokens_per_s": STACK_B * STACK_PREFILL * args.steps / (pre_max / 1e3),
        "decode_steps_per_s": STACK_DECODE * args.steps / (dec_max / 1e3),
        "prefill_ms": pre_max / args.steps,
        "decode_ms_per_step": dec_max / args.steps / STACK_DECODE,
        "roofline": {"bound": "tensor", "phase": "prefill", "achieved": tflops, "peak": tc_peak,
                     "unit": "TFLOP/s", "frac": tflops / tc_peak,
                     "peak_source": how + (" (sustained)" if "bf16_tflops_sustained" in pk else " (burst)"),
                     "algorithmic_flop_per_prefill": flop, "traffic": None,
                     "decode": {"bound": "hbm", "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"],
                                "algorithmic_bytes_per_pass": dbytes}},
        "e2e": {"value": n_tok * e2e_passes / (e2e_ms / 1e3), "unit": "tokens/s", "passes": e2e_passes,
                "h2d_bytes_per_step": h_prompt.numel() * h_prompt.element_size(),
                "d2h_bytes_per_step": h_out.numel() * h_out.element_size()},
        "gpu_launches": args.steps * (dec.launches["prefill"] +
                                      sum(dec.launches[STACK_PREFILL + s] for s in range(STACK_DECODE))),
        "clocks": clk.summary(),
    }


# ------------------------------------------------------------ CPU samples ---
def cpu_prefill_sample(threads, T=2048):
    """Oracle chunked prefill of one sequence x T tokens x 32 heads on the host; returns tokens/s."""
    from anemll_b200 import inputs
    from oracle import gdn as og
    torch.set_num_threads(threads)
    w = inputs.gdn_prefill_device(B=1, T=T, device="cpu")
    xs = [w[n].float() for n in ("q", "k", "v", "g", "beta")]
    S0 = torch.zeros(1, H_V, DK, DV)
    og.chunk_gated_delta_rule(*(x[:, :128] for x in xs), CHUNK, S0)
    t0 = time.perf_counter()
    og.chunk_gated_delta_rule(*xs, CHUNK, S0)
    return T / (time.perf_counter() - t0), f"1 sequence x {T} tokens x {H_V} heads of the fp32 torch CPU oracle"


def cpu_kv_sample(threads, window, n_chunks=4, n_dec=8):
    """Oracle KV attention calls (H_q 16, H_kv 2, hd 256, ctx 4096) on the host; returns tokens/s."""
    from anemll_b200 import inputs
    from oracle import kv_attention as ok
    torch.set_num_threads(threads)
    d = inputs.kv_attention()
    cache = d["cache"].float().clone()
    pos0 = d["prefill_from"]
    calls = [(pos0 + 64 * i, 64) for i in range(n_chunks)] + [(d["prefill_to"] + i, 1) for i in range(n_dec)]
    ntok = sum(n for _, n in calls)
    t0 = time.perf_counter()
    for p, n in calls:
        j = p - pos0
        ok.kv_attention_step(d["q"][:, :, j:j + n], d["k"][:, :, j:j + n], d["v"][:, :, j:j + n],
                             d["gate"][:, j:j + n], cache, 0, 1, p, window)
    return ntok / (time.perf_counter() - t0), (f"{n_chunks} prefill chunks of 64 and {n_dec} decode steps of the "
                                                "fp32 torch CPU oracle (the reference's own algorithm in fp32)")


CPU_CACHE_NL, CPU_CACHE_H, CPU_CACHE_SW, CPU_CACHE_HD = 18, 1, 512, 256
# bytes of one step of the CPU cache-op sample (the rotations, the mask writes and one state transition)
CPU_CACHE_STEP_BYTES = (CPU_CACHE_NL * 2 * CPU_CACHE_H * 2 * CPU_CACHE_SW * CPU_CACHE_HD * 2
                        + CPU_CACHE_NL * 2 * CPU_CACHE_H * 3 * 64 * CPU_CACHE_HD * 2 + 36 * (1000 * 256 + 4096 * 256) * 2)


def cpu_cache_ops_sample(threads):
    """The same cache-op step with the oracle's torch ops on the host cores; returns GB/s."""
    from oracle import cache_ops as oc
    torch.set_num_threads(threads)
    nl, H, sw, hd = CPU_CACHE_NL, CPU_CACHE_H, CPU_CACHE_SW, CPU_CACHE_HD
    kv = torch.randn(2 * nl, H, sw, hd).half()
    key = torch.randn(1, H, 1, hd).half()
    new = torch.randn(1, H, 64, hd).half()
    mask = torch.zeros(sw, 64)
    for t in range(64):
        mask[200 + t, t] = 1
    st = torch.randn(36, 1, 1024, 256).half()
    t0 = time.perf_counter()
    for i in range(2 * nl):
        kv[i:i + 1] = oc.rotate_append(kv[i:i + 1], key, 1)
    for i in range(2 * nl):
        kv[i:i + 1] = oc.update_mask_write(kv[i:i + 1], new, mask).half()
    oc.transition_state(st, 4096, 1000)
    dt = time.perf_counter() - t0
    return CPU_CACHE_STEP_BYTES / dt / 1e9, "one step of the same cache ops with the oracle's torch CPU ops"


def cpu_layer_sample(threads, n_dec=8):
    """Oracle GDN layer (torch projections + oracle core) on the host: 512-token prefill and n_dec steps."""
    from anemll_b200 import inputs
    from oracle import gdn as og
    import torch.nn.functional as F
    torch.set_num_threads(threads)
    w, hidden = inputs.gdn_layer()
    W = {n: w[n].float() for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")}
    params = dict(conv_w=w["conv_w"], A_log=w["A_log"], dt_bias=w["dt_bias"], norm_w=w["norm_w"])
    x = hidden.float()

    def proj(xx):
        return (F.linear(xx, W["in_proj_qkv"]), F.linear(xx, W["in_proj_z"]), F.linear(xx, W["in_proj_a"]),
                F.linear(xx, W["in_proj_b"]))

    t0 = time.perf_counter()
    m, z, a, b = proj(x[:, :LAYER_PREFILL])
    _, normed, conv, S = og.gdn_layer_prefill(m, z, a, b, params, H_QK, H_V, DK, DV)
    F.linear(normed.reshape(1, LAYER_PREFILL, -1), W["out_proj"])
    for i in range(n_dec):
        m, z, a, b = proj(x[:, LAYER_PREFILL + i:LAYER_PREFILL + i + 1])
        _, normed, conv, S = og.gdn_layer_decode(m, z, a, b, params, H_QK, H_V, DK, DV, conv, S)
        F.linear(normed.reshape(1, 1, -1), W["out_proj"])
    dt = time.perf_counter() - t0
    return (LAYER_PREFILL + n_dec) / dt, (f"one layer: 512-token prefill and {n_dec} decode steps, torch fp32 "
                                          "projections with the CPU oracle core")


def cpu_stack_sample(threads, T=64, n_dec=2):
    """The stack's layers restated by the CPU oracle (fp32 GEMMs, the oracle's GDN core and attention over
    the 4096-row cache) for one sequence: a T-token prefill and n_dec greedy steps through all 24
    layers, the final norm and the LM head; returns tokens/s.  The weights are fp32 copies of a
    random block tiled over each parameter (the values do not change the timing)."""
    from anemll_b200.stack import StackConfig
    from oracle import stack as ost
    torch.set_num_threads(threads)
    cfg = StackConfig()
    model = _CPU_STACK.get("model")
    if model is None:
        model = _CPU_STACK["model"] = _cpu_stack_model(cfg)
    state = ost.new_state(model, 1)
    ids = torch.randint(0, cfg.vocab, (1, T), generator=torch.Generator().manual_seed(STACK_SEED))
    t0 = time.perf_counter()
    pos, x_ids = 0, ids
    for _ in range(1 + n_dec):
        x = ost.bf(model.embed.weight[x_ids])
        for i in range(cfg.n_layers):
            x = ost.layer(model, i, x, state[i], pos)
        logits = torch.nn.functional.linear(ost.rms_norm(x[:, -1], model.norm, cfg.eps), model.lm_head.weight)
        pos += x_ids.shape[1]
        x_ids = logits.argmax(-1, keepdim=True)
    dt = time.perf_counter() - t0
    return (T + n_dec) / dt, (f"1 sequence: a {T}-token prefill and {n_dec} greedy steps through the 24 layers, "
                              "fp32 torch GEMMs with the CPU oracle's GDN core and attention")


_CPU_STACK = {}  # the host model of the CPU samples, built once per process


def _cpu_stack_model(cfg):
    """The stack's shapes on the host in fp32, weights a random block tiled over each parameter."""
    from anemll_b200.stack import HybridStack, rope_tables
    model = HybridStack(cfg, device="meta", dtype=torch.float32).to_empty(device="cpu")
    model.cos, model.sin = rope_tables(cfg.head_dim, cfg.ctx, cfg.rope_theta, "cpu")
    base = torch.randn(1 << 20, generator=torch.Generator().manual_seed(STACK_SEED)) * 0.02
    with torch.no_grad():
        for name, p in model.named_parameters():
            flat = p.view(-1)
            if "norm" in name and p.dim() == 1:
                p.fill_(1.0)
            elif name.endswith("A_log") or name.endswith("dt_bias"):
                p.fill_(0.5)
            else:
                for i in range(0, flat.numel(), base.numel()):
                    n = min(base.numel(), flat.numel() - i)
                    flat[i:i + n].copy_(base[:n] * (5.0 if name.endswith("conv_weight") else 1.0))
    return model


def dram_frac(traffic, per_launch_s, peak_gbs):
    """Measured DRAM bytes of one launch over its device time, as a fraction of the HBM peak (None
    without a capture)."""
    return None if traffic is None else traffic / per_launch_s / 1e9 / peak_gbs


def traffic_from_profiles(name):
    """Per-launch DRAM bytes recorded from an ncu capture, if a summary is committed."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")  # "<workload> <bytes per launch>" lines
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 2 and parts[0] == name:
                    return int(parts[1])
    except (OSError, ValueError):
        pass
    return None


SUB_KEYS = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "scaling", "dtype", "config", "roofline",
            "e2e", "gpu_launches", "clocks", "cpu_baseline", "prefill_us_per_chunk", "decode_us_per_step")


def sub_args(args, steps, warmup):
    """The argument set of a secondary line of the default run: its own step counts, capped by the run's."""
    a = argparse.Namespace(**vars(args))
    a.steps = max(3, min(args.steps, steps))
    a.warmup = max(3, min(args.warmup, warmup))
    return a


def cpu_line(config, threads, window=0, steps=3):
    """The CPU oracle port of one config on the host cores: (value, unit, ms per step, sample)."""
    vals = []
    for _ in range(max(1, min(steps, 3))):
        if config == "gdn_prefill":
            v1, sample = cpu_prefill_sample(threads)
        elif config == "kv_attention":
            v1, sample = cpu_kv_sample(threads, window)
        elif config == "cache_ops":
            v1, sample = cpu_cache_ops_sample(threads)
        elif config == "stack":
            v1, sample = cpu_stack_sample(threads)
        else:
            v1, sample = cpu_layer_sample(threads)
        vals.append(v1)
    if config == "cache_ops":
        v, unit = max(vals), "GB/s"
        ms = CPU_CACHE_STEP_BYTES / (v * 1e9) * 1e3  # one step = one sample
    else:
        sample_tokens = {"gdn_prefill": 2048, "kv_attention": 4 * 64 + 8, "gdn_layer": LAYER_PREFILL + 8,
                         "stack": 66}[config]
        v, unit = max(vals), "tokens/s"
        ms = sample_tokens / v * 1e3  # one step = one bounded sample
    return v, unit, ms, sample + f", best of {len(vals)}"


def cpu_decode_line(threads, steps, warmup):
    from anemll_b200 import inputs
    from oracle import gdn as og
    w = inputs.gdn_decode(B=DECODE_B, steps=DECODE_STEPS)
    S = w["state"]
    for i in range(warmup):
        t = i % DECODE_STEPS
        _, S = og.recurrent_gated_delta_rule(w["q"][t], w["k"][t], w["v"][t], w["g"][t], w["beta"][t], S)
    t0 = time.perf_counter()
    for i in range(steps):
        t = i % DECODE_STEPS
        _, S = og.recurrent_gated_delta_rule(w["q"][t], w["k"][t], w["v"][t], w["g"][t], w["beta"][t], S)
    dt = time.perf_counter() - t0
    return steps / dt, "steps/s", dt * 1e3 / steps, f"{steps} full-batch decode steps of the fp32 torch CPU oracle"


METRICS = {"gdn_decode": "gdn_decode_steps_per_s", "gdn_prefill": "gdn_prefill_tokens_per_s",
           "kv_attention": "kv_attention_tokens_per_s", "gdn_layer": "gdn_layer_tokens_per_s",
           "cache_ops": "kv_cache_ops_bytes_per_s", "stack": "stack_tokens_per_s"}


def reference_config(config, ws, window):
    if config == "gdn_decode":
        return decode_config(ws)
    if config == "gdn_prefill":
        return prefill_config(ws)
    if config == "kv_attention":
        return kv_config(ws, window)
    if config == "gdn_layer":
        return layer_config(ws)
    if config == "cache_ops":
        return cache_ops_config(ws)
    return stack_config(ws)


def reference_line(config, args, ws, threads, window=0):
    if config == "gdn_decode":
        v, unit, ms, sample = cpu_decode_line(threads, args.steps, args.warmup)
    else:
        v, unit, ms, sample = cpu_line(config, threads, window, args.steps)
    return {
        "impl": "reference",
        "metric": METRICS[config],
        "value": v,
        "unit": unit,
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak" if config in ("gdn_decode", "gdn_layer", "cache_ops") else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": reference_config(config, ws, window),
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def reference_arm(args, ws, rank):
    """The CPU path (the oracle port: the reference has no implementation of this path) on the host cores,
    on the same config, metric and unit as our arm; rank 0 only.  The default run also times the chunked
    prefill and the KV attention (causal and windowed) samples, as secondary lines."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    res = reference_line(args.config, args, ws, threads, args.window)
    if args.default_run:
        for key, cfg, window in SECONDARY:
            sub = reference_line(cfg, sub_args(args, 3, 3), ws, threads, window)
            res[key] = {k: sub[k] for k in SUB_KEYS if k in sub}
    return res


# the secondary lines of the default run: (key, config, window, steps, warmup)
SECONDARY = (("prefill", "gdn_prefill", 0), ("kv_attention", "kv_attention", 0),
             ("kv_attention_window", "kv_attention", 512), ("layer", "gdn_layer", 0), ("stack", "stack", 0))
SECONDARY_STEPS = {"gdn_prefill": (20, 5), "kv_attention": (50, 5), "gdn_layer": (50, 5), "stack": (3, 3)}


def cpu_baseline_for(config, args, threads, window=0):
    if config == "gdn_decode":
        v = cpu_decode_sample(args.cpu_baseline_steps, threads)
        return {"value": v, "unit": "steps/s", "cores": threads, "kind": "port",
                "sample": f"{args.cpu_baseline_steps} full-batch (B=64) decode steps of the fp32 torch CPU oracle"}
    if config == "cache_ops":
        v, sample = cpu_cache_ops_sample(threads)
        return {"value": v, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}
    v, sample = {"gdn_prefill": lambda: cpu_prefill_sample(threads),
                 "kv_attention": lambda: cpu_kv_sample(threads, window),
                 "gdn_layer": lambda: cpu_layer_sample(threads),
                 "stack": lambda: cpu_stack_sample(threads)}[config]()
    return {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}


def run_ours(config, args, ws, rank, local):
    fn = {"kv_attention": bench_kv_attention, "gdn_prefill": bench_gdn_prefill, "gdn_layer": bench_gdn_layer,
          "cache_ops": bench_cache_ops, "stack": bench_stack, "gdn_decode": bench_gdn_decode}[config]
    res = fn(args, ws, rank, local)
    if rank == 0:
        res["cpu_baseline"] = None
        if ws == 1:  # the host sample runs at N=1 only
            res["cpu_baseline"] = cpu_baseline_for(config, args, os.cpu_count() or 1, args.window)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="default 2560 (stack: 3)")
    ap.add_argument("--warmup", type=int, default=None, help="default 32 (stack: 3)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None,
                    choices=["gdn_decode", "gdn_prefill", "kv_attention", "gdn_layer", "cache_ops", "stack"],
                    help="one workload's line alone; without it: the decode line carrying the prefill and KV "
                         "attention lines")
    ap.add_argument("--window", type=int, default=0, help="kv_attention: sliding window (0 = causal)")
    ap.add_argument("--cpu-baseline-steps", type=int, default=8)
    ap.add_argument("--prefill-seqs", type=int, default=PREFILL_B, help="gdn_prefill: sequences (profiling cases)")
    ap.add_argument("--prefill-len", type=int, default=PREFILL_T, help="gdn_prefill: tokens per sequence")
    ap.add_argument("--stack-seqs", type=int, default=STACK_B, help="stack: sequences (profiling cases)")
    ap.add_argument("--stack-prefill", type=int, default=STACK_PREFILL, help="stack: prompt tokens")
    ap.add_argument("--stack-decode", type=int, default=STACK_DECODE, help="stack: greedy decode steps")
    args = ap.parse_args()
    args.default_run = args.config is None
    if args.default_run:
        args.config = "gdn_decode"
    if args.steps is None:
        args.steps = 3 if args.config == "stack" else 2560
    if args.warmup is None:
        args.warmup = 3 if args.config == "stack" else 32
    args.warmup = max(args.warmup, 3)
    ws, rank, local = init_dist(args)
    try:
        if args.impl == "reference":
            res = reference_arm(args, ws, rank)
        else:
            res = run_ours(args.config, args, ws, rank, local)
            if args.default_run:  # the other hot-path kernels as secondary lines
                for key, cfg, window in SECONDARY:
                    sa = sub_args(args, *SECONDARY_STEPS[cfg])
                    sa.window = window
                    sub = run_ours(cfg, sa, ws, rank, local)
                    if rank == 0:
                        res[key] = {k: sub[k] for k in SUB_KEYS if k in sub}
                    torch.cuda.empty_cache()
                if rank == 0:
                    res["gpu_launches_all_lines"] = res["gpu_launches"] + sum(res[k]["gpu_launches"]
                                                                              for k, _, _ in SECONDARY)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if ws > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
