"""Benchmark of the GDN hot path on B200 (one JSON line on stdout from rank 0).

Headline (BASELINE metric, configs[1] at B=64): GDN decode, one T=1 step over
B=64 sequences with qk16_v32 heads, fp32 state resident in HBM and updated in
place.  ``value`` = state bytes moved per second (B * 32 * 128 * 128 * 4 * 2
bytes per step) summed over ranks; ``ms_per_step`` = device time of one step.
L2 is flushed between timed steps (see L2Flush), outside the timed events.

Also reported on the same line:
* ``prefill``: configs[2] (one 8192-token sequence, chunked C=64) tokens/s and
  its tensor/HBM roofline, plus configs[3] (16 packed sequences) tokens/s;
* ``decode_sweep``: configs[1] B in {1, 8, 32, 64, 128, 256};
* ``sharded``: BASELINE configs[4] over the ranks (decode B=1024, 64-sequence
  prefill) and one 65,536-token sequence by context-parallel prefill;
* ``decode_pool``: the pooled / multi-token decode at B=64 (fp32 and bf16 state
  pools, T=1 and T=4, with and without per-token intermediate states);
* ``roofline``: the decode kernel against the measured HBM copy bandwidth;
* ``cpu_baseline``: the fp32 CPU oracle on the host cores (bounded sample);
* ``e2e``: the decode metric through the C ABI with pinned host buffers,
  host-to-device inputs and device-to-host output inside the timed region;
* ``clocks``: nvidia-smi samples taken during the measurements.

``--profile decode|decode_pool|prefill`` only launches a few kernels of one case (no
timing, no output line): the command that the ncu summaries under profiles/ were made
with.

``--impl reference`` times the reference's algorithm on the host cores
(the fp32 CPU restatement in oracle/, rank 0 only) for the same metric.

Multi-GPU (torchrun, one rank per GPU): every rank runs the same per-GPU
workload on its own sequences and state shard (weak scaling, no collective on
the data path); the step time is the max over ranks.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = ("GDN decode µs/step & HBM GB/s (B=64); chunked prefill tokens/s (T=8192)")
UNIT = "GB/s"
H_QK, H_V, D = 16, 32, 128
STATE_BYTES_PER_SEQ = H_V * D * D * 4 * 2          # read + write of the fp32 state
PREFILL_FLOP_PER_TOKEN_HEAD = 10 * 64 * D + 6 * D * D  # 180,224
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


NCU_METRICS = "dram__bytes_read.sum,dram__bytes_write.sum"
TRAFFIC_RANGE = "gdn_traffic"


def _ncu_rows(csv_path):
    """(ID, kernel name, metric name, value) rows of an ncu --csv log."""
    import csv
    with open(csv_path, newline="") as f:
        lines = [ln for ln in f if ln.startswith('"')]
    rows = []
    for rec in csv.DictReader(lines):
        try:
            val = float(str(rec.get("Metric Value", "")).replace(",", ""))
        except ValueError:
            continue
        rows.append((int(rec.get("ID", "0") or 0), rec.get("Kernel Name", ""),
                     rec.get("Metric Name", ""), val))
    return rows


def measure_traffic(profile_args, timeout_s=600):
    """DRAM traffic of one launch of this file's --profile case, from one ncu
    capture (a child process started before this process touches the GPU).

    The profile run brackets its last launch and one evict-only kernel after it
    (a read of 2x the L2 size of clean data) in the NVTX range TRAFFIC_RANGE,
    and ncu captures exactly the kernels inside it (--cache-control none: no
    flush by ncu; the profile case itself evicts L2 before the launch).  A
    kernel's dirty lines reach DRAM after its window closes, when the next
    kernel evicts them, so the launch's traffic is its kernels' DRAM reads and
    writes plus the evict kernel's DRAM writes (that kernel writes nothing else
    of its own).  Returns None when ncu is unavailable or the capture fails."""
    import shutil
    import tempfile
    ncu = shutil.which("ncu")
    if ncu is None:
        return None
    base = ["--metrics", NCU_METRICS, "--clock-control", "none", "--cache-control", "none",
            "--nvtx", "--nvtx-include", f"{TRAFFIC_RANGE}/"]
    with tempfile.TemporaryDirectory() as td:
        log_path = os.path.join(td, "traffic.csv")
        cmd = [ncu, *base, "--csv", "--print-units", "base", "--log-file", log_path,
               sys.executable, os.path.abspath(__file__), "--profile", *profile_args,
               "--flush-l2", "--traffic-range"]
        try:
            res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                                 timeout=timeout_s)
        except (OSError, subprocess.TimeoutExpired) as e:
            log(f"traffic capture failed: {e}")
            return None
        if res.returncode != 0 or not os.path.exists(log_path):
            log(f"traffic capture failed (rc={res.returncode}): {res.stdout[-2000:]}")
            return None
        rows = _ncu_rows(log_path)
    per = {}
    for kid, kname, metric, val in rows:
        d = per.setdefault(kid, {"name": kname})
        d[metric] = val
    if not per:
        return None
    ids = sorted(per)
    *own, evict = ids   # the evict-only kernel closes the range
    out = {"dram_read": sum(per[i].get("dram__bytes_read.sum", 0.0) for i in own),
           "dram_write_in_window": sum(per[i].get("dram__bytes_write.sum", 0.0) for i in own),
           "dram_write_drained_after": per[evict].get("dram__bytes_write.sum", 0.0)}
    out["bytes"] = out["dram_read"] + out["dram_write_in_window"] + out["dram_write_drained_after"]
    names = {}
    for i in own:
        n = per[i]["name"].split("(")[0].replace("void ", "").split("<")[0].strip()
        names[n] = names.get(n, 0) + 1
    out["kernels"] = names
    out["command"] = " ".join(["ncu", *base, "python bench.py --profile", *profile_args,
                               "--flush-l2", "--traffic-range"])
    return out


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 1.2 * min(power)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
                "samples": len(sm), "power_w_max": max(power), "reasons": sorted(reasons)}


# ----------------------------------------------------------------------------- GPU arm
class L2Flush:
    """Evicts the timed kernel's data from L2 between timed steps: writes a
    buffer of 2x the L2 size, then reads another buffer of 2x the L2 size so
    that the L2 is left holding clean lines (no write-back of the flush's own
    dirty lines is charged to the next timed kernel)."""

    def __init__(self, l2_bytes):
        n = max(256 << 20, 2 * l2_bytes) // 4
        self.w = torch.empty(n, dtype=torch.float32, device="cuda")
        self.r = torch.zeros(n, dtype=torch.float32, device="cuda")
        self.sink = torch.empty((), dtype=torch.float32, device="cuda")

    def zero_(self):
        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.sink)
        # keep the GPU busy a little longer, so that the host has enqueued the
        # timed launch before the GPU reaches the start event (host-side
        # argument checks then never show up as device time)
        torch.cuda._sleep(100_000)

    def evict_clean(self):
        """Read 2x the L2 size of clean data: evicts (writes back) every dirty
        line and writes nothing itself."""
        torch.sum(self.r, dim=0, out=self.sink)


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def time_decode(K, batch, steps, warmup, flush, seed=0):
    """Per-step device time (ms) of in-place decode steps; L2 flushed between steps."""
    from gdn_kernel_b200 import workloads as W

    x = W.make_decode_inputs(batch, seed=seed, device="cuda")
    out = torch.empty(batch, 1, H_V, D, dtype=torch.bfloat16, device="cuda")
    args = (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale, out, x.state)
    for _ in range(warmup):
        flush.zero_()
        K.gdn_decode(*args)
    torch.cuda.synchronize()
    ev = [_events() for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        K.gdn_decode(*args)
        e1.record()
    torch.cuda.synchronize()
    times = [e0.elapsed_time(e1) for e0, e1 in ev]
    del x, out
    return times


def time_decode_pool(K, batch, seq_len, steps, warmup, flush, state_dtype, inter, seed=0):
    """Per-call device time (ms) of the pooled / multi-token decode, in place on a
    pool of 2*batch slots (entries read distinct random slots)."""
    from gdn_kernel_b200 import workloads as W

    x = W.make_pool_decode_inputs(batch, seq_len, 2 * batch, seed=seed, device="cuda",
                                  state_dtype=state_dtype)
    out = torch.empty(batch, seq_len, H_V, D, dtype=torch.bfloat16, device="cuda")
    ibuf = (torch.empty(2 * batch, seq_len, H_V, D, D, dtype=state_dtype, device="cuda")
            if inter else None)
    args = (x.q, x.k, x.v, x.pool, x.indices, x.A_log, x.a, x.dt_bias, x.b, x.scale, out)
    for _ in range(warmup):
        flush.zero_()
        K.gdn_decode_pool(*args, intermediate_states=ibuf)
    torch.cuda.synchronize()
    ev = [_events() for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        K.gdn_decode_pool(*args, intermediate_states=ibuf)
        e1.record()
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) for e0, e1 in ev]


def time_steady(calls, flush, replays=10, warmup=3):
    """Device time (ms) per call of ``len(calls)`` calls run back to back, as a
    serving loop issues its steps: captured once into a CUDA graph, the graph
    replayed with the L2 flushed between replays.  Each call has its own inputs
    and state, together larger than the L2, so no call finds another's data
    cached; consecutive launches overlap only at their edges."""
    for c in calls:
        c()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    for _ in range(warmup):
        flush.zero_()
        g.replay()
    torch.cuda.synchronize()
    ev = [_events() for _ in range(replays)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        g.replay()
        e1.record()
    torch.cuda.synchronize()
    ms = statistics.median([e0.elapsed_time(e1) for e0, e1 in ev]) / len(calls)
    del g
    return ms


def steady_decode(K, hbm_peak, flush, n_sets=16):
    """The decode serving forms back to back (time_steady): the reference decode
    at B = 1, 8, 32, 64 and the pooled bf16 T=1 / fp32 T=4 decode at B=64."""
    from gdn_kernel_b200 import workloads as W

    res = {}
    for b in (1, 8, 32, 64):
        xs = [W.make_decode_inputs(b, seed=4000 + i, device="cuda") for i in range(n_sets)]
        outs = [torch.empty(b, 1, H_V, D, dtype=torch.bfloat16, device="cuda") for _ in xs]
        calls = [(lambda x=x, o=o: K.gdn_decode(x.q, x.k, x.v, x.state, x.A_log, x.a,
                                                x.dt_bias, x.b, x.scale, o, x.state))
                 for x, o in zip(xs, outs)]
        ms = time_steady(calls, flush)
        nbytes = b * STATE_BYTES_PER_SEQ
        res[f"decode_B{b}"] = {"us_per_step": round(ms * 1e3, 2),
                               "frac_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 3)}
        del xs, outs, calls
    for name, seq_len, sdt in (("pool_B64_T1_bf16", 1, torch.bfloat16),
                               ("pool_B64_T4_fp32", 4, torch.float32)):
        xs = [W.make_pool_decode_inputs(64, seq_len, 64, seed=5000 + i, device="cuda",
                                        state_dtype=sdt) for i in range(n_sets)]
        outs = [torch.empty(64, seq_len, H_V, D, dtype=torch.bfloat16, device="cuda")
                for _ in xs]
        calls = [(lambda x=x, o=o: K.gdn_decode_pool(x.q, x.k, x.v, x.pool, x.indices, x.A_log,
                                                     x.a, x.dt_bias, x.b, x.scale, o))
                 for x, o in zip(xs, outs)]
        ms = time_steady(calls, flush)
        esz = 4 if sdt == torch.float32 else 2
        nbytes = 64 * H_V * D * D * esz * 2
        res[name] = {"us_per_step": round(ms * 1e3, 2),
                     "frac_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 3)}
        del xs, outs, calls
    res["method"] = (f"{n_sets} steps on distinct inputs and states captured in one CUDA graph, "
                     "L2 flushed between replays; device time per step")
    return res


def time_decode_e2e(K, batch, steps, warmup, flush, seed=0):
    """Decode through the C ABI with pinned host inputs/outputs each step."""
    from gdn_kernel_b200 import workloads as W

    x = W.make_decode_inputs(batch, seed=seed, device="cuda")
    # The step's token inputs (q, k, v, a, b: all bf16) packed back to back in
    # one pinned host buffer and one device buffer, so each step moves them with
    # a single host-to-device copy; the kernel reads views of the device buffer.
    parts = (x.q, x.k, x.v, x.a, x.b)
    sizes = [t.numel() for t in parts]
    host_in = torch.cat([t.reshape(-1).cpu() for t in parts]).pin_memory()
    dev_in = torch.empty_like(host_in, device="cuda")
    views, off = [], 0
    for t, n in zip(parts, sizes):
        views.append(dev_in[off:off + n].view(t.shape))
        off += n
    out = torch.empty(batch, 1, H_V, D, dtype=torch.bfloat16, device="cuda")
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = host_in.numel() * host_in.element_size()
    d2h = host_out.numel() * host_out.element_size()

    def step():
        dev_in.copy_(host_in, non_blocking=True)
        q, k, v, a, b = views
        K.gdn_decode(q, k, v, x.state, x.A_log, a, x.dt_bias, b, x.scale, out, x.state)
        host_out.copy_(out, non_blocking=True)

    for _ in range(warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    ev = [_events() for _ in range(steps)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        step()
        e1.record()
    torch.cuda.synchronize()
    times = [e0.elapsed_time(e1) for e0, e1 in ev]
    return times, h2d, d2h


def time_prefill(K, lengths, iters, warmup, flush, seed=0, with_state=True):
    from gdn_kernel_b200 import workloads as W

    x = W.make_prefill_inputs(lengths, seed=seed, device="cuda", with_state=with_state)
    T = sum(lengths)
    out = torch.empty(T, H_V, D, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(len(lengths), H_V, D, D, dtype=torch.float32, device="cuda")
    args = (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out, ns)
    # the two-stage path's workspace is allocated once, outside the timed region
    ws = torch.empty(K.prefill_workspace_bytes(len(lengths), T, H_V), dtype=torch.uint8,
                     device="cuda")
    for _ in range(warmup):
        flush.zero_()
        K.gdn_prefill(*args, workspace=ws)
    torch.cuda.synchronize()
    ev = [_events() for _ in range(iters)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        K.gdn_prefill(*args, workspace=ws)
        e1.record()
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) for e0, e1 in ev]


def prefill_case(K, lengths, with_state, seed, iters, warmup, flush, prefix_curve=0):
    """Times the default prefill (two-stage path, workspace allocated outside the
    timed region) on configs-shaped inputs and keeps what the drift report needs
    on the host: the inputs, the outputs and, with ``prefix_curve`` > 0 (one
    sequence), the final state of the prefixes of prefix_curve, 2 prefix_curve, ...
    tokens run as their own calls."""
    from gdn_kernel_b200 import workloads as W

    x = W.make_prefill_inputs(lengths, seed=seed, device="cuda", with_state=with_state)
    T, N = sum(lengths), len(lengths)
    out = torch.empty(T, H_V, D, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty(N, H_V, D, D, dtype=torch.float32, device="cuda")
    ws = torch.empty(K.prefill_workspace_bytes(N, T, H_V), dtype=torch.uint8, device="cuda")
    args = (x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens, x.scale, out, ns)
    for _ in range(warmup):
        flush.zero_()
        K.gdn_prefill(*args, workspace=ws)
    torch.cuda.synchronize()
    ev = [_events() for _ in range(iters)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        K.gdn_prefill(*args, workspace=ws)
        e1.record()
    torch.cuda.synchronize()
    times = [e0.elapsed_time(e1) for e0, e1 in ev]
    prefix_states = []
    if prefix_curve and N == 1:
        for n in range(prefix_curve, T + 1, prefix_curve):
            cu = torch.tensor([0, n], dtype=x.cu_seqlens.dtype, device="cuda")
            o_p, s_p = K.prefill(x.q[:n], x.k[:n], x.v[:n], x.state, x.A_log, x.a[:n],
                                 x.dt_bias, x.b[:n], cu, x.scale)
            prefix_states.append((n, s_p.cpu()))
    host = {n: (getattr(x, n).cpu() if getattr(x, n) is not None else None)
            for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")}
    host["scale"] = x.scale
    res = {"times": times, "inputs": host, "out": out.cpu(), "new_state": ns.cpu(),
           "prefix_states": prefix_states, "gpu_inputs": x}
    return res


def prefill_drift_and_cpu(case, lengths):
    """The fp32 CPU oracle (chunked restatement of the reference prefill) on all
    host cores: its throughput is the CPU baseline of the case, and its results
    measure the GPU path's drift: output error, final-state relative Frobenius
    error per (sequence, head), and for one sequence the same error of the state
    after every prefix of the drift curve."""
    from oracle import gdn_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    x = case["inputs"]
    t0 = time.perf_counter()
    ro, rs, chunk_states = O.prefill_chunked(x["q"], x["k"], x["v"], x["state"], x["A_log"],
                                             x["a"], x["dt_bias"], x["b"], x["cu_seqlens"],
                                             x["scale"], return_chunk_states=True)
    sec = time.perf_counter() - t0
    T = sum(lengths)

    def relfro(a, b):
        a, b = a.double(), b.double()
        return ((a - b).flatten(-2).norm(dim=-1) / b.flatten(-2).norm(dim=-1).clamp_min(1e-30))

    err = (case["out"].float() - ro.float()).abs()
    sr = relfro(case["new_state"], rs)                                   # [N, H_v]
    drift = {"out_max_abs": float(err.max()), "out_mean_abs": float(err.mean()),
             "state_relfro_max": float(sr.max()), "state_relfro_mean": float(sr.mean()),
             "per_sequence_state_relfro_max": [round(float(v), 6) for v in sr.max(dim=1).values],
             "tolerance": "output atol = rtol = 2e-2; final state relative Frobenius <= 1e-2 "
                          "per (sequence, head)",
             "reference": "oracle.gdn_oracle.prefill_chunked (fp32 CPU)"}
    if case["prefix_states"]:
        curve = []
        cs = chunk_states[0]
        for n, st in case["prefix_states"]:
            ref = rs[0] if n >= T else cs[n // 64]
            w0 = max(0, n - case["prefix_states"][0][0])
            curve.append({"tokens": n,
                          "state_relfro_max": round(float(relfro(st[0], ref).max()), 6),
                          "out_max_abs_window": round(float(err[w0:n].max()), 6)})
        drift["curve"] = curve
    cpu = {"value": round(T / sec, 1), "unit": "tokens/s", "cores": os.cpu_count(),
           "kind": "port",
           "sample": f"the whole case ({T} tokens, {len(lengths)} sequences) through the fp32 "
                     f"chunked CPU oracle (torch, {torch.get_num_threads()} threads): "
                     f"{sec:.2f} s"}
    # The token-by-token recurrence (the reference's own sequential form, batched
    # over heads) on a prefix of the first sequence: its per-token cost does not
    # depend on the position, so the prefix rate is the whole case's.
    n = min(lengths[0], 2048)
    st0 = None if x["state"] is None else x["state"][:1]
    t0 = time.perf_counter()
    O.prefill_sequential(x["q"][:n], x["k"][:n], x["v"][:n], st0, x["A_log"], x["a"][:n],
                         x["dt_bias"], x["b"][:n], torch.tensor([0, n], dtype=torch.int32),
                         x["scale"])
    sec_seq = time.perf_counter() - t0
    cpu["sequential"] = {"value": round(n / sec_seq, 1), "unit": "tokens/s",
                         "cores": os.cpu_count(), "kind": "port",
                         "sample": f"the first {n} tokens of sequence 0 through the fp32 "
                                   f"token-sequential CPU oracle (torch, "
                                   f"{torch.get_num_threads()} threads): {sec_seq:.2f} s"}
    return drift, cpu, ro


def flashinfer_prefill(case, lengths, iters, warmup, flush):
    """FlashInfer's Blackwell chunked GDN prefill (CuTe-DSL tcgen05 kernel,
    flashinfer.gdn_kernels.blackwell) on the same inputs, timed the same way: a
    reference point only, never on this package's path.  Its gate input is the
    per-token decay g = exp(log g) and beta = sigmoid(b), both fp32 (formed once,
    outside the timed region)."""
    try:
        from flashinfer.gdn_kernels import _has_blackwell_prefill, chunk_gated_delta_rule_sm100
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer import failed: {e!r}"[:300]}
    if not _has_blackwell_prefill:
        return {"unavailable": "flashinfer reports no Blackwell prefill kernel"}
    import torch.nn.functional as F

    x = case["gpu_inputs"]
    xa = x.a.float() + x.dt_bias.float()
    gate = torch.exp(-torch.exp(x.A_log.float()) * F.softplus(xa, beta=1.0, threshold=20.0))
    gate = gate.contiguous()
    beta = torch.sigmoid(x.b.float()).contiguous()
    T, N = sum(lengths), len(lengths)
    out = torch.empty(T, H_V, D, dtype=torch.bfloat16, device="cuda")
    ost = torch.empty(N, H_V, D, D, dtype=torch.float32, device="cuda")
    cu32 = x.cu_seqlens.to(torch.int32)

    def run():
        chunk_gated_delta_rule_sm100(x.q, x.k, x.v, gate, beta, out, cu32, x.state, ost, x.scale)
    try:
        t0 = time.perf_counter()
        run()
        torch.cuda.synchronize()
        first_s = time.perf_counter() - t0
        for _ in range(warmup):
            flush.zero_()
            run()
        torch.cuda.synchronize()
        ev = [_events() for _ in range(iters)]
        for e0, e1 in ev:
            flush.zero_()
            e0.record()
            run()
            e1.record()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": (f"flashinfer routes to this kernel only for torch builds with "
                                f"CUDA >= 13 (this one: {torch.version.cuda}); called directly "
                                f"here it fails: {e!r}")[:400]}
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
    return {"us": round(ms * 1e3, 1), "tokens_per_s": round(T / (ms * 1e-3), 1),
            "first_call_s": round(first_s, 1), "out": out.cpu(), "new_state": ost.cpu(),
            "kernel": "flashinfer.gdn_kernels.chunk_gated_delta_rule_sm100 "
                      "(flashinfer 0.6.11.post2, CuTe DSL, sm_100)"}


def flashinfer_decode(batch, iters, warmup, flush, state_dtype, seed=0):
    """FlashInfer's pretranspose GDN decode (k-last state [B, H_v, V, K], in place,
    no in-kernel q/k normalisation) at the headline shape, timed like our decode:
    fp32 state takes its legacy T=1 kernel, bf16 state its BF16-state kernel."""
    from gdn_kernel_b200 import workloads as W

    try:
        from flashinfer.gdn_decode import gated_delta_rule_decode_pretranspose
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer import failed: {e!r}"[:300]}
    x = W.make_decode_inputs(batch, seed=seed, device="cuda")
    state = x.state.to(state_dtype).contiguous()
    out = torch.empty(batch, 1, H_V, D, dtype=torch.bfloat16, device="cuda")

    def run():
        gated_delta_rule_decode_pretranspose(x.q, x.k, x.v, state, x.A_log, x.a, x.dt_bias, x.b,
                                             x.scale, out, use_qk_l2norm=False)
    try:
        run()
        for _ in range(warmup):
            flush.zero_()
            run()
        torch.cuda.synchronize()
        ev = [_events() for _ in range(iters)]
        for e0, e1 in ev:
            flush.zero_()
            e0.record()
            run()
            e1.record()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flashinfer run failed: {e!r}"[:300]}
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
    esz = 4 if state_dtype == torch.float32 else 2
    nbytes = batch * H_V * D * D * esz * 2
    return {"us": round(ms * 1e3, 2), "state_GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "kernel": "flashinfer.gdn_decode.gated_delta_rule_decode_pretranspose "
                      f"({'fp32' if esz == 4 else 'bf16'} state, use_qk_l2norm=False)"}


def _max_over_ranks(ms, world):
    if world == 1:
        return ms
    import torch.distributed as dist
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _per_rank(value, world):
    """The value of every rank, in rank order (every rank calls this in turn)."""
    if world == 1:
        return [value]
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device="cuda")
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [float(x.item()) for x in parts]


def run_sharded(K, rank, world, flush, hbm_peak):
    """a fixed whole-box workload partitioned by sequence
    (strong scaling): (a) decode B=1024 as contiguous batch blocks; (b) packed
    prefill of 64 sequences with lengths U[1024, 16384], LPT-assigned."""
    from gdn_kernel_b200 import sharding as S, workloads as W
    import torch.distributed as dist

    res = {}
    lo, hi = S.decode_shards(1024, world)[rank]
    if world > 1:
        dist.barrier()
    ts = time_decode(K, hi - lo, 20, 3, flush, seed=5000 + rank)
    per_rank = _per_rank(statistics.median(ts) * 1e3, world)
    ms = _max_over_ranks(statistics.median(ts), world)
    step_bytes = 1024 * STATE_BYTES_PER_SEQ
    gbps = step_bytes / (ms * 1e-3) / 1e9
    res["decode_B1024"] = {"us_per_step": round(ms * 1e3, 2), "state_GBps": round(gbps, 1),
                           "per_gpu_frac_hbm": round(gbps / world / hbm_peak, 4),
                           "box_frac_hbm": round(gbps / (world * hbm_peak), 4),
                           "batch_per_gpu": hi - lo,
                           "per_rank_us": [round(x, 2) for x in per_rank]}
    lengths = W.varlen_lengths(64, 1024, 16384, seed=4)
    mine = [lengths[i] for i in S.prefill_shards(lengths, world)[rank]]
    if world > 1:
        dist.barrier()
    pts = time_prefill(K, mine, 3, 2, flush, seed=6000 + rank) if mine else [0.0]
    per_rank = _per_rank(statistics.median(pts) * 1e3, world)
    per_rank_tokens = _per_rank(sum(mine), world)
    pms = _max_over_ranks(statistics.median(pts), world)
    T = sum(lengths)
    hb = prefill_hbm_bytes(lengths, True)
    res["prefill_64seq"] = {"tokens": T, "us": round(pms * 1e3, 1),
                            "tokens_per_s": round(T / (pms * 1e-3), 1),
                            "hbm_GBps": round(hb / (pms * 1e-3) / 1e9, 1),
                            "box_frac_hbm": round(hb / (pms * 1e-3) / 1e9 / (world * hbm_peak), 4),
                            "tokens_this_rank": sum(mine),
                            "per_rank_us": [round(x, 1) for x in per_rank],
                            "per_rank_tokens": [int(x) for x in per_rank_tokens]}
    # (c) one long sequence split over the ranks (context-parallel prefill; one
    # all-gather of the per-segment affine state maps per call)
    res["prefill_context_parallel"] = time_context_parallel(K, rank, world, flush, 65536)
    return res


def time_context_parallel(K, rank, world, flush, total_tokens, iters=3, warmup=1):
    """One sequence of ``total_tokens`` tokens: the single-call prefill at one
    GPU, the context-parallel prefill over ``world`` ranks otherwise (device
    time per call, max over ranks)."""
    from gdn_kernel_b200 import context_parallel as CP, workloads as W
    import torch.distributed as dist

    x = W.make_prefill_inputs([total_tokens], seed=6100, device="cuda")
    lo, hi = CP.cp_segments(total_tokens, world, CP.first_segment_weight(world))[rank]
    if world == 1:
        out = torch.empty(total_tokens, H_V, D, dtype=torch.bfloat16, device="cuda")
        ns = torch.empty(1, H_V, D, D, dtype=torch.float32, device="cuda")
        ws = torch.empty(K.prefill_workspace_bytes(1, total_tokens, H_V), dtype=torch.uint8,
                         device="cuda")

        def run():
            K.gdn_prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                          x.scale, out, ns, workspace=ws)
    else:
        seg = lambda t: t[lo:hi].contiguous()
        q, k, v, a, b = (seg(t) for t in (x.q, x.k, x.v, x.a, x.b))

        def run():
            CP.cp_prefill(rank, world, q, k, v, x.state[0], x.A_log, a, x.dt_bias, b, x.scale)
    for _ in range(warmup):
        flush.zero_()
        run()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        if world > 1:
            dist.barrier()
        e0, e1 = _events()
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    per_rank = _per_rank(statistics.median(ts) * 1e3, world)
    per_rank_tokens = _per_rank(hi - lo, world)
    ms = _max_over_ranks(statistics.median(ts), world)
    del x
    return {"tokens": total_tokens, "us": round(ms * 1e3, 1),
            "per_rank_us": [round(v, 1) for v in per_rank],
            "per_rank_segment_tokens": [int(v) for v in per_rank_tokens],
            "tokens_per_s": round(total_tokens / (ms * 1e-3), 1),
            "segment_tokens_this_rank": hi - lo,
            "method": "single call (one sequence in overlapping pieces)" if world == 1 else
                      f"context-parallel over {world} ranks (rank 0 runs its segment; the "
                      f"others run pass A, two concurrent recurrences; all-gather of the "
                      f"affine maps; fold; output correction GEMM)"}


def prefill_hbm_bytes(lengths, with_state):
    """Algorithmic HBM bytes of one prefill launch: q,k,v,a,b read, output written,
    initial state read (if any) and final state written."""
    T, N = sum(lengths), len(lengths)
    tok = T * (2 * H_QK * D * 2 + H_V * D * 2 + 2 * H_V * 2)
    out = T * H_V * D * 2
    st = N * H_V * D * D * 4 * (2 if with_state else 1)
    return tok + out + st


def cpu_decode_sample(batch, steps, seed=0):
    """The CPU oracle's decode on the host cores: seconds per step."""
    from gdn_kernel_b200 import workloads as W
    from oracle import gdn_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    x = W.make_decode_inputs(batch, seed=seed)
    state = x.state
    O.decode_step(x.q, x.k, x.v, state, x.A_log, x.a, x.dt_bias, x.b, x.scale)  # warm
    t0 = time.perf_counter()
    for _ in range(steps):
        _, state = O.decode_step(x.q, x.k, x.v, state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    return (time.perf_counter() - t0) / steps


def run_gpu(args, rank, world, local_rank, traffic=None):
    import torch.distributed as dist

    from gdn_kernel_b200 import _lib, kernel as K

    torch.cuda.set_device(local_rank)
    _lib.load()
    peaks, peaks_src = load_peaks()
    hbm_peak = float(peaks["hbm_gbs"])
    tc_peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    l2 = torch.cuda.get_device_properties(local_rank).L2_cache_size
    flush = L2Flush(l2)
    B = args.batch

    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)

    # ---- headline: decode B=64, K timed steps
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    times = time_decode(K, B, args.steps, args.warmup, flush, seed=1000 + rank)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = sum(times)
    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    step_bytes = B * STATE_BYTES_PER_SEQ
    value = world * step_bytes * args.steps / (total_ms * 1e-3) / 1e9
    mean_launch_ms = statistics.mean(times)
    achieved = step_bytes / (mean_launch_ms * 1e-3) / 1e9

    # ---- e2e through the C ABI with host buffers
    e2e_times, h2d, d2h = time_decode_e2e(K, B, max(args.steps // 2, 10), args.warmup, flush,
                                          seed=2000 + rank)
    e2e_ms = sum(e2e_times)
    t = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = world * step_bytes * len(e2e_times) / (float(t.item()) * 1e-3) / 1e9

    extra = {}
    if not args.quick:
        # ---- decode sweep
        sweep = {}
        for b in (1, 8, 32, 64, 128, 256):
            ts = time_decode(K, b, 30, 3, flush, seed=3000 + b)
            ms = statistics.median(ts)
            sweep[str(b)] = {"us_per_step": round(ms * 1e3, 2),
                             "state_GBps": round(b * STATE_BYTES_PER_SEQ / (ms * 1e-3) / 1e9, 1),
                             "frac_hbm": round(b * STATE_BYTES_PER_SEQ / (ms * 1e-3) / 1e9
                                               / hbm_peak, 3)}
        extra["decode_sweep"] = sweep
        # ---- pooled / multi-token decode (the serving forms of the step)
        pool = {}
        for name, seq_len, sdt, inter in (("B64_T1_fp32", 1, torch.float32, False),
                                          ("B64_T1_bf16", 1, torch.bfloat16, False),
                                          ("B64_T4_fp32", 4, torch.float32, False),
                                          ("B64_T4_fp32_intermediate", 4, torch.float32, True)):
            ts = time_decode_pool(K, 64, seq_len, 30, 3, flush, sdt, inter, seed=7000)
            ms = statistics.median(ts)
            esz = 4 if sdt == torch.float32 else 2
            # state read once and written once, plus one stored state per token
            nbytes = 64 * H_V * D * D * esz * (2 + (seq_len if inter else 0))
            pool[name] = {"us": round(ms * 1e3, 2),
                          "tokens_per_s": round(64 * seq_len / (ms * 1e-3), 1),
                          "state_GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "frac_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 3)}
        extra["decode_pool"] = pool
        # ---- the same forms back to back, as a serving loop runs them
        extra["decode_steady"] = steady_decode(K, hbm_peak, flush)
        # ---- prefill configs[2] and configs[3]
        from gdn_kernel_b200 import workloads as W
        pre, cases = {}, {}
        for name, lengths, with_state in (
                ("T8192", [8192], False),
                ("varlen16", W.varlen_lengths(16, 128, 8192, seed=3), True)):
            case = prefill_case(K, lengths, with_state, 4000 + rank, 5, 2, flush,
                                prefix_curve=1024 if len(lengths) == 1 else 0)
            ms = statistics.median(case["times"])
            T = sum(lengths)
            flop = T * H_V * PREFILL_FLOP_PER_TOKEN_HEAD
            hb = prefill_hbm_bytes(lengths, with_state)
            pre[name] = {
                "tokens": T, "sequences": len(lengths), "us": round(ms * 1e3, 1),
                "tokens_per_s": round(world * T / (ms * 1e-3), 1),
                "tflops": round(flop / (ms * 1e-3) / 1e12, 2),
                "tensor_frac": round(flop / (ms * 1e-3) / 1e12 / tc_peak, 4),
                "hbm_GBps": round(hb / (ms * 1e-3) / 1e9, 1),
                "hbm_frac": round(hb / (ms * 1e-3) / 1e9 / hbm_peak, 4),
                "algorithmic_flop": flop, "algorithmic_bytes": hb,
                "path": "gdn_prefill (two-stage kernels, caller workspace)",
            }
            if world == 1 and rank == 0 and not args.no_comparators:
                fi = flashinfer_prefill(case, lengths, 5, 2, flush)
                if "us" in fi:
                    fi["ours_speedup"] = round(fi["us"] / (ms * 1e3), 3)
                pre[name]["flashinfer_sm100"] = fi
            if (traffic or {}).get(f"prefill_{name}"):
                t = traffic[f"prefill_{name}"]
                pre[name]["traffic"] = dict(t, x_algorithmic=round(t["bytes"] / hb, 3))
            case.pop("gpu_inputs")
            cases[name] = (case, lengths)
        extra["prefill"] = pre
        if world == 1 and rank == 0 and not args.no_comparators:
            extra["decode_comparators"] = {
                "flashinfer_B64_fp32_state": flashinfer_decode(64, 30, 3, flush, torch.float32),
                "flashinfer_B64_bf16_state": flashinfer_decode(64, 30, 3, flush, torch.bfloat16)}
        extra["sharded"] = run_sharded(K, rank, world, flush, hbm_peak)

    clocks = sampler.stop()

    line = None
    if rank == 0 and world == 1 and not args.quick and not args.no_cpu:
        # CPU baseline and drift of each prefill case (host only, after the GPU work)
        for name, (case, lengths) in cases.items():
            drift, cpu_pre, ro = prefill_drift_and_cpu(case, lengths)
            extra["prefill"][name]["cpu_baseline"] = cpu_pre
            extra["prefill"][name]["drift"] = drift
            fi = extra["prefill"][name].get("flashinfer_sm100", {})
            if "out" in fi:
                fo, fs = fi.pop("out"), fi.pop("new_state")
                fi["out_max_abs_vs_oracle"] = round(float((fo.float() - ro.float()).abs().max()), 6)
                fi["out_max_abs_vs_ours"] = round(float((fo.float() - case["out"].float()).abs().max()), 6)
    for v in (extra.get("prefill") or {}).values():
        fi = v.get("flashinfer_sm100")
        if fi:
            fi.pop("out", None)
            fi.pop("new_state", None)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            steps_cpu = args.cpu_steps
            sec = cpu_decode_sample(B, steps_cpu)
            cpu = {"value": round(step_bytes / sec / 1e9, 3), "unit": UNIT,
                   "cores": os.cpu_count(), "kind": "port",
                   "sample": f"decode B={B} qk16_v32, {steps_cpu} steps of the fp32 CPU oracle "
                             f"(torch, {torch.get_num_threads()} threads); "
                             f"{sec * 1e3:.1f} ms/step"}
        dec_traffic = (traffic or {}).get("decode")
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "us_per_step": round(ms_per_step * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"decode B={B} per GPU, qk16_v32, D=128, T=1, in-place fp32 "
                                   f"state (BASELINE configs[1] at B={B})",
                       "batch_per_gpu": B, "num_qk_heads": H_QK, "num_v_heads": H_V,
                       "head_dim": D, "l2": "flushed between timed steps (write 2x L2, then read 2x L2)",
                       "parallelism": f"sequence-sharded x{world}, no collective"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "traffic": (round(dec_traffic["bytes"]) if dec_traffic else None),
                         "traffic_detail": dec_traffic,
                         "peak_source": f"{peaks_src} hbm_gbs (STREAM-style copy)",
                         "kernel": "gdn_decode_kernel",
                         "algorithmic_bytes_per_launch": step_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "gdn_kernel_b200.gdn_decode -> libgdn_b200.so gdn_b200_decode, "
                            "q/k/v/a/b packed in one pinned host buffer (one host-to-device "
                            "copy per step), output copied back each step; state resident in "
                            "HBM"},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
        line.update(extra)
    return line


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's algorithm on the host cores (fp32 CPU restatement; the
    reference's own code path is CUDA-only, so the port stands in)."""
    B = args.batch
    steps = max(1, min(args.steps, args.cpu_steps))
    for _ in range(min(args.warmup, 1)):
        cpu_decode_sample(B, 1, seed=7)
    sec = cpu_decode_sample(B, steps)
    step_bytes = B * STATE_BYTES_PER_SEQ
    value = step_bytes / sec / 1e9
    return {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"decode B={B}, qk16_v32, D=128, T=1 (BASELINE configs[1] at "
                               f"B={B}) on the host cores", "batch_per_gpu": B},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"{steps} decode steps at B={B} of the fp32 CPU oracle "
                                   f"(torch, {torch.get_num_threads()} threads)"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_profile(args):
    """A handful of launches of one case, for ncu captures.  With --flush-l2 the
    L2 is evicted before each launch, as between the timed runs."""
    from gdn_kernel_b200 import _lib, kernel as K, workloads as W

    torch.cuda.set_device(0)
    _lib.load()
    flush = L2Flush(torch.cuda.get_device_properties(0).L2_cache_size) if args.flush_l2 else None

    def before():
        if flush is not None:
            flush.zero_()
        if args.traffic_range and i == args.launches - 1:
            torch.cuda.nvtx.range_push(TRAFFIC_RANGE)

    def after():
        if args.traffic_range and i == args.launches - 1:
            flush.evict_clean()
            torch.cuda.nvtx.range_pop()
    if args.profile == "decode":
        x = W.make_decode_inputs(args.batch, seed=0, device="cuda")
        out = torch.empty(args.batch, 1, H_V, D, dtype=torch.bfloat16, device="cuda")
        for i in range(args.launches):
            before()
            K.gdn_decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale, out,
                         x.state)
            after()
    elif args.profile == "decode_pool":
        sdt = torch.bfloat16 if args.pool_dtype == "bf16" else torch.float32
        x = W.make_pool_decode_inputs(args.batch, args.seq_len, 2 * args.batch, seed=7000,
                                      device="cuda", state_dtype=sdt)
        out = torch.empty(args.batch, args.seq_len, H_V, D, dtype=torch.bfloat16, device="cuda")
        for i in range(args.launches):
            before()
            K.gdn_decode_pool(x.q, x.k, x.v, x.pool, x.indices, x.A_log, x.a, x.dt_bias, x.b,
                              x.scale, out)
            after()
    else:
        lengths = ([args.tokens] if args.sequences == 1
                   else W.varlen_lengths(args.sequences, 128, args.tokens, seed=3))
        x = W.make_prefill_inputs(lengths, seed=0, device="cuda", with_state=args.sequences > 1)
        out = torch.empty(sum(lengths), H_V, D, dtype=torch.bfloat16, device="cuda")
        ns = torch.empty(len(lengths), H_V, D, D, dtype=torch.float32, device="cuda")
        ws = torch.empty(K.prefill_workspace_bytes(len(lengths), sum(lengths), H_V),
                         dtype=torch.uint8, device="cuda")
        for i in range(args.launches):
            before()
            K.gdn_prefill(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.cu_seqlens,
                          x.scale, out, ns, workspace=ws)
            after()
    torch.cuda.synchronize()
    assert _lib.device_status(0) == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=20)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--quick", action="store_true", help="headline decode + e2e only")
    ap.add_argument("--no-ncu", action="store_true", help="skip the in-run ncu traffic capture")
    ap.add_argument("--no-comparators", action="store_true",
                    help="skip the FlashInfer reference-point timings")
    ap.add_argument("--flush-l2", action="store_true",
                    help="--profile: evict L2 (as the timed runs do) before each launch")
    ap.add_argument("--traffic-range", action="store_true",
                    help="--profile with --flush-l2: bracket the last launch and an evict-only "
                         "kernel in an NVTX range (the in-run traffic capture)")
    ap.add_argument("--profile", choices=["decode", "decode_pool", "prefill"], default=None)
    ap.add_argument("--seq-len", type=int, default=4, help="--profile decode_pool: tokens per entry")
    ap.add_argument("--pool-dtype", choices=["fp32", "bf16"], default="fp32",
                    help="--profile decode_pool: state pool type")
    ap.add_argument("--launches", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--sequences", type=int, default=1)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.profile:
        run_profile(args)
        return

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    traffic = None
    if world == 1 and not args.quick and not args.no_ncu:
        # one small ncu capture per kernel group, as child processes, before this
        # process creates its CUDA context
        traffic = {
            "decode": measure_traffic(["decode", "--batch", str(args.batch), "--launches", "3"]),
            "prefill_T8192": measure_traffic(["prefill", "--tokens", "8192", "--launches", "2"]),
        }
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_gpu(args, rank, world, local_rank, traffic)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
