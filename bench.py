"""Benchmark of flash_lab's attention path on B200 (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extra]
                    [--no-cpu] [--no-llama]

Headline workload (the benchmark's prefill configuration): bf16 prefill forward, (B, H, H_kv, S, D) =
(4, 32, 32, 4096, 128), non-causal, Q/K/V ~ N(0, 1) from one seed, scale 1/sqrt(128). One step is
one pass of flash_lab's prefill over that problem; metric TFLOP/s counts 4*B*H*S_q*S_k*D FLOP per
step (the reference's bench/flops.py convention). Inputs (402 MB) are larger than the 126 MB L2,
so no flush is needed between steps.

Multi-GPU (torchrun, one rank per GPU): strong scaling. Every rank builds the same seeded
problem, and rank r runs only its share of it: the (batch, KV head) units
[r U / N, (r + 1) U / N) of the U = B * H_kv units (flash_lab.distributed.attention_sharded: zero-copy
head / batch slices, no communication). value = the whole problem's FLOP / the slowest rank's
time. The decode configurations shard over sequences the same way; the B=1 long-context decode
shards the KV sequence and merges over NVLink.

Every timed configuration is checked first, on the very call that is then timed, against the
oracle (numpy fp64 restatement of the reference's flash_lab/reference.py) on sampled rows /
sequences: error <= 2 x the error of the bf16-rounded fp64 result, and the LSE. The sharded
outputs are also compared bit for bit with one unsharded call. Results go to `correct` in each
entry; if any check fails the line is still printed and the run exits with status 1.

  value        whole-job TFLOP/s with inputs resident in HBM
  e2e          the same work through the public API with pinned HOST inputs: each step copies
               this rank's q, k, v host->device, runs the prefill and copies o and lse back,
               pipelined (copies of one chunk overlap the kernel of the previous one)
  roofline     the prefill kernel: achieved FLOP/s from CUDA-event time over the timed region
               against the measured dense bf16 peak of MEASURED_PEAKS.json; traffic (DRAM bytes
               per launch) from the committed ncu capture in profiles/ when present
  cpu_baseline the oracle on this host's cores, on sampled query rows of the same workload
               (rank 0, N=1)
  extra        causal prefill, decode B=8 H=H_kv=32 at 32K, GQA decode B=8 H_kv=8 with lengths
               U[16K, 32K] (contiguous and 16-row pages), fp32 decode, the B=1 decode split over
               the ranks, the CPU-plumbing configuration timed on the host, and (N=1) the
               Llama-3.1-8B-architecture generation end to end

--impl reference times the reference's own CPU implementation of the path (the oracle port: the
reference is Python and cannot travel to this box) on rank 0 only, with all host threads.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-attention-lab_b200"))
sys.path.insert(0, str(ROOT))

PREFILL = dict(batch=4, heads=32, heads_kv=32, seqlen=4096, head_dim=128)
C0 = dict(batch=1, heads=4, heads_kv=4, seqlen=256, head_dim=64)
E2E_Q_ROWS = 512   # query rows per host->device chunk of the e2e pipeline
METRIC = "prefill TFLOP/s @(4,32,32,4096,128) bf16; decode HBM GB/s @32K cache"
CPU_SAMPLE_ROWS = 1536
REFERENCE_STEP_ROWS = 256
CHECK_ROWS = 256


def prefill_flops(batch, heads, seqlen_q, seqlen_k, head_dim, causal) -> float:
    f = 4.0 * batch * heads * seqlen_q * seqlen_k * head_dim
    return f / 2 if causal else f


def decode_bytes(heads, heads_kv, head_dim, lens, batch) -> float:
    """K and V rows of every sequence read once, plus q read and o written (2-byte elements)."""
    return 2.0 * heads_kv * head_dim * 2 * float(sum(lens)) + 2.0 * batch * heads * head_dim * 2


def load_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained"),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic() -> dict:
    """Per-launch DRAM bytes of each kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


def host_cores() -> int:
    return len(os.sched_getaffinity(0))


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every 5 ms while the timed region runs
    (nvidia-smi's own loop is too coarse for a ~20 ms region). Reads only; changes nothing."""

    REASONS = {  # NVML clocks-event-reason bits
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.005):
        self.index = index
        self.period = period_s
        self.samples: list[tuple[float, int, float]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)

            def loop():
                while not self._stop.is_set():
                    try:
                        clk = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                        pw = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                        self.samples.append((float(clk), int(rs), pw))
                    except Exception:  # noqa: BLE001 - sampling must never break the bench
                        pass
                    self._stop.wait(self.period)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001 - no NVML: report no samples
            self._nvml = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        sm = [c for c, _, _ in self.samples]
        reasons = sorted({name for _, r, _ in self.samples for name, bit in self.REASONS.items()
                          if r & bit})
        power = [p for _, _, p in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.max_mhz) if self.max_mhz else None,
                "reasons": reasons, "samples": len(sm),
                "power_w_median": statistics.median(power) if power else None,
                "source": "NVML, 5 ms period, during the timed region"}


def max_over_ranks(value: float, dist, device) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(fn, steps: int, warmup: int, dist=None, device=None):
    """Runs fn warmup times, then times exactly `steps` calls between CUDA events with a barrier
    and a synchronize on both sides. Returns (this rank's ms per step, max over ranks)."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    return ms, max_over_ranks(ms, dist, device)


# ------------------------------------------------------------------------------------------------
# Checks against the oracle (outside every timed region)
# ------------------------------------------------------------------------------------------------

def _round_err(ref, dtype) -> float:
    import torch

    t = torch.from_numpy(ref)
    return float((t.to(dtype).double() - t).abs().max()) if t.numel() else 0.0


def sample_rows(seqlen: int, n: int, seed: int):
    """n query rows, the first and the last included, the rest drawn without replacement."""
    import numpy as np

    n = min(n, seqlen)
    rng = np.random.default_rng(seed)
    inner = rng.choice(np.arange(1, seqlen - 1), size=max(0, n - 2), replace=False) \
        if seqlen > 2 else np.array([], dtype=np.int64)
    return np.unique(np.concatenate([[0, seqlen - 1], inner]).astype(np.int64))


def check_prefill(o, lse, q, k, v, causal, scale, rows) -> dict:
    """o [B, S_q, H, D] / lse [B, H, S_q] of one call on q, k, v (device tensors, any strides)
    against oracle.attention_rows on `rows`: max |o - ref| <= 2 max |bf16(ref) - ref|, the LSE
    within 1e-3 where finite and -inf exactly where the oracle's is."""
    import numpy as np
    import torch

    import oracle

    rows_t = torch.as_tensor(rows, device=o.device)
    qh = np.zeros(tuple(q.shape))                       # only the sampled rows are read
    qh[:, rows] = q[:, rows_t].double().cpu().numpy()
    ref, ref_lse = oracle.attention_rows(qh, k.double().cpu().numpy(), v.double().cpu().numpy(),
                                         rows, causal=causal, softmax_scale=scale,
                                         return_lse=True)
    got = o[:, rows_t].double().cpu().numpy()
    got_lse = lse[:, :, rows_t].double().cpu().numpy()
    err = float(np.abs(got - ref).max())
    bound = 2 * _round_err(ref, q.dtype)
    finite = np.isfinite(ref_lse)
    lse_ok = bool(np.array_equal(np.isfinite(got_lse), finite))
    lse_err = float(np.abs(got_lse[finite] - ref_lse[finite]).max()) if finite.any() else 0.0
    return {"max_err_vs_ref64": err, "2x_rounding": bound, "lse_err": lse_err,
            "correct": bool(np.isfinite(got).all() and err <= bound and lse_ok
                            and lse_err <= 1e-3),
            "checked": f"{len(rows)} query rows x {q.shape[0] * q.shape[2]} (b,h)"}


def check_decode(o, lse, q3, k_cache, v_cache, seq_lens, scale, seqs, kv_heads,
                 block_tables=None) -> dict:
    """Decode outputs o [B, H, D] / lse [B, H] against oracle.decode on sequences `seqs` and the
    query heads of KV heads `kv_heads` (the same error rule as check_prefill)."""
    import numpy as np
    import torch

    import oracle

    group = q3.shape[1] // k_cache.shape[2]
    heads = [g * group + i for g in kv_heads for i in range(group)]
    lens = seq_lens[seqs].cpu().numpy()
    if block_tables is None:   # [n, S, g, D]: only the sampled sequences and KV heads
        kk = torch.stack([k_cache[i][:, kv_heads] for i in seqs])
        vv = torch.stack([v_cache[i][:, kv_heads] for i in seqs])
    else:   # gather each sequence's pages into a contiguous [n, S, g, D] cache
        kk = torch.stack([k_cache[block_tables[i].long()][:, :, kv_heads].flatten(0, 1)
                          for i in seqs])
        vv = torch.stack([v_cache[block_tables[i].long()][:, :, kv_heads].flatten(0, 1)
                          for i in seqs])
    n = int(lens.max())
    ref, ref_lse = oracle.decode(q3[seqs][:, heads].double().cpu().numpy(),
                                 kk[:, :n].double().cpu().numpy(),
                                 vv[:, :n].double().cpu().numpy(), lens, softmax_scale=scale,
                                 return_lse=True)
    got = o[seqs][:, heads].double().cpu().numpy()
    got_lse = lse[seqs][:, heads].double().cpu().numpy()
    err = float(np.abs(got - ref).max())
    lse_err = float(np.abs(got_lse - ref_lse).max())
    if q3.dtype == torch.float32:   # fp32 output: no 16-bit rounding term; fixed bounds
        bound, lse_tol = 1e-5, 1e-5
    else:
        bound, lse_tol = 2 * _round_err(ref, q3.dtype), 1e-3
    return {"max_err_vs_ref64": err, "2x_rounding" if q3.dtype != torch.float32 else "bound":
            bound, "lse_err": lse_err,
            "correct": bool(np.isfinite(got).all() and err <= bound and lse_err <= lse_tol),
            "checked": f"sequences {list(seqs)} x KV heads {list(kv_heads)} ({len(heads)} "
                       f"query heads, lengths {lens.tolist()})"}


def merge_checks(parts: list) -> dict:
    """One rank's or several ranks' check results as one entry."""
    parts = [p for p in parts if p]
    if not parts:
        return {"correct": True, "checked": "nothing on this rank"}
    out = {"correct": all(p["correct"] for p in parts),
           "max_err_vs_ref64": max(p["max_err_vs_ref64"] for p in parts),
           "lse_err": max(p["lse_err"] for p in parts), "checked": parts[0]["checked"]}
    for key in ("2x_rounding", "bound"):
        if key in parts[0]:
            out[key] = min(p[key] for p in parts)
    if len(parts) > 1:
        out["checked"] = f"{len(parts)} checks, e.g. {parts[0]['checked']}"
    return out


def gather_checks(check: dict, dist) -> dict:
    """Every rank's check on rank 0 (collective)."""
    if dist is None:
        return check
    allc = [None] * dist.get_world_size()
    dist.all_gather_object(allc, check)
    merged = merge_checks(allc)
    merged["ranks"] = len(allc)
    return merged


# ------------------------------------------------------------------------------------------------
# CPU baselines (the oracle, i.e. the reference's algorithm in fp64, on this host's cores)
# ------------------------------------------------------------------------------------------------

def cpu_baseline_prefill(rows: int = CPU_SAMPLE_ROWS) -> dict:
    """The oracle (numpy fp64) on `rows` sampled query rows of the prefill workload."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    b, h, s, d = PREFILL["batch"], PREFILL["heads"], PREFILL["seqlen"], PREFILL["head_dim"]
    q = rng.standard_normal((b, s, h, d)).astype(np.float32)
    k = rng.standard_normal((b, s, h, d)).astype(np.float32)
    v = rng.standard_normal((b, s, h, d)).astype(np.float32)
    sample = np.sort(rng.choice(s, size=rows, replace=False))
    t0 = time.perf_counter()
    oracle.attention_rows(q, k, v, sample, causal=False, softmax_scale=1 / math.sqrt(d))
    dt = time.perf_counter() - t0
    flops = 4.0 * b * h * rows * s * d
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": host_cores(), "kind": "port",
            "sample": f"oracle.attention_rows, {rows} of 4096 query rows x all 128 (b,h), "
                      f"non-causal, fp64 numpy (BLAS threads = host cores), {dt:.2f} s",
            "seconds": dt}


def cpu_baseline_decode(heads: int, heads_kv: int, length: int) -> dict:
    """oracle.decode (fp64, the reference's decode) on one sequence of `length` keys and a
    quarter of the KV heads (with their query heads) of a decode configuration; GB/s counts the
    16-bit cache bytes that sample covers, as the device line does."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(1)
    d = 128
    g = max(1, heads_kv // 4)
    hq = g * (heads // heads_kv)
    q = rng.standard_normal((1, hq, d)).astype(np.float32)
    k = rng.standard_normal((1, length, g, d)).astype(np.float32)
    v = rng.standard_normal((1, length, g, d)).astype(np.float32)
    t0 = time.perf_counter()
    oracle.decode(q, k, v, np.array([length]), softmax_scale=1 / math.sqrt(d))
    dt = time.perf_counter() - t0
    nbytes = decode_bytes(hq, g, d, [length], 1)
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": host_cores(), "kind": "port",
            "sample": f"oracle.decode fp64, 1 sequence x {length} keys x {g} of {heads_kv} KV "
                      f"heads ({hq} query heads), {dt:.2f} s"}


def cpu_c0() -> dict:
    """The CPU-plumbing configuration: the oracle's fp64 attention at (B, H, H_kv, S, D) =
    (1, 4, 4, 256, 64), non-causal and causal, on this host's cores (median of 5)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    b, h, s, d = C0["batch"], C0["heads"], C0["seqlen"], C0["head_dim"]
    out = {"config": "(B,H,H_kv,S,D)=(1,4,4,256,64) fp64, scale 1/8, oracle.attention with LSE",
           "cores": host_cores()}
    q, k, v = (rng.standard_normal((b, s, h, d)) for _ in range(3))
    for causal in (False, True):
        times = []
        for _ in range(5):
            t0 = time.perf_counter()
            oracle.attention(q, k, v, causal=causal, softmax_scale=0.125, return_lse=True)
            times.append((time.perf_counter() - t0) * 1e3)
        out["causal_ms" if causal else "noncausal_ms"] = statistics.median(times)
    return out


def run_reference_arm(args) -> None:
    """--impl reference: the oracle port of the reference's CPU path, rank 0 only. One step is
    one bounded sample (REFERENCE_STEP_ROWS query rows of the workload); ms_per_step is its
    measured time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    times = []
    for _ in range(max(args.warmup, 0)):
        cpu_baseline_prefill(rows=REFERENCE_STEP_ROWS)
    for _ in range(args.steps):
        times.append(cpu_baseline_prefill(rows=REFERENCE_STEP_ROWS))
    value = statistics.median(t["value"] for t in times)
    sec = statistics.median(t["seconds"] for t in times)
    b = PREFILL
    full_ms = prefill_flops(b["batch"], b["heads"], b["seqlen"], b["seqlen"], b["head_dim"],
                            False) / (value * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "prefill (B,H,H_kv,S,D)=(4,32,32,4096,128) non-causal",
                   "sample": f"{REFERENCE_STEP_ROWS} query rows per step (all 128 (b,h), 4096 keys)",
                   "ms_per_step_is": "measured time of one sampled step",
                   "full_call_ms_extrapolated": full_ms},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": times[0]["cores"],
                         "kind": "port", "sample": times[0]["sample"] + f"; median {sec:.2f} s"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


_JSON_OUT = None


def emit(line: dict) -> None:
    """Writes the one JSON result line to the real stdout (everything else goes to stderr)."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def _claim_stdout() -> None:
    """Points file descriptor 1 at stderr so library chatter (NCCL's banner, warnings) cannot
    precede the result line, and keeps the original stdout for emit()."""
    global _JSON_OUT
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    _JSON_OUT = os.fdopen(saved, "w", buffering=1)
    sys.stdout = sys.stderr


def log(msg: str) -> None:
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------------------------
# The sharded prefill step and its end-to-end (host buffers) form
# ------------------------------------------------------------------------------------------------

def shard_views(q, k, v, pieces):
    """Zero-copy (q, k, v) views of each piece."""
    grp = q.shape[2] // k.shape[2]
    return [(q[p.b0:p.b1, :, p.g0 * grp:p.g1 * grp], k[p.b0:p.b1, :, p.g0:p.g1],
             v[p.b0:p.b1, :, p.g0:p.g1]) for p in pieces]


class HostPipeline:
    """One e2e step over this rank's pieces with pinned host buffers (the shard a serving caller
    holds on the host). Per piece and sequence: K and V go to the device first (copy stream),
    then the queries in E2E_Q_ROWS-row chunks; each chunk is attended against the full K / V
    (compute stream; non-causal rows are independent, so the chunks give the full result) and
    its output goes back (second copy stream) while later chunks still arrive. Every byte
    crosses PCIe inside the step, which ends when the last result is on the host."""

    def __init__(self, torch, flash_lab, views, scale, device):
        self.torch, self.fl, self.scale, self.device = torch, flash_lab, scale, device
        self.parts = []
        for q, k, v in views:
            hq, hk, hv = (x.contiguous().cpu().pin_memory() for x in (q, k, v))
            b, s, h, _ = q.shape
            self.parts.append(dict(
                hq=hq, hk=hk, hv=hv,
                ho=torch.empty(hq.shape, dtype=q.dtype).pin_memory(),
                hl=torch.empty((b, h, s), dtype=torch.float32).pin_memory(),
                dq=torch.empty_like(hq, device=device), dk=torch.empty_like(hk, device=device),
                dv=torch.empty_like(hv, device=device),
                dl=torch.empty((b, h, s), device=device, dtype=torch.float32)))
        self.s_in = torch.cuda.Stream(device)
        self.s_out = torch.cuda.Stream(device)

    @property
    def h2d_bytes(self) -> int:
        return sum((p["hq"].numel() + p["hk"].numel() + p["hv"].numel()) * p["hq"].element_size()
                   for p in self.parts)

    @property
    def d2h_bytes(self) -> int:
        return sum(p["ho"].numel() * p["ho"].element_size() + p["hl"].numel() * 4
                   for p in self.parts)

    def step(self):
        torch = self.torch
        compute = torch.cuda.current_stream(self.device)
        self.s_in.wait_stream(compute)      # the previous step no longer reads dq, dk, dv
        self.s_out.wait_stream(compute)     # nor is it copying out of dl
        for p in self.parts:
            b, s = p["hq"].shape[:2]
            rows = min(E2E_Q_ROWS, s)
            for i in range(b):
                with torch.cuda.stream(self.s_in):
                    p["dk"][i].copy_(p["hk"][i], non_blocking=True)
                    p["dv"][i].copy_(p["hv"][i], non_blocking=True)
                for r0 in range(0, s, rows):
                    r1 = min(s, r0 + rows)
                    with torch.cuda.stream(self.s_in):
                        p["dq"][i, r0:r1].copy_(p["hq"][i, r0:r1], non_blocking=True)
                    compute.wait_stream(self.s_in)
                    o, lse = self.fl.attention(p["dq"][i:i + 1, r0:r1], p["dk"][i:i + 1],
                                               p["dv"][i:i + 1], causal=False,
                                               softmax_scale=self.scale, return_lse=True)
                    p["dl"][i, :, r0:r1].copy_(lse[0])
                    self.s_out.wait_stream(compute)
                    with torch.cuda.stream(self.s_out):
                        p["ho"][i:i + 1, r0:r1].copy_(o, non_blocking=True)
                    o.record_stream(self.s_out)
                with torch.cuda.stream(self.s_out):
                    p["hl"][i].copy_(p["dl"][i], non_blocking=True)
        compute.wait_stream(self.s_out)      # the step ends with the last result on the host


# ------------------------------------------------------------------------------------------------
# main
# ------------------------------------------------------------------------------------------------

def main() -> int:
    _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary configurations")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-llama", action="store_true",
                    help="skip the Llama-3.1-8B-architecture generation in the extras")
    ap.add_argument("--profile", default=None,
                    choices=["prefill", "prefill_causal", "decode_mha", "decode_gqa",
                             "decode_gqa_ragged", "decode_gqa_ragged_paged16"],
                    help="run only warmup + steps launches of one kernel (for ncu captures)")
    ap.add_argument("--batch", type=int, default=None, help="batch size of --profile")
    ap.add_argument("--e2e-llama", action="store_true",
                    help="only the end-to-end Llama-3.1-8B-architecture generation")
    ap.add_argument("--host-time", action="store_true",
                    help="only the host time of eager decode calls (short-context latency)")
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=8192)
    args = ap.parse_args()
    if args.profile is not None:
        return run_profile_case(args)
    if args.e2e_llama:
        emit(run_e2e_llama(args))
        return 0
    if args.host_time:
        emit(run_host_time())
        return 0
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
        return 0

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
        # The ranks' oracle checks share the host: split its cores among them.
        try:
            from threadpoolctl import threadpool_limits

            threadpool_limits(max(1, host_cores() // world))
        except ImportError:
            pass
        torch.set_num_threads(max(1, host_cores() // world))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)

    import flash_lab
    from flash_lab import ops
    from flash_lab.distributed import attention_sharded, prefill_pieces

    if not ops.HAS_EXTENSION:
        raise SystemExit(f"the sm_100a library did not load: {ops.EXTENSION_ERROR}")
    peaks = load_peaks()
    traffic = load_traffic()

    b, h, hkv, s, d = (PREFILL[x] for x in ("batch", "heads", "heads_kv", "seqlen", "head_dim"))
    gen = torch.Generator(device=device).manual_seed(1234)     # one problem, the same on all ranks
    q = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    scale = 1.0 / math.sqrt(d)
    pieces = prefill_pieces(b, hkv, world, rank)
    views = shard_views(q, k, v, pieces)
    flops = prefill_flops(b, h, s, s, d, False)
    rank_flops = sum(prefill_flops(qq.shape[0], qq.shape[2], s, s, d, False) for qq, _, _ in views)

    def step():
        for qq, kk, vv in views:
            flash_lab.attention(qq, kk, vv, causal=False, softmax_scale=scale)

    # Check the call that is timed: this rank's pieces against the oracle, and (N > 1) the
    # gathered shards bit for bit against one unsharded call.
    log(f"rank {rank}/{world}: {len(pieces)} prefill piece(s) {pieces}")
    sp = attention_sharded(q, k, v, causal=False, softmax_scale=scale, world_size=world, rank=rank)
    rows = sample_rows(s, CHECK_ROWS, seed=7)
    checks = [check_prefill(o, lse, qq, kk, vv, False, scale, rows)
              for (o, lse), (qq, kk, vv) in zip(sp.outputs, views)]
    check = gather_checks(merge_checks(checks), dist)
    if world > 1:
        o_all, lse_all = sp.gather()
        same = True
        if rank == 0:
            o_one, lse_one = flash_lab.attention(q, k, v, causal=False, softmax_scale=scale,
                                                 return_lse=True)
            same = bool(torch.equal(o_all, o_one) and torch.equal(lse_all, lse_one))
            del o_one, lse_one
        if rank == 0:
            check["sharded_equals_one_call_bitwise"] = same
            check["correct"] = check["correct"] and same
        del o_all, lse_all
    del sp
    log(f"prefill check: {check}")

    with ClockSampler(local_rank) as clocks:
        ms_rank, ms = time_steps(step, args.steps, args.warmup, dist, device)
    value = flops / (ms * 1e-3) / 1e12
    log(f"prefill: {ms:.4f} ms per step (max over ranks), {value:.1f} TFLOP/s")

    # End to end through the public API with pinned host buffers of this rank's shard.
    pipe = HostPipeline(torch, flash_lab, views, scale, device)
    _, e2e_ms = time_steps(pipe.step, max(3, args.steps // 4), 3, dist, device)
    torch.cuda.synchronize(device)
    e2e_same = all(torch.equal(p["ho"], o.cpu()) and torch.equal(p["hl"], lse.cpu())
                   for p, (o, lse) in zip(pipe.parts,
                                          (flash_lab.attention(qq, kk, vv, causal=False,
                                                               softmax_scale=scale,
                                                               return_lse=True)
                                           for qq, kk, vv in views)))
    e2e_same = gather_checks({"correct": e2e_same, "max_err_vs_ref64": 0.0, "lse_err": 0.0,
                              "checked": "host output vs the device call"}, dist)["correct"]
    e2e = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": pipe.h2d_bytes, "d2h_bytes_per_step": pipe.d2h_bytes,
           "per": "rank (the whole job moves world x these bytes)",
           "host_output_equals_device_call": e2e_same,
           "pipeline": f"per sequence K/V, then {E2E_Q_ROWS}-row query chunks: h2d (copy "
                       "stream) | attention (compute) | d2h (copy stream)"}
    del pipe

    achieved = rank_flops / (ms_rank * 1e-3) / 1e12 if rank_flops else 0.0
    tr = traffic.get("prefill_kernel_noncausal")
    units = sum(p.units for p in pieces)
    roofline = {"kernel": "prefill_kernel<bf16> (tcgen05)", "bound": "tensor",
                "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "traffic": (tr["bytes_per_launch"] * units / (b * hkv)) if tr else None,
                "peak_source": f"{peaks['source']} bf16_tflops (burst, kernel timed alone)",
                "algorithmic": f"{rank_flops:.4e} FLOP per step on rank 0 (4*B*H*S^2*D over its "
                               f"{units} (b, KV head) units)"}

    extra = {}
    ok = check["correct"] and e2e_same
    if not args.no_extra:
        extra = run_extra(torch, flash_lab, device, dist, world, rank, args, peaks, traffic)
        ok = ok and all(v.get("check", {}).get("correct", True) for v in extra.values()
                        if isinstance(v, dict))

    if rank == 0:
        cpu = None if args.no_cpu or world > 1 else cpu_baseline_prefill()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "prefill (B,H,H_kv,S,D)=(4,32,32,4096,128) bf16 non-causal",
                       "sharding": f"(batch, KV head) units over {world} GPU(s), rank 0 runs "
                                   f"{units} of {b * hkv}; no communication in the step",
                       "l2": "inputs 402 MB > 126 MB L2, no flush", "seed": 1234},
            "correct": check["correct"] and e2e_same,
            "check": check,
            "clocks": clocks.summary(),
            "e2e": e2e,
            "gpu_launches": args.steps * len(pieces),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "extra": extra,
        }
        emit(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if not ok:
        log("a correctness check failed (see the line's check entries)")
        return 1
    return 0


def run_extra(torch, flash_lab, device, dist, world, rank, args, peaks, traffic) -> dict:
    """Secondary configurations: causal prefill, the 32K decode configurations, the B=1 decode
    split over the ranks, the CPU-plumbing configuration and the e2e generation."""
    from flash_lab.distributed import attention_sharded, prefill_pieces

    out = {}

    def prefill_case(b, h, hkv, s, d, causal, seed, check_seed):
        """One secondary prefill configuration, sharded like the headline: oracle check on
        sampled rows, then the device-timed step (max over ranks)."""
        gen = torch.Generator(device=device).manual_seed(seed)
        q = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
        k = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
        v = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
        scale = 1.0 / math.sqrt(d)
        pieces = prefill_pieces(b, hkv, world, rank)
        views = shard_views(q, k, v, pieces)
        sp = attention_sharded(q, k, v, causal=causal, world_size=world, rank=rank)
        rows = sample_rows(s, CHECK_ROWS, seed=check_seed)
        check = gather_checks(merge_checks([check_prefill(o, lse, qq, kk, vv, causal, scale, rows)
                                            for (o, lse), (qq, kk, vv) in zip(sp.outputs, views)]),
                              dist)
        del sp
        flops = prefill_flops(b, h, s, s, d, causal)
        rank_flops = sum(prefill_flops(qq.shape[0], qq.shape[2], s, s, d, causal)
                         for qq, _, _ in views)

        def step():
            for qq, kk, vv in views:
                flash_lab.attention(qq, kk, vv, causal=causal, softmax_scale=scale)

        ms_rank, ms = time_steps(step, args.steps, args.warmup, dist, device)
        achieved = rank_flops / (ms_rank * 1e-3) / 1e12 if rank_flops else 0.0
        return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
                "roofline_frac": achieved / peaks["bf16_tflops"], "flop_per_call": flops,
                "scaling": "strong", "check": check}

    b, h, hkv, s, d = (PREFILL[x] for x in ("batch", "heads", "heads_kv", "seqlen", "head_dim"))
    res = prefill_case(b, h, hkv, s, d, True, 99, 8)
    tr = traffic.get("prefill_kernel_causal")
    res["traffic"] = tr.get("bytes_per_launch") if tr else None
    out["prefill_causal"] = res
    log(f"prefill causal: {out['prefill_causal']}")
    # head_dim 64, the reference's other head size, at the same tokens per launch (B = 8).
    for causal in (False, True):
        key = "prefill_d64_causal" if causal else "prefill_d64"
        res = prefill_case(2 * b, h, hkv, s, 64, causal, 77, 9)
        res["config"] = f"(B,H,H_kv,S,D)=({2 * b},{h},{hkv},{s},64) bf16 causal={causal}"
        out[key] = res
        log(f"{key}: {res}")

    l2_flush = torch.empty(512 * 2**20, dtype=torch.uint8, device=device)
    l2_drain = torch.zeros(128 * 2**20, dtype=torch.float32, device=device)   # 512 MB

    def flush_l2():
        # Write a 512 MB buffer (4x L2), then read another: the written lines are dirty, and
        # without the read pass their write-back would land inside the next timed call.
        l2_flush.zero_()
        l2_drain.sum()

    def time_calls(fn, steps, warmup):
        """Median CUDA-event time of fn with L2 flushed before every call (outside the events),
        max over ranks."""
        times = []
        for i in range(warmup + steps):
            flush_l2()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            fn()
            en.record()
            if i >= warmup:
                times.append((st, en))
        torch.cuda.synchronize(device)
        return max_over_ranks(statistics.median(a.elapsed_time(z) for a, z in times), dist,
                              device)

    # (batch, heads, heads_kv, lengths, cache dtype, page size or 0 for a contiguous cache).
    # N > 1: rank r decodes sequences [r B / N, (r + 1) B / N) of the one seeded batch.
    for name, (bb, hh, hk, lens_kind, cdt, page) in {
        "decode_mha_32k": (8, 32, 32, "full", torch.bfloat16, 0),
        "decode_gqa_32k": (8, 32, 8, "ragged", torch.bfloat16, 0),
        "decode_gqa_32k_paged16": (8, 32, 8, "ragged", torch.bfloat16, 16),
        "decode_mha_32k_fp32": (4, 32, 32, "full", torch.float32, 0),
    }.items():
        smax = 32768
        gen = torch.Generator(device=device).manual_seed(7)
        qd = torch.randn(bb, 1, hh, d, device=device, dtype=cdt, generator=gen)
        kc = torch.randn(bb, smax, hk, d, device=device, dtype=cdt, generator=gen)
        vc = torch.randn(bb, smax, hk, d, device=device, dtype=cdt, generator=gen)
        tables = None
        if page:
            # The same cache as a pool of pages in a shuffled order (the reference's paged layout).
            nb = smax // page
            perm = torch.randperm(bb * nb, device=device, generator=gen)
            kc = kc.view(bb * nb, page, hk, d)[torch.argsort(perm)]
            vc = vc.view(bb * nb, page, hk, d)[torch.argsort(perm)]
            tables = perm.view(bb, nb).to(torch.int32)
        if lens_kind == "full":
            lens = [smax] * bb
        else:
            lens = torch.randint(16384, smax + 1, (bb,),
                                 generator=torch.Generator().manual_seed(0)).tolist()
        seq_lens = torch.tensor(lens, device=device, dtype=torch.int32)
        s0, s1 = rank * bb // world, (rank + 1) * bb // world
        nbytes = decode_bytes(hh, hk, d, lens, bb) * (2 if cdt == torch.float32 else 1)
        entry = {"unit": "GB/s", "bytes_per_call": nbytes, "scaling": "strong",
                 "peak_gbs": peaks["hbm_gbs"],
                 "config": f"B={bb} H={hh} H_kv={hk} S_max=32768 D=128 "
                           f"{str(cdt).removeprefix('torch.')} "
                           f"lengths={'32768' if lens_kind == 'full' else lens}"
                           + (f" paged: {page}-row pages in a shuffled pool" if page else "")
                           + (f"; sequences sharded over {world} GPUs" if world > 1 else ""),
                 "l2": "512 MB buffer written, then another 512 MB read, before every call "
                       "(outside the events)"}
        if s1 > s0:
            qr, lr = qd[s0:s1], seq_lens[s0:s1]
            kr = kc if page else kc[s0:s1]
            vr = vc if page else vc[s0:s1]
            tr_ = tables[s0:s1] if page else None
            rank_bytes = decode_bytes(hh, hk, d, lens[s0:s1], s1 - s0) * \
                (2 if cdt == torch.float32 else 1)

            def call():
                return flash_lab.decode(qr, kr, vr, lr, block_tables=tr_, return_lse=True)

            o, lse = call()
            picks = sorted({0, s1 - s0 - 1})
            chk = check_decode(o[:, 0], lse, qr[:, 0], kr, vr, lr, 1 / math.sqrt(d), picks,
                               sorted({0, hk - 1}), block_tables=tr_)
            del o, lse
        else:
            rank_bytes, chk = 0.0, None

            def call():
                return None
        entry["check"] = gather_checks(merge_checks([chk]), dist)
        ms = time_calls(call, args.steps, args.warmup)
        rank_ms = ms
        entry.update(value=nbytes / (ms * 1e-3) / 1e9, ms_per_step=ms,
                     roofline_frac=(rank_bytes / (rank_ms * 1e-3) / 1e9) / peaks["hbm_gbs"]
                     if rank_bytes else None)

        if s1 > s0:
            # End to end: q and seq_lens from pinned host memory, o and lse back to it; the
            # cache stays resident in HBM (a KV cache is device state).
            hq = qr.cpu().pin_memory()
            hl = lr.cpu().pin_memory()
            ho = torch.empty(qr.shape, dtype=cdt).pin_memory()
            hlse = torch.empty((s1 - s0, hh), dtype=torch.float32).pin_memory()
            dq, dl = torch.empty_like(qr), torch.empty_like(lr)

            def e2e_call():
                dq.copy_(hq, non_blocking=True)
                dl.copy_(hl, non_blocking=True)
                o, lse = flash_lab.decode(dq, kr, vr, dl, block_tables=tr_, return_lse=True)
                ho.copy_(o, non_blocking=True)
                hlse.copy_(lse, non_blocking=True)

            e2e_ms = time_calls(e2e_call, args.steps, args.warmup)
            entry["e2e"] = {"value": nbytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                            "ms_per_step": e2e_ms,
                            "h2d_bytes_per_step": hq.numel() * hq.element_size() + hl.numel() * 4,
                            "d2h_bytes_per_step": ho.numel() * ho.element_size() +
                            hlse.numel() * 4,
                            "how": "q and seq_lens host->device, decode, o and lse "
                                   "device->host, per call; the cache is resident"}
        else:
            time_calls(lambda: None, args.steps, args.warmup)   # same collectives as the others
        if rank == 0 and world == 1 and not args.no_cpu and name in ("decode_mha_32k",
                                                                     "decode_gqa_32k"):
            entry["cpu_baseline"] = cpu_baseline_decode(hh, hk, 32768)
        out[name] = entry
        log(f"{name}: {entry}")
        del qd, kc, vc, tables

    out.update(run_b1_split(torch, device, dist, world, rank, args, peaks, flush_l2))
    if rank == 0 and world == 1 and not args.no_cpu:
        out["c0_cpu_reference"] = cpu_c0()
    if rank == 0 and world == 1 and not args.no_llama:
        try:
            del l2_flush, l2_drain
            torch.cuda.empty_cache()
            out["e2e_llama"] = run_e2e_llama(args)
        except Exception as exc:  # noqa: BLE001 - report, do not lose the line
            out["e2e_llama"] = {"error": f"{type(exc).__name__}: {exc}"}
    return out


def run_b1_split(torch, device, dist, world, rank, args, peaks, flush_l2) -> dict:
    """B=1 MHA at 32K with the KV sequence split across the ranks. decode_b1_split: the peer
    exchange (each rank's split kernel pushes its partials into every rank's buffer over
    NVLink, then a bounded device wait and the fixed-order merge). decode_b1_split_allgather:
    per-rank partials, NCCL all_gather, merge. On one rank both are the plain split decode.
    Checked against the oracle (a head subset) and, bit for bit, against the same global split
    windows computed on one GPU."""
    from flash_lab.distributed import (PeerExchange, ShardSpec, decode_sharded,
                                       default_splits_per_rank, merge_partials, shard_partials)

    out = {}
    d, smax, hh, hk = 128, 32768, 32, 32
    shard = ShardSpec.even(smax, world, rank)
    gen = torch.Generator(device=device).manual_seed(17)  # same cache on every rank
    qd = torch.randn(1, hh, d, device=device, dtype=torch.bfloat16, generator=gen)
    full_k = torch.randn(1, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
    full_v = torch.randn(1, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
    k_shard = full_k[:, shard.offset:shard.offset + shard.length].contiguous()
    v_shard = full_v[:, shard.offset:shard.offset + shard.length].contiguous()
    seq_lens = torch.full((1,), smax, device=device, dtype=torch.int32)
    sm = torch.cuda.get_device_properties(device).multi_processor_count
    splits = default_splits_per_rank(1, hh, hk, shard.length, sm)
    scale = 1 / math.sqrt(d)
    # One-GPU result of the same global split windows: every shard's partials from the full
    # cache on this GPU, in rank order, then the merge.
    pos, pmls = [], []
    for r in range(world):
        sh = ShardSpec.even(smax, world, r)
        po, pml = shard_partials(qd, full_k[:, sh.offset:sh.offset + sh.length],
                                 full_v[:, sh.offset:sh.offset + sh.length], seq_lens, sh.offset,
                                 splits, scale)
        pos.append(po)
        pmls.append(pml)
    o_one, lse_one = merge_partials(torch.cat(pos, dim=2), torch.cat(pmls, dim=2), torch.bfloat16)
    nbytes = decode_bytes(hh, hk, d, [smax], 1)
    exchange = PeerExchange(1, hh, d, splits_per_rank=splits) if world > 1 else None
    try:
        for name, ex, how in (("decode_b1_split", exchange, "partials pushed into every rank's "
                               "buffer over NVLink peer memory, bounded device wait, merge"
                               if world > 1 else "local partials and merge"),
                              ("decode_b1_split_allgather", None, "partials all-gathered over "
                               "NCCL, merge" if world > 1 else "local partials and merge")):
            o, lse = decode_sharded(qd, k_shard, v_shard, seq_lens, shard,
                                    splits_per_rank=splits, exchange=ex, return_lse=True)
            same = bool(torch.equal(o, o_one) and torch.equal(lse, lse_one))
            chk = check_decode(o, lse, qd, full_k, full_v, seq_lens, scale, [0], [0, 11, 22, 31])
            chk["equals_one_gpu_bitwise"] = same
            chk["correct"] = chk["correct"] and same
            times = []
            tick = torch.zeros(1, device=device)
            for i in range(args.warmup + args.steps):
                flush_l2()
                if dist is not None:
                    # Device-side rendezvous: the ranks' streams leave the all_reduce together,
                    # so host launch skew stays out of the time.
                    dist.all_reduce(tick)
                # ~100 us of device sleep: the host enqueues the whole call before the start
                # event fires, so the events time the device work, not Python launch overhead.
                torch.cuda._sleep(200_000)
                st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                st.record()
                decode_sharded(qd, k_shard, v_shard, seq_lens, shard, splits_per_rank=splits,
                               exchange=ex)
                en.record()
                if i >= args.warmup:
                    times.append((st, en))
            torch.cuda.synchronize(device)
            ms = max_over_ranks(statistics.median(a.elapsed_time(z) for a, z in times), dist,
                                device)
            if ex is not None and ex.read_status() != 0:
                chk["correct"] = False
                chk["exchange_status"] = "a peer-exchange wait timed out"
            gbs = nbytes / (ms * 1e-3) / 1e9
            out[name] = {
                "value": gbs, "unit": "GB/s", "ms_per_step": ms, "bytes_per_call": nbytes,
                "per_gpu_roofline_frac": gbs / world / peaks["hbm_gbs"], "scaling": "strong",
                "config": f"B=1 H=H_kv=32 D=128 32K keys split over {world} GPU(s), {splits} "
                          f"splits per GPU, {how} in a fixed order",
                "l2": "512 MB buffer written, then another 512 MB read, before every call "
                      "(outside the events)",
                "check": gather_checks(chk, dist)}
            log(f"{name}: {out[name]}")
    finally:
        if exchange is not None:
            exchange.close()
    return out


def run_e2e_llama(args) -> dict:
    """The e2e configuration: Llama-3.1-8B architecture (32 layers, d_model 4096, 32 heads, 8 KV
    heads, head_dim 128, RoPE theta 500000, vocab 128256) with random-init bf16 weights, batch 1,
    a random 8192-token prompt, 256 greedy tokens, a static KV cache and the decode step compiled
    (torch.compile, CUDA graphs), attention through the flash_lab HF backend; the same run with
    transformers' SDPA backend beside it, and the greedy tokens of the two compared."""
    import torch
    from transformers import CompileConfig, LlamaConfig, LlamaForCausalLM, StaticCache

    import flash_lab.hf

    t_start = time.perf_counter()
    flash_lab.hf.register()
    device = torch.device("cuda", 0)
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rope_theta=500000.0, max_position_embeddings=131072)
    torch.manual_seed(0)
    with torch.device(device):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16)
    model = model.eval()
    ids = torch.randint(0, 128000, (1, args.prompt_len),
                        generator=torch.Generator().manual_seed(0)).to(device)
    mask = torch.ones_like(ids)
    max_len = args.prompt_len + args.new_tokens
    results = {}
    tokens = {}
    for attn in ("flash_lab", "sdpa"):
        model.config._attn_implementation = attn
        torch._dynamo.reset()
        cache = StaticCache(config=cfg, max_cache_len=max_len)

        def generate(n):
            cache.reset()
            return model.generate(ids, attention_mask=mask, max_new_tokens=n, do_sample=False,
                                  past_key_values=cache, pad_token_id=0, min_new_tokens=n,
                                  compile_config=CompileConfig(fullgraph=True))

        with torch.no_grad():
            t0 = time.perf_counter()
            generate(16)        # compiles the decode step
            generate(16)
            warm_s = time.perf_counter() - t0

            def timed(n):
                torch.cuda.synchronize()
                st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                st.record()
                out = generate(n)
                en.record()
                torch.cuda.synchronize()
                return st.elapsed_time(en), out

            ttft = min(timed(1)[0] for _ in range(3))
            total, out = timed(args.new_tokens)
        results[attn] = {"ttft_ms": ttft, "total_ms": total,
                         "decode_step_ms": (total - ttft) / (args.new_tokens - 1),
                         "compile_and_warmup_s": warm_s}
        tokens[attn] = out[0, ids.shape[1]:].tolist()
    agree = sum(1 for a, b in zip(tokens["flash_lab"], tokens["sdpa"]) if a == b)
    first_diff = next((i for i, (a, b) in enumerate(zip(tokens["flash_lab"], tokens["sdpa"]))
                       if a != b), None)
    del model
    torch.cuda.empty_cache()
    return {"metric": "e2e Llama-3.1-8B arch: decode step ms / TTFT ms (lower is better)",
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic (random init, "
            "random prompt)", "config": {"model": "Llama-3.1-8B architecture",
            "prompt_len": args.prompt_len, "new_tokens": args.new_tokens, "batch": 1,
            "cache": "static", "decode": "torch.compile, CUDA graphs (transformers turns "
            "fullgraph off for attention backends named flash*)"},
            "flash_lab": results["flash_lab"], "sdpa": results["sdpa"],
            "greedy_tokens_equal": agree, "greedy_tokens": args.new_tokens,
            "first_divergence": first_diff,
            "wall_s": time.perf_counter() - t_start}


def run_host_time() -> dict:
    """Host time of an eager flash_lab.decode call at short contexts (B=1 and B=8, H=32, head_dim
    128, 512 to 4096 keys): 400 back-to-back calls after warm-up, best of five windows, with the
    device time of the same call (a CUDA-graph replay) beside it. The host time is the cost of
    the Python API, its validation and the launch; above the device time, a short-context decode
    loop that does not capture graphs is bound by the host."""
    import torch

    import flash_lab

    device = torch.device("cuda", 0)

    def per_call_us(fn, n=400, reps=5):
        best = float("inf")
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            t1 = time.perf_counter()
            torch.cuda.synchronize()
            best = min(best, (t1 - t0) / n * 1e6)
        return best

    rows = []
    for batch, heads_kv in ((1, 32), (8, 8)):
        for keys in (512, 2048, 4096):
            gen = torch.Generator(device=device).manual_seed(3)
            q = torch.randn(batch, 1, 32, 128, device=device, dtype=torch.bfloat16, generator=gen)
            kc = torch.randn(batch, keys, heads_kv, 128, device=device, dtype=torch.bfloat16,
                             generator=gen)
            lens = torch.full((batch,), keys, device=device, dtype=torch.int32)

            def call():
                return flash_lab.decode(q, kc, kc, lens)

            for _ in range(20):
                call()
            host = per_call_us(call)
            graph = torch.cuda.CUDAGraph()
            stream = torch.cuda.Stream(device)
            stream.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(stream):
                with torch.cuda.graph(graph, stream=stream):
                    call()
            torch.cuda.current_stream(device).wait_stream(stream)
            for _ in range(10):
                graph.replay()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            for _ in range(200):
                graph.replay()
            en.record()
            torch.cuda.synchronize(device)
            rows.append({"batch": batch, "heads": 32, "heads_kv": heads_kv, "keys": keys,
                         "host_us_per_call": host,
                         "device_us_per_call": st.elapsed_time(en) / 200 * 1e3})
            del graph
    return {"metric": "eager flash_lab.decode host time per call (us, lower is better)",
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic",
            "method": "400 back-to-back eager calls after 20 warm-up calls, best of 5 windows; "
                      "device time from 200 CUDA-graph replays of the same call",
            "rows": rows}


def run_profile_case(args) -> int:
    """A few launches of one kernel at a reduced batch, for Nsight Compute captures."""
    import torch

    import flash_lab

    device = torch.device("cuda", 0)
    gen = torch.Generator(device=device).manual_seed(0)
    d = 128
    if args.profile.startswith("prefill"):
        b = args.batch or 2
        s, h = PREFILL["seqlen"], PREFILL["heads"]
        q = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
        k = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
        v = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
        causal = args.profile == "prefill_causal"
        fn = lambda: flash_lab.attention(q, k, v, causal=causal)  # noqa: E731
        what = f"prefill B={b} H=32 S=4096 D=128 causal={causal}"
    else:
        b = args.batch or 2
        hk = 32 if args.profile == "decode_mha" else 8
        smax = 32768
        qd = torch.randn(b, 1, 32, d, device=device, dtype=torch.bfloat16, generator=gen)
        kc = torch.randn(b, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
        vc = torch.randn(b, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
        lens = torch.full((b,), smax, device=device, dtype=torch.int32)
        if args.profile.startswith("decode_gqa_ragged"):   # the bench's lengths, U[16384, 32768]
            lens = torch.randint(16384, smax + 1, (b,), generator=torch.Generator().manual_seed(0))
            lens = lens.to(device=device, dtype=torch.int32)
        tables = None
        if args.profile.endswith("paged16"):   # the bench's pool of 16-row pages, shuffled
            page, nb = 16, smax // 16
            perm = torch.randperm(b * nb, device=device, generator=gen)
            kc = kc.view(b * nb, page, hk, d)[torch.argsort(perm)]
            vc = vc.view(b * nb, page, hk, d)[torch.argsort(perm)]
            tables = perm.view(b, nb).to(torch.int32)
        fn = lambda: flash_lab.decode(qd, kc, vc, lens, block_tables=tables)  # noqa: E731
        what = f"decode B={b} H=32 H_kv={hk} S=32768 D=128 lengths={lens.tolist()}"
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(f"profile case done: {what}, {args.warmup + args.steps} calls")
    return 0


if __name__ == "__main__":
    sys.exit(main())
