"""Benchmark of flash_lab's attention path on B200 (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-extra]

Headline workload (the benchmark's prefill configuration): bf16 prefill forward, (B, H, H_kv, S, D) =
(4, 32, 32, 4096, 128), non-causal, Q/K/V ~ N(0, 1) from a seed, scale 1/sqrt(128). One step is
one flash_lab.attention call over that batch; metric TFLOP/s counts 4*B*H*S_q*S_k*D FLOP per
call (the reference's bench/flops.py convention). Inputs (402 MB) are larger than the 126 MB L2,
so no flush is needed between steps.

  value        whole-job TFLOP/s with inputs resident in HBM (sum over ranks / max rank time)
  e2e          the same work through the public API with pinned HOST inputs: each step copies
               q, k, v host->device, runs flash_lab.attention and copies o and lse back,
               pipelined over the batch (copies of one sequence overlap the next one's kernel)
  roofline     the prefill kernel: achieved FLOP/s from CUDA-event time over the timed region
               against the measured dense bf16 peak of MEASURED_PEAKS.json; traffic (DRAM bytes
               per launch) from the committed ncu capture in profiles/ when present
  cpu_baseline the oracle (numpy fp64 restatement of the reference's flash_lab/reference.py) on
               this host's cores, on 256 sampled query rows of the same workload (rank 0, N=1)
  extra        secondary configurations measured the same way on the device: causal prefill,
               decode B=8 H=H_kv=32 at 32K, GQA decode B=8 H_kv=8 with lengths U[16K, 32K]

Multi-GPU (torchrun, one rank per GPU): every rank runs the full workload on its own GPU with its
own seed (prefill shards over batch x heads with no communication), so scaling is weak.

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
E2E_Q_ROWS = 512   # query rows per host->device chunk of the e2e pipeline
METRIC = "prefill TFLOP/s @(4,32,32,4096,128) bf16; decode HBM GB/s @32K cache"
CPU_SAMPLE_ROWS = 1536
REFERENCE_STEP_ROWS = 256


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


def time_steps(fn, steps: int, warmup: int, dist=None, device=None):
    """Runs fn warmup times, then times exactly `steps` calls between CUDA events with a barrier
    and a synchronize on both sides. Returns (ms per step, max over ranks)."""
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
    if dist is not None:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


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
    cores = len(os.sched_getaffinity(0))
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"oracle.attention_rows, {rows} of 4096 query rows x all 128 (b,h), "
                      f"non-causal, fp64 numpy (BLAS threads = host cores), {dt:.2f} s",
            "seconds": dt}


def run_reference_arm(args) -> None:
    """--impl reference: the oracle port of the reference's CPU path, rank 0 only."""
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
        "ms_per_step": full_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "prefill (B,H,H_kv,S,D)=(4,32,32,4096,128) non-causal",
                   "sample": f"{REFERENCE_STEP_ROWS} query rows per step (all 128 (b,h), 4096 keys)",
                   "ms_per_step_is": "extrapolated time of one full call at the sampled rate"},
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


def main() -> int:
    _claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary configurations")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--profile", default=None,
                    choices=["prefill", "prefill_causal", "decode_mha", "decode_gqa",
                             "decode_gqa_ragged"],
                    help="run only warmup + steps launches of one kernel (for ncu captures)")
    ap.add_argument("--batch", type=int, default=None, help="batch size of --profile")
    ap.add_argument("--e2e-llama", action="store_true",
                    help="end-to-end Llama-3.1-8B-architecture generation (the e2e configuration)")
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--prompt-len", type=int, default=8192)
    args = ap.parse_args()
    if args.profile is not None:
        return run_profile_case(args)
    if args.e2e_llama:
        return run_e2e_llama(args)
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
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)

    import flash_lab
    from flash_lab import ops

    if not ops.HAS_EXTENSION:
        raise SystemExit(f"the sm_100a library did not load: {ops.EXTENSION_ERROR}")
    peaks = load_peaks()
    traffic = load_traffic()

    b, h, hkv, s, d = (PREFILL[x] for x in ("batch", "heads", "heads_kv", "seqlen", "head_dim"))
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    q = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    scale = 1.0 / math.sqrt(d)

    def step():
        flash_lab.attention(q, k, v, causal=False, softmax_scale=scale)

    flops = prefill_flops(b, h, s, s, d, False)
    with ClockSampler(local_rank) as clocks:
        ms = time_steps(step, args.steps, args.warmup, dist, device)
    value = world * flops / (ms * 1e-3) / 1e12

    # End to end through the public API with pinned host buffers.
    hq = q.cpu().pin_memory()
    hk = k.cpu().pin_memory()
    hv = v.cpu().pin_memory()
    ho = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    hl = torch.empty((b, h, s), dtype=torch.float32).pin_memory()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    # The step is pipelined as a serving caller would run it. Per sequence, its K and V go to
    # the device (copy stream), then its queries in chunks of E2E_Q_ROWS rows; each chunk is
    # attended against the full K / V (compute stream; non-causal rows are independent, so the
    # chunks give the full result) and its output goes back to the host (second copy stream)
    # while later chunks are still arriving. Small chunks keep the tail after the last
    # host->device copy short. Every byte still crosses PCIe inside the step, and the step ends
    # when the last result is on the host.
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dl = torch.empty((b, h, s), device=device, dtype=torch.float32)
    q_rows = min(E2E_Q_ROWS, s)

    def e2e_step():
        compute = torch.cuda.current_stream(device)
        s_in.wait_stream(compute)        # the previous step no longer reads dq, dk, dv
        s_out.wait_stream(compute)       # nor is it copying out of dl
        for i in range(b):
            with torch.cuda.stream(s_in):
                dk[i].copy_(hk[i], non_blocking=True)
                dv[i].copy_(hv[i], non_blocking=True)
            for r0 in range(0, s, q_rows):
                r1 = min(s, r0 + q_rows)
                with torch.cuda.stream(s_in):
                    dq[i, r0:r1].copy_(hq[i, r0:r1], non_blocking=True)
                compute.wait_stream(s_in)
                o, lse = flash_lab.attention(dq[i:i + 1, r0:r1], dk[i:i + 1], dv[i:i + 1],
                                             causal=False, softmax_scale=scale, return_lse=True)
                dl[i, :, r0:r1].copy_(lse[0])
                s_out.wait_stream(compute)
                with torch.cuda.stream(s_out):
                    ho[i:i + 1, r0:r1].copy_(o, non_blocking=True)
                o.record_stream(s_out)
            with torch.cuda.stream(s_out):
                hl[i].copy_(dl[i], non_blocking=True)
        compute.wait_stream(s_out)       # the step ends with the last result on the host

    e2e_ms = time_steps(e2e_step, max(3, args.steps // 4), 3, dist, device)
    # The pipelined step returns what one call on the whole resident batch returns, bit for bit.
    o_full, lse_full = flash_lab.attention(q, k, v, causal=False, softmax_scale=scale,
                                           return_lse=True)
    torch.cuda.synchronize(device)
    if not (torch.equal(ho, o_full.cpu()) and torch.equal(hl, lse_full.cpu())):
        raise SystemExit("e2e: the pipelined step's host output differs from the full call")
    del o_full, lse_full
    e2e = {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
           "ms_per_step": e2e_ms,
           "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2,
           "d2h_bytes_per_step": ho.numel() * 2 + hl.numel() * 4,
           "pipeline": f"per sequence K/V, then {q_rows}-row query chunks: h2d (copy stream) | "
                       "attention (compute) | d2h (copy stream)"}

    achieved = flops / (ms * 1e-3) / 1e12
    tr = traffic.get("prefill_kernel_noncausal")
    roofline = {"kernel": "prefill_kernel<bf16> (tcgen05)", "bound": "tensor",
                "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "traffic": tr.get("bytes_per_launch") if tr else None,
                "peak_source": f"{peaks['source']} bf16_tflops (burst, kernel timed alone)",
                "algorithmic": f"{flops:.4e} FLOP per launch (4*B*H*S^2*D)"}

    extra = {}
    if not args.no_extra:
        extra = run_extra(torch, flash_lab, device, dist, world, rank, args, peaks, traffic)

    if rank == 0:
        cpu = None if args.no_cpu or world > 1 else cpu_baseline_prefill()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "prefill (B,H,H_kv,S,D)=(4,32,32,4096,128) bf16 non-causal",
                       "per_gpu_batch": "full config per rank (sharded over batch x heads)",
                       "l2": "inputs 402 MB > 126 MB L2, no flush", "seed": "1234 + rank"},
            "clocks": clocks.summary(),
            "e2e": e2e,
            "gpu_launches": args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "extra": extra,
        }
        emit(line)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_extra(torch, flash_lab, device, dist, world, rank, args, peaks, traffic) -> dict:
    """Secondary configurations: causal prefill and the two 32K decode configurations."""
    out = {}
    b, h, hkv, s, d = (PREFILL[x] for x in ("batch", "heads", "heads_kv", "seqlen", "head_dim"))
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    q = torch.randn(b, s, h, d, device=device, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(b, s, hkv, d, device=device, dtype=torch.bfloat16, generator=gen)
    flops = prefill_flops(b, h, s, s, d, True)
    ms = time_steps(lambda: flash_lab.attention(q, k, v, causal=True), args.steps, args.warmup,
                    dist, device)
    achieved = flops / (ms * 1e-3) / 1e12
    tr = traffic.get("prefill_kernel_causal")
    out["prefill_causal"] = {"value": world * achieved, "unit": "TFLOP/s", "ms_per_step": ms,
                             "roofline_frac": achieved / peaks["bf16_tflops"],
                             "traffic": tr.get("bytes_per_launch") if tr else None,
                             "flop_per_call": flops}
    del q, k, v

    l2_flush = torch.empty(512 * 2**20, dtype=torch.uint8, device=device)
    l2_drain = torch.zeros(128 * 2**20, dtype=torch.float32, device=device)   # 512 MB

    def flush_l2():
        # Write a 512 MB buffer (4x L2), then read another: the written lines are dirty, and
        # without the read pass their write-back would land inside the next timed call.
        l2_flush.zero_()
        l2_drain.sum()

    # (batch, heads, heads_kv, lengths, cache dtype, page size or 0 for a contiguous cache)
    for name, (bb, hh, hk, lens_kind, cdt, page) in {
        "decode_mha_32k": (8, 32, 32, "full", torch.bfloat16, 0),
        "decode_gqa_32k": (8, 32, 8, "ragged", torch.bfloat16, 0),
        "decode_gqa_32k_paged16": (8, 32, 8, "ragged", torch.bfloat16, 16),
        "decode_mha_32k_fp32": (4, 32, 32, "full", torch.float32, 0),
    }.items():
        smax = 32768
        gen = torch.Generator(device=device).manual_seed(7 + rank)
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
        nbytes = decode_bytes(hh, hk, d, lens, bb) * (2 if cdt == torch.float32 else 1)

        # Kernel-only time with L2 flushed before every call (flush outside the events).
        times = []
        for i in range(args.warmup + args.steps):
            flush_l2()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            flash_lab.decode(qd, kc, vc, seq_lens, block_tables=tables)
            en.record()
            if i >= args.warmup:
                times.append((st, en))
        torch.cuda.synchronize(device)
        ms = statistics.median(st.elapsed_time(en) for st, en in times)
        if dist is not None:
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"value": world * gbs, "unit": "GB/s", "ms_per_step": ms,
                     "bytes_per_call": nbytes, "roofline_frac": gbs / peaks["hbm_gbs"],
                     "peak_gbs": peaks["hbm_gbs"], "config": f"B={bb} H={hh} H_kv={hk} "
                     f"S_max=32768 D=128 {str(cdt).removeprefix('torch.')} "
                     f"lengths={'32768' if lens_kind == 'full' else lens}"
                     + (f" paged: {page}-row pages in a shuffled pool" if page else ""),
                     "l2": "512 MB buffer written, then another 512 MB read, before every "
                           "call (outside the events)"}
        del qd, kc, vc, tables

    # B=1 MHA at 32K with the KV sequence split across the ranks. decode_b1_split: the peer
    # exchange (each rank's split kernel pushes its partials into every rank's buffer over
    # NVLink, then a bounded device wait and the fixed-order merge). decode_b1_split_allgather:
    # per-rank partials, NCCL all_gather, merge. On one rank both are the plain split decode.
    from flash_lab.distributed import (PeerExchange, ShardSpec, decode_sharded,
                                       default_splits_per_rank)

    smax, hh, hk = 32768, 32, 32
    shard = ShardSpec.even(smax, world, rank)
    gen = torch.Generator(device=device).manual_seed(17)  # same cache on every rank
    qd = torch.randn(1, hh, d, device=device, dtype=torch.bfloat16, generator=gen)
    full_k = torch.randn(1, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
    full_v = torch.randn(1, smax, hk, d, device=device, dtype=torch.bfloat16, generator=gen)
    k_shard = full_k[:, shard.offset:shard.offset + shard.length].contiguous()
    v_shard = full_v[:, shard.offset:shard.offset + shard.length].contiguous()
    del full_k, full_v
    seq_lens = torch.full((1,), smax, device=device, dtype=torch.int32)
    sm = torch.cuda.get_device_properties(device).multi_processor_count
    splits = default_splits_per_rank(1, hh, hk, shard.length, sm)
    nbytes = decode_bytes(hh, hk, d, [smax], 1)
    # On one rank there is nothing to exchange: both lines time the local partials + merge.
    exchange = PeerExchange(1, hh, d, splits_per_rank=splits) if world > 1 else None
    try:
        for name, ex, how in (("decode_b1_split", exchange, "partials pushed into every rank's "
                               "buffer over NVLink peer memory, bounded device wait, merge"
                               if world > 1 else "local partials and merge"),
                              ("decode_b1_split_allgather", None, "partials all-gathered over "
                               "NCCL, merge" if world > 1 else "local partials and merge")):
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
            ms = statistics.median(a.elapsed_time(b) for a, b in times)
            if dist is not None:
                t = torch.tensor([ms], device=device, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            gbs = nbytes / (ms * 1e-3) / 1e9
            out[name] = {
                "value": gbs, "unit": "GB/s", "ms_per_step": ms, "bytes_per_call": nbytes,
                "per_gpu_roofline_frac": gbs / world / peaks["hbm_gbs"], "scaling": "strong",
                "config": f"B=1 H=H_kv=32 D=128 32K keys split over {world} GPU(s), {splits} "
                          f"splits per GPU, {how} in a fixed order",
                "l2": "512 MB buffer written, then another 512 MB read, before every call "
                      "(outside the events)"}
        if exchange is not None and exchange.read_status() != 0:
            raise RuntimeError("a peer-exchange wait timed out during the bench")
    finally:
        if exchange is not None:
            exchange.close()
    return out


def run_e2e_llama(args) -> int:
    """The e2e configuration: Llama-3.1-8B architecture (32 layers, d_model 4096, 32 heads, 8 KV
    heads, head_dim 128, RoPE theta 500000, vocab 128256) with random-init bf16 weights, batch 1,
    a random 8192-token prompt, 256 greedy tokens, a static KV cache and the decode step compiled
    (torch.compile fullgraph, CUDA graphs), attention through the flash_lab HF backend; the same
    run with transformers' SDPA backend beside it. Prints one JSON line."""
    import torch
    from transformers import CompileConfig, LlamaConfig, LlamaForCausalLM, StaticCache

    import flash_lab.hf

    flash_lab.hf.register()
    device = torch.device("cuda", 0)
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rope_theta=500000.0, max_position_embeddings=131072)
    torch.manual_seed(0)
    with torch.device(device):
        model = LlamaForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
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
            generate(16)        # compiles the decode step
            generate(16)

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
                         "decode_step_ms": (total - ttft) / (args.new_tokens - 1)}
        tokens[attn] = out[0, ids.shape[1]:].tolist()
    agree = sum(1 for a, b in zip(tokens["flash_lab"], tokens["sdpa"]) if a == b)
    first_diff = next((i for i, (a, b) in enumerate(zip(tokens["flash_lab"], tokens["sdpa"]))
                       if a != b), None)
    line = {"metric": "e2e Llama-3.1-8B arch: decode step ms / TTFT ms (lower is better)",
            "higher_is_better": False, "dtype": "bf16", "data": "synthetic (random init, "
            "random prompt)", "config": {"model": "Llama-3.1-8B architecture",
            "prompt_len": args.prompt_len, "new_tokens": args.new_tokens, "batch": 1,
            "cache": "static", "decode": "torch.compile, CUDA graphs (transformers turns "
            "fullgraph off for attention backends named flash*)"},
            "flash_lab": results["flash_lab"], "sdpa": results["sdpa"],
            "greedy_tokens_equal": agree, "first_divergence": first_diff}
    emit(line)
    return 0


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
        if args.profile == "decode_gqa_ragged":   # the bench's lengths, U[16384, 32768]
            lens = torch.randint(16384, smax + 1, (b,), generator=torch.Generator().manual_seed(0))
            lens = lens.to(device=device, dtype=torch.int32)
        fn = lambda: flash_lab.decode(qd, kc, vc, lens)  # noqa: E731
        what = f"decode B={b} H=32 H_kv={hk} S=32768 D=128 lengths={lens.tolist()}"
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(f"profile case done: {what}, {args.warmup + args.steps} calls")
    return 0


if __name__ == "__main__":
    sys.exit(main())
