"""bench.py's models and result lines, on CPU (the reference's tests/test_bench.py pins its FLOP
and byte models the same way): the work per call that every roofline fraction is computed
from, the measured-peak and traffic records, and the reference arm's JSON line."""

import argparse
import io
import json

import pytest

import bench


def test_prefill_flop_model():
    # 4 * B * H * S_q * S_k * D, halved when causal (the FA2 convention of bench/flops.py).
    assert bench.prefill_flops(4, 32, 4096, 4096, 128, False) == 4 * 4 * 32 * 4096 ** 2 * 128
    assert bench.prefill_flops(4, 32, 4096, 4096, 128, False) == pytest.approx(1.0995e12, rel=1e-4)
    assert bench.prefill_flops(4, 32, 4096, 4096, 128, True) == pytest.approx(5.498e11, rel=1e-4)
    assert bench.prefill_flops(1, 4, 300, 1000, 64, False) == 4 * 4 * 300 * 1000 * 64


def test_decode_byte_model():
    # K and V rows once per KV head plus q and o, 2-byte elements.
    mha = bench.decode_bytes(32, 32, 128, [32768] * 8, 8)
    assert mha == 4295098368.0                       # 4.295e9: the MHA 32K configuration
    ragged = [22713, 19238, 18982, 27719, 18962, 25728, 18646, 23007]
    gqa = bench.decode_bytes(32, 8, 128, ragged, 8)
    assert gqa == 2 * 8 * 128 * 2 * sum(ragged) + 2 * 8 * 32 * 128 * 2
    assert gqa == 716910592.0                        # the ragged GQA line's bytes_per_call


def test_peaks_and_traffic_records():
    peaks = bench.load_peaks()
    assert peaks["source"] in ("measured", "fallback")
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 100
    traffic = bench.load_traffic()
    for name in ("prefill_kernel_noncausal", "prefill_kernel_causal"):
        assert traffic[name]["bytes_per_launch"] > 0


def test_reference_arm_line(monkeypatch):
    # The line's shape, with the timed oracle call replaced by a fixed sample.
    sample = {"value": 0.04, "unit": "TFLOP/s", "cores": 8, "kind": "port",
              "sample": "fixed", "seconds": 1.0}
    monkeypatch.setattr(bench, "cpu_baseline_prefill", lambda rows: dict(sample))
    out = io.StringIO()
    monkeypatch.setattr(bench, "_JSON_OUT", out)
    monkeypatch.delenv("RANK", raising=False)
    bench.run_reference_arm(argparse.Namespace(gpus=1, steps=3, warmup=3))
    line = json.loads(out.getvalue())
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["value"] == 0.04 and line["unit"] == "TFLOP/s" and line["higher_is_better"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] == 8
    assert line["e2e"] == {"value": 0.04, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # ms_per_step is the measured sampled step; the full-call time is extrapolated beside it.
    assert line["ms_per_step"] == pytest.approx(1000.0)
    full = bench.prefill_flops(4, 32, 4096, 4096, 128, False)
    assert line["config"]["full_call_ms_extrapolated"] == pytest.approx(full / 0.04e12 * 1e3)


def test_reference_arm_is_rank_zero_only(monkeypatch):
    out = io.StringIO()
    monkeypatch.setattr(bench, "_JSON_OUT", out)
    monkeypatch.setenv("RANK", "1")
    bench.run_reference_arm(argparse.Namespace(gpus=2, steps=3, warmup=3))
    assert out.getvalue() == ""


def test_sample_rows_include_both_ends():
    rows = bench.sample_rows(4096, 256, seed=7)
    assert len(rows) == 256 and rows[0] == 0 and rows[-1] == 4095
    assert (rows[1:] > rows[:-1]).all()
    assert list(bench.sample_rows(3, 256, seed=1)) == [0, 1, 2]


def test_merge_checks():
    a = {"correct": True, "max_err_vs_ref64": 1e-3, "2x_rounding": 4e-3, "lse_err": 1e-6,
         "checked": "x"}
    b = dict(a, correct=False, max_err_vs_ref64=5e-3)
    m = bench.merge_checks([a, None, b])
    assert m["correct"] is False and m["max_err_vs_ref64"] == 5e-3
    assert bench.merge_checks([None])["correct"] is True


def test_cpu_checks_on_the_oracle():
    """check_prefill / check_decode accept the oracle's own fp64 result (rounded to bf16) and
    reject a perturbed one; CPU tensors stand in for device tensors."""
    import numpy as np
    import torch

    import oracle

    gen = torch.Generator().manual_seed(0)
    q = torch.randn(1, 40, 4, 64, generator=gen).bfloat16()
    k = torch.randn(1, 40, 2, 64, generator=gen).bfloat16()
    v = torch.randn(1, 40, 2, 64, generator=gen).bfloat16()
    o64, lse64 = oracle.attention(q.double().numpy(), k.double().numpy(), v.double().numpy(),
                                  causal=True, return_lse=True)
    o = torch.from_numpy(o64).bfloat16()
    lse = torch.from_numpy(lse64).float()
    rows = bench.sample_rows(40, 10, seed=1)
    assert bench.check_prefill(o, lse, q, k, v, True, 0.125, rows)["correct"]
    bad = o.clone()
    bad[0, rows[3], 1, 5] += 0.25
    assert not bench.check_prefill(bad, lse, q, k, v, True, 0.125, rows)["correct"]

    qd = torch.randn(3, 8, 64, generator=gen).bfloat16()
    kc = torch.randn(3, 50, 2, 64, generator=gen).bfloat16()
    vc = torch.randn(3, 50, 2, 64, generator=gen).bfloat16()
    lens = torch.tensor([50, 7, 31], dtype=torch.int32)
    od64, lsed64 = oracle.decode(qd.double().numpy(), kc.double().numpy(), vc.double().numpy(),
                                 lens.numpy(), return_lse=True)
    od = torch.from_numpy(od64).bfloat16()
    lsed = torch.from_numpy(lsed64).float()
    assert bench.check_decode(od, lsed, qd, kc, vc, lens, 0.125, [0, 2], [0, 1])["correct"]
    # Paged: the same cache as 10-row pages in a shuffled pool.
    perm = torch.randperm(15, generator=gen)
    pool_k = kc.reshape(15, 10, 2, 64)[torch.argsort(perm)]
    pool_v = vc.reshape(15, 10, 2, 64)[torch.argsort(perm)]
    tables = perm.view(3, 5).to(torch.int32)
    assert bench.check_decode(od, lsed, qd, pool_k, pool_v, lens, 0.125, [0, 1, 2], [1],
                              block_tables=tables)["correct"]
    bad = od.clone()
    bad[1, 2, 0] += 0.1
    assert not bench.check_decode(bad, lsed, qd, kc, vc, lens, 0.125, [1], [0, 1])["correct"]
