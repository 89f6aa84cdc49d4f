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
    full = bench.prefill_flops(4, 32, 4096, 4096, 128, False)
    assert line["ms_per_step"] == pytest.approx(full / 0.04e12 * 1e3)


def test_reference_arm_is_rank_zero_only(monkeypatch):
    out = io.StringIO()
    monkeypatch.setattr(bench, "_JSON_OUT", out)
    monkeypatch.setenv("RANK", "1")
    bench.run_reference_arm(argparse.Namespace(gpus=2, steps=3, warmup=3))
    assert out.getvalue() == ""
