"""bench.py's reference arm on the CPU: the JSON line it assembles carries the contract's keys
(the oracle's timing is replaced by a constant so that the test takes milliseconds)."""
import argparse

import bench


def test_reference_arm_line(monkeypatch):
    monkeypatch.setattr(bench, "cpu_decode_sample", lambda *a, **k: (123.0, "stub sample"))
    args = argparse.Namespace(steps=2, warmup=1, gpus=1, seqs=256)
    res = bench.run_reference(args, bench.Dist())
    # the same config dict as the GPU arm's line (rank 0's sequence lengths)
    assert res["config"] == bench.decode_config(1, 256, bench.seq_lens(1000, 256), 32, 32, 128, 0)
    assert res["impl"] == "reference"
    for key in ("metric", "value", "unit", "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert key in res, key
    assert res["metric"] == bench.METRIC
    assert res["value"] == 123.0
    assert res["e2e"]["value"] == res["value"]
    assert res["e2e"]["h2d_bytes_per_step"] == 0 and res["e2e"]["d2h_bytes_per_step"] == 0
    assert res["cpu_baseline"]["kind"] in ("port", "reference")


def test_peaks_fallback_or_measured():
    pk = bench.peaks()
    assert pk["src"] in ("measured", "fallback")
    assert pk["hbm_gbs"] > 1000 and pk["bf16_tflops"] > 100
