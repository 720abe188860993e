"""bench.py's result line (driver contract) built from synthetic measurements — CPU."""

import argparse
import json

import bench


def _args(**kw):
    a = argparse.Namespace(steps=10, warmup=3, config="llama8b", no_cpu_baseline=True)
    a.__dict__.update(kw)
    return a


ROOF = {"bound": "hbm", "achieved": 1.0, "peak": 2.0, "unit": "GB/s", "frac": 0.5, "traffic": None}
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "clocks", "e2e",
        "gpu_launches"}


def test_single_gpu_line():
    res = {"n_params": 8_030_261_248, "ms_per_step": 100.0, "pass1_ms": 17.0, "pass2_ms": 83.0,
           "bytes_per_param": 20, "roofline": ROOF, "clocks": None,
           "e2e": {"value": 1.0, "unit": "Gparams/s", "h2d_bytes_per_step": 1,
                   "d2h_bytes_per_step": 1}, "gpu_launches": 20}
    line = bench.result_line(_args(), res, 1, "weak", "bf16", {"workload": "w"})
    assert KEYS <= set(line)
    assert abs(line["value"] - 80.30261248) < 1e-3
    assert abs(line["hbm_gbs_per_gpu"] - 8_030_261_248 * 20 / 0.1 / 1e9) < 0.1
    json.dumps(line)


def test_multi_gpu_line():
    res = {"n_params": 8_030_261_248, "ms_per_step": 40.0, "pass1_ms": None, "pass2_ms": None,
           "local_step_ms": 30.0, "allgather_ms": 15.0, "allgather_gbs_per_rank": 500.0,
           "overlap_saving_ms": 5.0, "step_only_gparams": 267.0, "shard_params": 10,
           "buckets": 8, "max_ctas": 132, "bytes_per_param": 20, "roofline": ROOF,
           "clocks": None, "e2e": None, "gpu_launches": 160}
    line = bench.result_line(_args(), res, 4, "strong", "bf16", {"workload": "w"})
    assert KEYS <= set(line) and line["n_gpus"] == 4 and line["pass1_ms"] is None
    assert line["buckets"] == 8 and line["allgather_ms"] == 15.0
    json.dumps(line)


def test_workload_param_counts():
    import math
    assert sum(math.prod(s) if s else 1 for s in bench.llama3_8b_shapes()) == 8_030_261_248
    assert len(bench.llama3_8b_shapes()) == 291
    assert sum(math.prod(s) for s in bench.gpt2_small_shapes()) == 124_439_808
    assert len(bench.gpt2_small_shapes()) == 148
    assert bench.bytes_per_param(bench.torch.bfloat16, bench.torch.bfloat16) == (6, 14)
    assert bench.bytes_per_param(bench.torch.float32, bench.torch.float32) == (8, 20)
