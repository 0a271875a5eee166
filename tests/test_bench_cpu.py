"""bench.py's host-side arithmetic, checked on the CPU: the algorithmic bytes of every workload
(the roofline numerator) against the per-config figures derived from the reference's shapes
(K, V, scales, q, out counted once; split-K scratch excluded), and the plan / kernel labels."""
from __future__ import annotations

import importlib.util

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("name,expected", [
    ("fp16", 536_870_912 + 131_072),                       # cfg1: K,V [256,4096,128] f16 + q,o
    ("int8", 8_589_934_592 + 134_217_728 + 4_194_304),     # cfg2: codes + scales + q,o (R=8192)
    ("int4", 4_294_967_296 + 134_217_728 + 4_194_304),     # cfg3 at D=128
    ("gqa", 2 * 64 * 8 * 16384 * 128 * 2 + 2 * 64 * 32 * 128 * 2),
    ("gqa_int8", 2 * 64 * 8 * 16384 * 130 + 2 * 64 * 32 * 128 * 2),
    ("sk", 32 * 16384 * 128 + 128 * 128),                  # cfg4 batch 1: 32*N*D + 128*D (67.1 MB)
    ("qpt", 8192 * 4096 * (2 * 128 + 128 + 2)),            # quantizer: 2D read, D + 2 written per token
    ("quant_int4", 8192 * 4096 * (2 * 128 + 64 + 2)),
])
def test_algorithmic_bytes(bench, name, expected):
    assert bench.algorithmic_bytes(bench.WORKLOADS[name]) == expected


def test_b2048_sweeps_scale_with_rows(bench):
    assert bench.algorithmic_bytes(bench.WORKLOADS["int8_b2048"]) == 69_826_772_992
    assert bench.algorithmic_bytes(bench.WORKLOADS["int4_b2048"]) == 35_467_034_624


def test_every_sweep_entry_names_a_workload(bench):
    for name, key, over in bench.CONFIG_SWEEP:
        w = dict(bench.WORKLOADS[key])
        w.update(over)
        assert bench.algorithmic_bytes(w) > 0, name


def test_plan_and_kernel_labels(bench):
    w = bench.WORKLOADS["sk"]
    assert bench.dominant_kernel(w, [22, 0, 176, 768, 0]).endswith("combine_kernel (PDL-chained)")
    assert bench.dominant_kernel(w, [16, 16, 128, 1024, 0]) == "decode_f16_kernel<128,1>"
    assert bench.dominant_kernel(bench.WORKLOADS["int4"], [1, 0, 444, 4096, 4]) == "decode_qtc_kernel<128,true,true>"
    rec = bench.plan_record([16, 16, 128, 1024, 0])
    assert rec["split_merge"].startswith("thread-block cluster") and rec["ctas"] == 128
    assert bench.plan_record([1, 0, 296, 16384, 0])["split_merge"] == "none"
    assert bench.plan_record(None) is None


def test_committed_traffic_reports_its_source(bench):
    traffic, source = bench.committed_traffic("gqa")
    assert traffic is None or traffic > 0
    assert isinstance(source, str) and source


def test_committed_traffic_covers_the_algorithmic_bytes(bench):
    """Every committed DRAM-traffic figure is within 1 % of, or above, its workload's algorithmic bytes
    (every byte is read or written at least once; well above would mean re-reads), and names its source."""
    for name in ("gqa", "int8", "int8_b2048", "int4", "int4_b2048", "gqa_int8", "qpt", "quant_int4"):
        traffic, source = bench.committed_traffic(name)
        assert traffic is not None and source, name
        alg = bench.algorithmic_bytes(bench.WORKLOADS[name])
        assert 0.99 * alg <= traffic <= 1.05 * alg, (name, traffic, alg)
