"""bench.py's host side (CPU): the reference arm prints the same metric and
workload config as the engine's arm for the same arguments, and the per-GPU
byte counts of the batch-64 roofline split as the expert-parallel layout
does."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, str(ROOT))
    import bench as b

    return b


def _reference_line(*extra, env=None):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--layers", "1", "--steps",
                          "1", "--warmup", "1", *extra], cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_reference_arm_bs1_config_matches(bench):
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    line = _reference_line()
    assert line["impl"] == "reference" and line["metric"] == "decode tok/s (bs1, configs[2])"
    assert line["config"] == bench.bs1_config(synthetic_config(num_layers=1), 1)
    assert line["cpu_baseline"]["kind"] == "port" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--layers", "1", "--steps",
                          "1", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0 and out.stdout.strip() == ""


def test_bs64_bytes_split_over_ranks(bench):
    from maple_flash_dgx_spark_b200.synth import synthetic_config

    cfg = synthetic_config()
    one, two, eight = (bench.bs64_step_bytes(cfg, w, 8192) for w in (1, 2, 8))
    kv = 64 * cfg["num_hidden_layers"] * cfg["num_key_value_heads"] * cfg["head_dim"] * 4 * 8192
    assert one > kv and two < one and eight < two
    # the K/V part splits exactly by rows; weights keep a replicated share
    assert (one - kv) > 2 * (two - kv // 2) - (one - kv)
    c = bench.bs64_config(cfg, 2, 8192, 3, 10)
    assert c["global_batch"] == 64 and c["parallelism"] == "ep2+dp-attention2"
