"""bench.py's reference arm on the CPU: the JSON line the driver reads, and
the TP shard it times (one rank's heads at N GPUs, same bytes per step)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _run(gpus: int) -> dict:
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    env.pop("RANK", None)
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", str(gpus),
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600,
                       env=env, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("gpus,unit", [(1, 2048), (4, 512)])
def test_reference_arm_line_and_shard(gpus, unit):
    line = _run(gpus)
    assert line["impl"] == "reference" and line["n_gpus"] == gpus
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["shard"]["tp"] == gpus and line["shard"]["unit_bytes"] == unit
    assert line["shard"]["processes"] == 1 and line["cpu_baseline"]["cores"] == os.cpu_count()
    assert line["config"]["tp"] == gpus and line["config"]["kv_heads_per_rank"] == 8 // gpus


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, PYTHONPATH=str(ROOT), RANK="1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=300,
                       env=env, cwd=str(ROOT))
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_duplex_thread_rule():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.duplex_threads(256 << 20) == (1, 2)
    assert bench.duplex_threads(5 << 29) == (2, 3)


@pytest.mark.parametrize("kv,bs,unit", [(2, 16, 2048), (1, 64, 1152)], ids=["kv", "k_only"])
def test_cpu_geometry_sample_moves_the_configuration_payload(kv, bs, unit):
    """the per-configuration CPU baseline: one pass over a small sample of the
    geometry (K+V as the 70B config, K only as the MLA config)"""
    sys.path.insert(0, str(ROOT))
    import bench
    res = bench.cpu_geometry_sample("test", 3, unit, bs, kv, 2, 2, 0.0)
    assert res["value"] > 0 and res["unit"] == "GB/s" and res["kind"] == "port" and res["cores"] == 2
    rec_mib = kv * 3 * bench.CHUNK * unit / 2**20
    assert f"2 records of {rec_mib:.2f} MiB (3 layers, {'K+V' if kv == 2 else 'K only'}" in res["sample"]


def test_host_copy_probe_reports_a_rate():
    """the host memory copy rate the bench takes around its e2e steps"""
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.host_copy_gbs(2, 0.05) > 0
