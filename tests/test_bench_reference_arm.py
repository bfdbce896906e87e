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
