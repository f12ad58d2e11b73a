"""``bench.py --impl reference`` (the CPU arm) keeps the bench line contract,
and under a multi-rank launch only rank 0 runs and prints it; the engine arm's
launch count of a ``load`` follows the engine's paths."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CMD = [sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1", "--cpu-seconds", "1"]


def run(env_extra: dict) -> subprocess.CompletedProcess:
    env = {**os.environ, **env_extra}
    return subprocess.run(CMD, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    out = run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["steps"] == 2 and line["warmup"] == 1 and line["value"] > 0
    installed = (ROOT / "baseline" / "_ref" / "sheetsage2_refined" / "engine.py").exists()
    assert line["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["one_thread"]["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # a step is one bounded sample of about cpu-seconds / steps of decode
    assert 100.0 < line["ms_per_step"] < 60_000.0
    assert line["config"]["workload"].startswith("single-song decode")


def test_reference_arm_other_ranks_exit_without_work():
    out = run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [l for l in out.stdout.splitlines() if l.startswith("{")]


def test_load_launch_count_matches_the_engine_paths():
    """``gpu_launches`` counts a load's kernels from the engine's paths: one cross K/V launch for
    up to 32 layers, then prefill chunks of 128 positions, chunks of more than 8 rows on the
    tensor-core layer (11 launches a layer, LayerNorm + QKV in the last).  For a 2,048-token prefix
    at the single-song shape that is the 1,969 launches the ncu launch list of such a load holds."""

    sys.path.insert(0, str(ROOT))
    import bench

    class Eng:
        def __init__(self, per_step):
            self.step_launches = per_step

    L = 12
    one_slot = Eng(4 * L + 1)   # fused FFN decode: 4 launches a layer + logits
    batched = Eng(11 * L + 2)   # tensor-core decode: 11 a layer + LayerNorm and logits GEMM
    assert bench.load_launches(one_slot, L, 2048) == 1 + 16 * (11 * (L - 1) + 2) == 1969
    assert bench.load_launches(batched, L, 2048) == 1969
    # [SOS, OUT]: one row at position 0, on the decode kernels (prefill FFN as fc1 + fc2)
    assert bench.load_launches(one_slot, L, 2) == 1 + 5 * (L - 1) + 1
    assert bench.load_launches(batched, L, 2) == 1 + 11 * (L - 1) + 2
    # 9 rows: the decode kernels; 10 rows: the tensor-core layer
    assert bench.load_launches(one_slot, L, 9) == 1 + 5 * (L - 1) + 1
    assert bench.load_launches(one_slot, L, 10) == 1 + 11 * (L - 1) + 2
    assert bench.load_launches(one_slot, L, 1) == 1
