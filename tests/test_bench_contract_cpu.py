"""bench.py's reference arm (the reference's own search on the host cores) prints the JSON line the
driver parses: the contract's keys, impl "reference", the B200 arm's config, a cpu_baseline
describing the run, an e2e object with no host<->device traffic, and the labelled extra CPU
baselines. Runs on the CPU in under a minute (short searches)."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1", "--cpu-seconds", "2", "--sims", "128", "--wave", "64"],
                         capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["n_gpus"] == 1
    assert line["higher_is_better"] is True and "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert abs(cb["value"] - line["value"]) < 1e-6 * max(1.0, line["value"])
    e2e = line["e2e"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert e2e["unit"] == line["unit"] and e2e["value"] == line["value"]
    # same config keys as the B200 arm's line
    for k in ("roots_per_gpu", "global_batch", "sims", "wave", "capacity", "model", "parallelism"):
        assert k in line["config"], k
    if cb["kind"] == "reference":        # the staged reference ran: the port and Cython numbers beside it
        assert line["baselines"]["oracle_port"]["kind"] == "port"
        assert "reference_cython" in line["baselines"]
