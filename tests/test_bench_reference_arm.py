"""bench.py's reference arm on the CPU: one JSON line with the contract's keys.

``bench.py --impl reference`` times the reference's own CPU code for the paging
path -- its ``ExpertTable.acquire`` from the unmodified install under
baseline/_ref on both tables, plus a threaded memcpy of the missed rows -- or,
without the install, the numpy restatement under oracle/.  It needs no GPU, so
its output line is checked here: the metric, unit and config of the GPU arm, a
cpu_baseline block describing the sample, and an e2e block with no
host<->device bytes.
"""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "3", "--window", "64"],
        cwd=ROOT, capture_output=True, text=True, timeout=600,
        env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"].startswith("paged expert GB/s") and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 1, 3)
    assert d["ms_per_step"] > 0 and d["scaling"] == "weak" and d["vs_baseline"] is None
    assert d["config"]["workload"].startswith("config2")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1
    assert cb["unit"] == "GB/s" and cb["sample"]
    ref_installed = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "vllm_expert_pager"))
    assert cb["kind"] == ("reference" if ref_installed else "port")
    if ref_installed:  # the reference's encoder and the numpy port are reported beside it
        assert d["codec_config1"]["kind"] == "reference" and d["codec_config1"]["encode_mb_s"] > 0
        assert d["port"]["value"] > 0
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == "GB/s"
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
