"""bench.py's reference arm runs on the host cores alone (the CPU port of the
path), so its JSON line can be checked here: the contract keys, and the same
`config` the B200 arm prints, the bounded sample described in cpu_baseline."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_line():
    sys.path.insert(0, str(ROOT))
    import bench

    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3", "--cpu-tokens", "64"],
                         check=True, capture_output=True, text=True, cwd=ROOT, timeout=600)
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["config"] == bench.config2(1, bench.PREFILL_B)
    assert line["value"] > 0 and line["warmup"] >= 3
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and "64 ACGT tokens" in cb["sample"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
