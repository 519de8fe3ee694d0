"""The reference arm of bench.py (the CPU restatement timed on the host, the
driver's `--impl reference` line) runs without a GPU: its JSON line carries
the keys the benchmark contract names."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("workload,unit", [("quant-mxfp8", "GB/s"), ("mcts8b", "queries/s")])
def test_reference_arm_line(workload, unit):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                          "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == unit and line["value"] > 0
    assert line["warmup"] >= 3 and line["higher_is_better"] is True
    assert line["config"]["workload"] == workload
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == unit
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_maps_no_product_library():
    """The reference arm times only the CPU restatement: the process must not
    load libdendrite_b200.so (not even by importing the package)."""
    code = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'quant-mxfp8', '--steps', '1', "
        "'--warmup', '0']\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('PRODUCT_SO_LOADED' if 'libdendrite_b200' in maps else 'PRODUCT_SO_ABSENT')\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "PRODUCT_SO_ABSENT" in out.stdout
    code2 = code.replace("'quant-mxfp8'", "'mcts8b'")
    out = subprocess.run([sys.executable, "-c", code2], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    assert "PRODUCT_SO_ABSENT" in out.stdout
