"""bench.py's reference arm (`--impl reference`), on the CPU: the JSON line
the driver reads, and that the arm runs the CPU restatement only.  If it
loaded the product library, the reference-vs-product ratio would be void.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Runs bench.py's main in this interpreter, then prints the shared objects
# the process has mapped, after the bench's own JSON line.
_RUNNER = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--series", "4"]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as e:
    if e.code not in (0, None):
        raise
maps = sorted({l.split()[-1] for l in open("/proc/self/maps") if l.rstrip().endswith(".so")})
print("MAPPED " + " ".join(maps))
"""


def test_reference_arm_line_and_no_product_library():
    r = subprocess.run([sys.executable, "-c", _RUNNER], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-3000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "series/s" and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["one_thread"]["cores"] == 1 and cb["one_thread"]["value"] > 0
    mapped = next(l for l in r.stdout.splitlines() if l.startswith("MAPPED ")).split()[1:]
    assert not any(os.path.basename(p).startswith("libt0b") for p in mapped), mapped
    assert any(os.path.basename(p) == "libt0oracle.so" for p in mapped), mapped
