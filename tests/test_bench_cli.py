"""bench.py's output contract on the CPU: stdout carries JSON lines only.

The driver reads bench.py's stdout as one JSON line per run.  Libraries the
bench loads may print to the process's stdout from C (NCCL's version banner
under torchrun, the reference kernel's banner); bench.py sends file
descriptor 1 to stderr for the whole run and writes its JSON lines to the
original stdout, which these tests check without a GPU."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args, timeout=120):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


def test_vae_reference_arm_prints_one_json_line():
    r = _run("--vae", "--impl", "reference")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and "unavailable" in d


def test_emit_json_bypasses_redirected_stdout():
    """Output written to fd 1 after the redirection (as a C library would)
    lands on stderr; emit_json still reaches the original stdout."""
    code = (
        "import os, sys; sys.path.insert(0, %r); import bench; "
        "bench._JSON_FD = os.dup(1); os.dup2(2, 1); "
        "os.write(1, b'banner from C\\n'); print('stray print'); "
        "bench.emit_json({'metric': 'x', 'value': 1})" % str(ROOT))
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == json.dumps({"metric": "x", "value": 1})
    assert "banner from C" in r.stderr and "stray print" in r.stderr
