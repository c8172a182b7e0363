"""bench.py's result line stays the last line of stdout under torchrun: after
quiet_stdout() (every rank calls it before the last barrier) anything the
process still writes, from Python or from C (NCCL's teardown lines), goes to
stderr, and emit() writes the JSON through the saved stdout."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import ctypes, sys
sys.argv = ["bench.py"]
sys.path.insert(0, ROOT)
import bench
libc = ctypes.CDLL(None)
print("python before", flush=True)
libc.printf(b"c before\n")
bench.quiet_stdout()
print("python after", flush=True)
bench.emit({"metric": "m", "value": 1.5})
libc.printf(b"c after\n")
libc.fflush(None)
print("python late", flush=True)
"""


def test_result_line_is_last_on_stdout():
    r = subprocess.run([sys.executable, "-c", "ROOT = %r\n" % ROOT + CHILD], capture_output=True, text=True,
                       timeout=120, cwd=ROOT)
    assert r.returncode == 0, r.stderr
    out = r.stdout.strip().splitlines()
    assert out[:2] == ["python before", "c before"]
    assert json.loads(out[-1]) == {"metric": "m", "value": 1.5}
    assert len(out) == 3
    for line in ("python after", "c after", "python late"):
        assert line in r.stderr
