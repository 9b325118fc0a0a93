"""The command-line harness with the reference's surface (ada-mla_b200/mla.py,
mirroring lechebs/ada-mla mla.py:153-194): --test in fp16 and --fp32, --for-ncu
and --bench, each run as the reference's user would run it."""
import os
import re
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "ada-mla_b200", "mla.py")


def _run(*args, timeout=600):
    r = subprocess.run([sys.executable, CLI, *args], capture_output=True, text=True, timeout=timeout,
                       cwd=ROOT)
    assert r.returncode == 0, (args, r.stdout[-2000:], r.stderr[-2000:])
    return r.stdout


def _fused_errors(out):
    rows = re.findall(r"\[fused\] seq_len=(\d+) max=([0-9.eE+-]+) mean=([0-9.eE+-]+)", out)
    assert rows, out
    return [(int(n), float(mx), float(mean)) for n, mx, mean in rows]


def test_cli_test_fp16_split():
    out = _run("--test", "-s", "4096", "1000", "-k", "fused", "torch")
    for n, mx, mean in _fused_errors(out):
        assert mx <= 1e-2 and mean <= 1e-3, (n, mx, mean)


def test_cli_test_fp32_fused():
    out = _run("--fp32", "--test", "-s", "4096", "-k", "fused", "torch")
    for n, mx, mean in _fused_errors(out):
        assert mx <= 1e-4, (n, mx, mean)


def test_cli_for_ncu_and_bench():
    _run("--for-ncu", "-s", "2048", "-k", "fused")
    out = _run("--bench", "-s", "4096", "-k", "fused", "torch")
    line = [l for l in out.splitlines() if l.strip().startswith("4096")]
    assert line, out
    ms = [float(x) for x in line[0].split()[1:]]
    assert len(ms) == 2 and all(m > 0 for m in ms)
