"""Host logic of the per-context set-up cache (``lf::PerContextOnce``), compiled with nvcc and
run on the CPU against a stub context id: once per context, again after a failure, again after
eviction.  Needs no GPU."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not on PATH")
def test_per_context_once_runs_setup_once_per_context(tmp_path):
    exe = tmp_path / "per_context_once"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "-o", str(exe),
                    os.path.join(HERE, "cpp", "per_context_once.cu")],
                   check=True, capture_output=True, timeout=300)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "ok"
