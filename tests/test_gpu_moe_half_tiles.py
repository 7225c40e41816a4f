"""The fused-MoE GPU parity suite (tests/test_gpu_moe.py, tests/test_gpu_moe_options.py)
re-run with AITER_B200_MOE_HALF_TILES=0.  By default expert blocks whose rows 64..
are all padding run as M=64 tcgen05 tiles whose epilogue reads half the TMEM bytes
(the suites' shapes hit such blocks everywhere, and about half the experts' last
blocks at config-1 size); with the variable at 0 every block runs as a full 128-row
tile, the path this test keeps covered.  The variable is read once per process, so
the suite runs in a child process.  (The A8W4 kernels always run full tiles.)"""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def test_moe_parity_suite_with_full_tiles_only():
    env = dict(os.environ, AITER_B200_MOE_HALF_TILES="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(ROOT, "tests", "test_gpu_moe.py"),
                        os.path.join(ROOT, "tests", "test_gpu_moe_options.py")],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
