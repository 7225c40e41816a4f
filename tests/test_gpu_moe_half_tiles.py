"""The fused-MoE GPU parity suite (tests/test_gpu_moe.py, tests/test_gpu_a8w4.py)
re-run with AITER_B200_MOE_HALF_TILES=1: expert blocks whose rows 64.. are all
padding then run as M=64 tcgen05 tiles whose epilogue reads half the TMEM bytes.
Its shapes hit such blocks everywhere (few tokens per expert) and at config-1 size
(about half the experts' last blocks at M=4096).  The variable is read once per
process, so the suite runs in a child process."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def test_moe_parity_suite_with_half_tiles():
    env = dict(os.environ, AITER_B200_MOE_HALF_TILES="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(ROOT, "tests", "test_gpu_moe.py"), os.path.join(ROOT, "tests", "test_gpu_a8w4.py")],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
