"""The TMEM read-throughput diagnostic (`tmem_ld_probe`, run by `bench.py --mode tmem_ld`)
launches every variant on every SM and returns positive clock spans with no device error.
Runs only with AITER_B200_TEST_UNRUN=1 until it has been run on a B200."""
import os

import pytest
import torch

from aiter_b200 import _lib
from gpu_util import check_no_device_error, requires_cuda

pytestmark = [pytest.mark.gpu, requires_cuda,
              pytest.mark.skipif(os.environ.get("AITER_B200_TEST_UNRUN") != "1",
                                 reason="the TMEM probe has not been run on a B200 yet")]


def test_every_variant_runs_on_every_sm():
    dev = torch.device("cuda", 0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    for v in range(_lib.lib().tmem_ld_probe_variants()):
        cycles = torch.zeros(sms, dtype=torch.int64, device=dev)
        sink = torch.zeros(sms * 16 * 32, device=dev)
        _lib.call("tmem_ld_probe", v, 4, cycles, sink)
        torch.cuda.synchronize()
        assert (cycles > 0).all(), v
        check_no_device_error()
