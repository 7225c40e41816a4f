"""Helpers shared by the GPU parity tests."""
import numpy as np
import pytest
import torch

requires_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def dev():
    return torch.device("cuda", 0)


def to_dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev())


def fp8_from_codes(codes):
    return torch.from_numpy(np.ascontiguousarray(codes, dtype=np.uint8)).view(torch.float8_e4m3fn).to(dev())


def codes(t):
    return t.view(torch.uint8).cpu().numpy()


def check_no_device_error():
    import aiter_b200
    assert aiter_b200.device_error(clear=True) == 0
