"""Helpers shared by the GPU parity tests (no GPU work at import time)."""
import numpy as np
import torch

ATOL, RTOL, MAX_RMS = 2e-2, 1e-2, 5e-3     # bf16 gate: max-abs/rel and RMS (scripts/probe_varlen.py:24-25)
F32_TOL = 1e-5                              # float32 gate


def dev():
    return torch.device('cuda', 0)


def to_dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=dev(), dtype=dtype)


def i32(x):
    return torch.tensor(list(map(int, x)), dtype=torch.int32, device=dev())


def assert_bf16_close(actual, expected):
    a = actual.float().cpu().numpy().astype(np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape
    assert np.isfinite(a).all()
    np.testing.assert_allclose(a, e, atol=ATOL, rtol=RTOL)
    rms = float(np.sqrt(np.mean((a - e) ** 2)))
    assert rms <= MAX_RMS, f'rms {rms}'
    return rms


def status_clean(pkg):
    assert pkg.read_device_status(clear=True) == 0
