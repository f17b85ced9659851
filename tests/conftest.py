import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


# Tolerances stated by the spec: output relative 1e-5 (f32), 2e-3 (f16), 1.6e-2 (bf16); LSE 1e-4.
import torch  # noqa: E402

OUT_TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}
LSE_TOL = 1e-4


def assert_out_close(got, ref, dtype, what=""):
    """|got - ref| <= tol * (|ref| + mean|ref|) elementwise (relative, with the mean
    magnitude as the floor for entries near zero)."""
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    tol = OUT_TOL[dtype]
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    floor = ref.abs().mean().item() if ref.numel() else 0.0
    err = (got - ref).abs()
    bound = tol * (ref.abs() + floor)
    bad = err > bound
    if bad.any():
        i = int(torch.argmax((err - bound).flatten()))
        raise AssertionError(f"{what}: {int(bad.sum())} of {ref.numel()} outside tol {tol}; worst at flat {i}: "
                             f"got {got.flatten()[i].item()} ref {ref.flatten()[i].item()}")


def assert_lse_close(got, ref, what=""):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(got)), f"{what}: -inf pattern differs"
    if fin.any():
        err = (got[fin] - ref[fin]).abs()
        bound = LSE_TOL * (1 + ref[fin].abs())
        assert (err <= bound).all(), f"{what}: LSE max err {err.max().item()}"


def gpu_available():
    return torch.cuda.is_available()
