"""Shared comparison helpers for the parity tests."""

import pytest
import torch

BF16 = torch.bfloat16


def ulp_diff(a: torch.Tensor, b: torch.Tensor, floor: float = 0.0) -> torch.Tensor:
    """Distance in BF16 ulps (at the larger magnitude, but at least ``floor``) between two tensors."""
    a32, b32 = a.float().cpu(), b.float().cpu()
    mag = torch.maximum(a32.abs(), b32.abs()).clamp_min(max(floor, 1e-30))
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    return (a32 - b32).abs() / ulp


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a32, b32 = a.float().cpu(), b.float().cpu()
    return float((a32 - b32).norm() / b32.norm().clamp_min(1e-30))


def assert_bf16_close(actual, expected, *, max_ulp=1.0, max_frac=0.02, rel=1e-2, floor_rel=2.0 ** -6):
    """Tolerance for BF16 outputs of the same rounding sequence: at most `max_ulp` BF16 ulps
    apart (FP32 summation order / transcendental differences), on at most `max_frac` of the
    elements, and a relative Frobenius error within `rel` (the 1e-2 bound for BF16 paths).
    Ulps are measured at a magnitude of at least `floor_rel` x rms(expected): outputs that are
    the result of near-total cancellation carry FP32 summation-order noise that is large in
    their own ulps but negligible at the scale of the tensor."""
    assert tuple(actual.shape) == tuple(expected.shape), (actual.shape, expected.shape)
    floor = floor_rel * float(expected.float().pow(2).mean().sqrt())
    d = ulp_diff(actual, expected, floor)
    assert float(d.max()) <= max_ulp, f"max ulp diff {float(d.max())}"
    assert float((d > 0).float().mean()) <= max_frac, f"mismatch fraction {float((d > 0).float().mean())}"
    assert rel_err(actual, expected) <= rel


def assert_swiglu_close(actual, expected, rel=5e-3, abs_rms=2.0 ** -6):
    """SwiGLU outputs of GEMMs: bf16(silu(g)) * u with g, u BF16-rounded projections. In the
    negative tail silu(g) ~ g e^g, so a one-ulp difference in g moves the output by ~|g| ulps;
    compare by relative Frobenius error and by absolute error against the tensor's rms."""
    assert tuple(actual.shape) == tuple(expected.shape)
    a, b = actual.float(), expected.float()
    assert rel_err(a, b) <= rel, rel_err(a, b)
    rms = float(b.pow(2).mean().sqrt())
    # per element: two BF16 ulps of the value, with a floor at abs_rms of the tensor's rms
    excess = (a - b).abs() - (2.0 ** -6 * b.abs() + abs_rms * rms)
    worst = int(excess.argmax())
    assert float(excess.max()) <= 0, (worst, float(a.flatten()[worst]), float(b.flatten()[worst]), rms)


def assert_residual_close(actual, residual, update, max_frac=0.02):
    """In-place residual epilogue bf16(r + bf16(y)): y comes from a GEMM whose FP32 summation order
    differs from the oracle's, so bf16(y) may differ by one ulp of |y|; after the add (which can
    cancel) the result may differ by that plus one rounding of the sum."""
    want = (residual.float() + update.float()).to(BF16)
    a, w, y = actual.float().cpu(), want.float(), update.float()
    def ulp(t):
        return torch.exp2(torch.floor(torch.log2(t.abs().clamp_min(1e-30))) - 7)
    excess = (a - w).abs() - (ulp(y) + ulp(w))
    assert float(excess.max()) <= 0, float(excess.max())
    assert float((a != w).float().mean()) <= max_frac
    assert rel_err(a, w) <= 1e-2


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def randn(*shape, seed=0, scale=1.0, dtype=BF16):
    return (torch.randn(*shape, generator=gen(seed)) * scale).to(dtype)


requires_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
