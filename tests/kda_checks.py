"""Tolerance checks shared by the GPU parity tests.

The bars are BASELINE.json's ``north_star``:

* outputs: max |o - o_ref| / rms(o_ref) <= 5e-3, taken on the kernel's fp32
  pre-cast output (the C ABI's ``out_fp32`` verification mode). On a bf16
  output the same bar is applied after allowing half a bf16 ulp of o_ref per
  element for the final round-to-nearest, which alone can exceed 5e-3 * rms
  at the heavy-tailed maxima (max/rms ~ 10);
* fp32 states: ||S - S_ref||_2 / ||S_ref||_2 <= 1e-3;
* slot addressing: untouched pool slots bit-identical.
"""

import torch

OUT_TOL = 5e-3
STATE_TOL = 1e-3


def out_error(out: torch.Tensor, ref: torch.Tensor) -> float:
    """Normalised max-abs error. A bf16 output against an fp32 reference is
    credited half a bf16 ulp (its own round-to-nearest); against a reference
    that is itself bf16 (both sides rounded), one ulp."""
    ref_bf16 = ref.dtype == torch.bfloat16
    ref = ref.detach().float().cpu()
    got = out.detach().cpu()
    rms = ref.pow(2).mean().sqrt().clamp_min(1e-30)
    diff = (got.float() - ref).abs()
    if got.dtype == torch.bfloat16:
        _, e = torch.frexp(ref)
        # ulp of a bf16 in [2^(e-1), 2^e) is 2^(e-8); half of it 2^(e-9).
        credit = torch.ldexp(torch.ones_like(ref), e - (8 if ref_bf16 else 9))
        diff = (diff - credit).clamp_min(0.0)
    return float(diff.max() / rms)


def assert_out_close(out, ref, tol: float = OUT_TOL, what: str = "output"):
    err = out_error(out, ref)
    assert err <= tol, f"{what}: normalised max-abs error {err:.3e} > {tol:.1e}"


def state_error(got: torch.Tensor, ref: torch.Tensor) -> float:
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    return float((got - ref).norm() / ref.norm().clamp_min(1e-30))


def assert_state_close(got, ref, tol: float = STATE_TOL, what: str = "state"):
    err = state_error(got, ref)
    assert err <= tol, f"{what}: relative RMS error {err:.3e} > {tol:.1e}"


def assert_untouched(after: torch.Tensor, before: torch.Tensor, touched):
    touched = {int(s) for s in touched}
    other = [s for s in range(before.shape[0]) if s not in touched]
    a = after.detach().cpu()
    b = before.detach().cpu()
    assert torch.equal(a[other], b[other]), "a pool slot outside the touched set changed"


def clone_pool(pool: torch.Tensor) -> torch.Tensor:
    """Copy a K-contiguous pool keeping its [V,K] backing."""
    return pool.transpose(-1, -2).clone().transpose(-1, -2)
