"""Exhaustive accuracy of the float transcendentals and of 16-bit pow.

Every float bit pattern (2^32 inputs) of sin / cos / exp / log, and every
f16 and bf16 (a, b) pair (2^32 pairs) of pow, is checked against the same op
evaluated in f64 through the engine: exact widening, CUDA's double-precision
function, one rounding back. That reference is the correctly rounded result
except within ~1e-16 of a rounding boundary. The f32 / 16-bit kernels must be
within 1 ulp of it, NaN exactly where it is NaN, with identical signed zeros.
libm's float functions (the CPU reference path) are within 1 ulp of the
correctly rounded value as well, which is where the 2-ulp parity bar against
the oracle comes from.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

CHUNK = 1 << 28


def _ordered(bits: torch.Tensor, sign_bit: int) -> torch.Tensor:
    """Sign-magnitude bit patterns (int64) onto a monotone integer line."""
    mag = bits & (sign_bit - 1)
    return torch.where((bits & sign_bit) != 0, -mag, mag)


def _check(got: torch.Tensor, ref: torch.Tensor, what: str) -> None:
    """got/ref: float tensors of one dtype; within 1 ulp, NaN where NaN,
    signed zeros identical."""
    gnan, rnan = torch.isnan(got), torch.isnan(ref)
    assert torch.equal(gnan, rnan), f"{what}: NaN pattern differs ({int((gnan != rnan).sum())} elements)"
    if got.dtype == torch.float32:
        gi, ri, sign = got.view(torch.int32).long() & 0xFFFFFFFF, ref.view(torch.int32).long() & 0xFFFFFFFF, 1 << 31
    else:
        gi, ri, sign = got.view(torch.int16).long() & 0xFFFF, ref.view(torch.int16).long() & 0xFFFF, 1 << 15
    d = (_ordered(gi, sign) - _ordered(ri, sign)).abs()
    d = torch.where(rnan, torch.zeros_like(d), d)
    worst = int(d.max())
    assert worst <= 1, f"{what}: {worst} ulp at input index {int(d.argmax())}"
    zero = (ref == 0) & ~rnan
    assert torch.equal(gi[zero], ri[zero]), f"{what}: signed zero differs"


@pytest.mark.parametrize("op", ["sin", "cos", "exp", "log"])
def test_f32_all_inputs(ms, op):
    f = getattr(ms, op)
    for c in range((1 << 32) // CHUNK):
        bits = torch.arange(c * CHUNK, (c + 1) * CHUNK, dtype=torch.int64, device="cuda")
        bits = torch.where(bits >= (1 << 31), bits - (1 << 32), bits).to(torch.int32)
        x = ms.from_torch(bits.view(torch.float32))
        got = f(x).torch()
        ref = ms.astype(f(ms.astype(x, "f64")), "f32").torch()
        _check(got, ref, f"{op} chunk {c}")
        del bits, x, got, ref
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_pow_all_16bit_pairs(ms, dt):
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    for c in range((1 << 32) // CHUNK):
        i = torch.arange(c * CHUNK, (c + 1) * CHUNK, dtype=torch.int64, device="cuda")
        hi, lo = i >> 16, i & 0xFFFF
        a_bits = torch.where(hi >= (1 << 15), hi - (1 << 16), hi).to(torch.int16)
        b_bits = torch.where(lo >= (1 << 15), lo - (1 << 16), lo).to(torch.int16)
        a, b = ms.from_torch(a_bits.view(tdt)), ms.from_torch(b_bits.view(tdt))
        got = ms.pow(a, b).torch()
        ref = ms.astype(ms.pow(ms.astype(a, "f64"), ms.astype(b, "f64")), dt).torch()
        _check(got, ref, f"{dt} pow chunk {c}")
        del i, hi, lo, a_bits, b_bits, a, b, got, ref
    torch.cuda.empty_cache()
