"""The division the kernels use when many values share one divisor (common.cuh div_rn_by): q = x * inv with inv the
correctly rounded reciprocal of d, then one correction q + (x - q d) * inv by fused multiply-adds (Markstein's
division step).  Emulated here in float64, where every float32 product is exact and the residual x - q d is exact
in float32, and compared with the correctly rounded float32 quotient over the operand ranges the kernels meet:
address halves over their norms (pk_address), exponentials over their sum (soft weights), memory reads over
den + eps (RunTimeSdm.finish)."""
import numpy as np


def markstein(x, d):
    x64, d64 = x.astype(np.float64), d.astype(np.float64)
    inv = (1.0 / d64).astype(np.float32).astype(np.float64)  # __frcp_rn(d)
    q = (x64 * inv).astype(np.float32).astype(np.float64)  # x * inv, rounded
    r = (x64 - q * d64).astype(np.float32).astype(np.float64)  # fmaf(-q, d, x): exact here, so one rounding
    return (r * inv + q).astype(np.float32)  # fmaf(r, inv, q)


def correctly_rounded(x, d):
    return (x.astype(np.float64) / d.astype(np.float64)).astype(np.float32)


def test_shared_divisor_division_is_correctly_rounded():
    rng = np.random.default_rng(0)
    n = 2_000_000
    cases = [
        # normalised address halves: components over a norm of the same vector
        (lambda: (rng.standard_normal(n) * 10.0 ** rng.uniform(-2, 2, n)).astype(np.float32),
         lambda: np.sqrt(rng.uniform(1e-3, 1e4, n)).astype(np.float32)),
        # soft weights: exp(score - max) in (0, 1] over a sum in [1, 32]
        (lambda: np.exp(-rng.uniform(0, 30, n)).astype(np.float32),
         lambda: rng.uniform(1.0, 32.0, n).astype(np.float32)),
        # the mean read: num over den + 1e-3
        (lambda: (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 3, n)).astype(np.float32),
         lambda: (rng.uniform(0, 100, n) + 1e-3).astype(np.float32)),
    ]
    for mx, md in cases:
        x, d = mx(), md()
        got, want = markstein(x, d), correctly_rounded(x, d)
        assert np.array_equal(got, want), int((got != want).sum())
