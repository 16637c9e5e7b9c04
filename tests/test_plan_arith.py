"""Arithmetic identities the plan kernel relies on (csrc/plan.cu), checked in float32 on the CPU."""
import numpy as np


def test_magic_number_rint_is_rint_half_even():
    # the bisection forms rint(x) as (x + 1.5 * 2^23) - 1.5 * 2^23; its x = (log2 g - mid) / 2 stays
    # well inside |x| < 2^22
    C = np.float32(12582912.0)
    rng = np.random.default_rng(0)
    x = np.concatenate([
        (rng.standard_normal(2_000_000) * 60).astype(np.float32),
        np.arange(-256, 256, 0.25, dtype=np.float32),             # every half-integer tie
        np.nextafter(np.arange(-64, 64, 0.5, dtype=np.float32), np.float32(np.inf)),
        np.nextafter(np.arange(-64, 64, 0.5, dtype=np.float32), np.float32(-np.inf)),
        np.float32([0.0, -0.0, 4194303.5, -4194303.5, np.inf]),
    ])
    got = (x + C) - C
    assert got.dtype == np.float32
    assert np.array_equal(got, np.rint(x))
    # the clamp that follows maps NaN to 0 both ways (fmaxf returns the non-NaN operand)
    nan = np.float32(np.nan)
    assert np.fmin(np.fmax((nan + C) - C, np.float32(0)), np.float32(4)) == 0


def test_two_step_bisection_rounds_visit_the_one_step_mids():
    # the kernel evaluates mid and both possible next mids per round; following the outcomes gives the
    # same (lo, hi) sequence as one step per iteration
    rng = np.random.default_rng(1)
    f32 = np.float32
    for _ in range(200):
        lg = (rng.standard_normal(128) * 8).astype(f32)
        B = f32(rng.integers(1, 400))

        def total(mid):
            x = ((lg - f32(mid)).astype(f32) * f32(0.5)).astype(f32)
            return f32(np.clip(np.rint(x), 0, 4).sum())

        lo, hi = f32(-60), f32(60)
        for _ in range(30):
            mid = f32(f32(lo + hi) * f32(0.5))
            if total(mid) > B:
                lo = mid
            else:
                hi = mid
        lo2, hi2 = f32(-60), f32(60)
        for _ in range(15):
            m1 = f32(f32(lo2 + hi2) * f32(0.5))
            mL = f32(f32(lo2 + m1) * f32(0.5))
            mH = f32(f32(m1 + hi2) * f32(0.5))
            if total(m1) > B:
                lo2 = m1
                if total(mH) > B:
                    lo2 = mH
                else:
                    hi2 = mH
            else:
                hi2 = m1
                if total(mL) > B:
                    lo2 = mL
                else:
                    hi2 = mL
        assert (lo, hi) == (lo2, hi2)
