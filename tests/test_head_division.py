"""The fused output head (head_tc.cu) divides by the action standard
deviation with Markstein's correction instead of the general IEEE division
routine: y = RN(1 / b), q = RN(a y), r = RN(a - b q) (one fused multiply-add),
result RN(q + r y) (another).  ActorCritic::logp (ppo.rs:297-305) divides
(a - mu) / exp(log_std) in f32, so the head's log-probabilities are only
the reference's if this gives the correctly rounded quotient on the head's
operands.  Checked here in exact rational arithmetic on a seeded sample of
that domain: b = exp(log_std) with log_std in the clamp range [-1.6, 1.0]
(ppo.rs:508), a a difference of an action and a mean over eight decades."""
import random
from fractions import Fraction as F

import numpy as np


def rn32(x: F) -> F:
    """x rounded to the nearest float32 (ties to even), exactly."""
    if x == 0:
        return F(0)
    s = -1 if x < 0 else 1
    x = abs(x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    while F(2) ** e > x:
        e -= 1
    while F(2) ** (e + 1) <= x:
        e += 1
    scale = F(2) ** (23 - e)
    m = x * scale
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return s * F(fl) / scale


def test_markstein_division_is_correctly_rounded_on_the_head_domain():
    rng = random.Random(2024)
    for i in range(20000):
        ls = np.float32(rng.uniform(-1.6, 1.0))
        b = F(float(np.float32(np.exp(ls)))) if i % 2 else F(float(np.float32(rng.uniform(0.2, 2.72))))
        a = F(float(np.float32(rng.gauss(0.0, 1.0) * 10 ** rng.uniform(-6, 1))))
        y = rn32(1 / b)
        q = rn32(a * y)
        r = rn32(a - b * q)
        assert rn32(q + r * y) == rn32(a / b), (float(a), float(b))
