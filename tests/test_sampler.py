"""run.c's sampler (the reference keeps it as llm/runtime.py:37-72): the token
streams of runtime.Sampler equal the reference's own Sampler on the same
seeded logits (tests/golden/sampler.npz, written by make_golden.py from the
reference's class) for greedy, full-distribution and top-p draws."""
import os

import numpy as np

from torch2riscv_accelerator_b200.runtime import Sampler, XorShift64Star

GOLD = os.path.join(os.path.dirname(__file__), "golden", "sampler.npz")


def test_token_streams_equal_the_reference_sampler():
    g = np.load(GOLD)
    for (t, p, seed), want in zip(g["cfgs"], g["tokens"]):
        smp = Sampler(float(t), float(p), int(seed))
        got = [smp(row) for row in g["logits"]]
        assert got == list(want), (t, p, seed)


def test_generator_is_xorshift64_star():
    # run.c's random_u32 from state 1: the first outputs, worked out by hand
    r = XorShift64Star(1)
    x = 1
    x ^= x >> 12
    x ^= (x << 25) & ((1 << 64) - 1)
    x ^= x >> 27
    assert r.u32() == ((x * 0x2545F4914F6CDD1D) & ((1 << 64) - 1)) >> 32
    assert XorShift64Star(0).state == 1
    u = XorShift64Star(3).unit()
    assert 0.0 <= u < 1.0
