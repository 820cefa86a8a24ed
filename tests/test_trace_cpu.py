"""The device-timeline reader (torch2riscv_accelerator_b200/trace.py) on
synthetic records: grouping into launches and the per-kind summary."""
import numpy as np

from torch2riscv_accelerator_b200 import trace

M = trace.MARKS


def block(kind, grid, cta, t0, marks):
    """One CTA's record block: mark j at global time t0 + marks[j] ns, the SM
    clock equal to it (1 GHz). t0 > 0: a zero time marks an unused block."""
    b = np.zeros((M, 3), dtype=np.uint64)
    for j, dt in marks.items():
        b[j, 0] = t0 + dt
        b[j, 1] = t0 + dt
        b[j, 2] = (kind << 56) | (j << 48) | (7 << 32) | (grid << 16) | cta
    return b


def test_launches_split_on_grid_size_and_count():
    # a 3-CTA GEMV launch, then a 4-CTA one whose first CTA index (3) is new to
    # the first launch, then a 3-CTA launch of the same size as the first
    blocks = []
    for c in (2, 0, 1):
        blocks.append(block(1, 3, c, 1000, {0: 0, 1: 500, 2: 900}))
    for c in (3, 1, 0, 2):
        blocks.append(block(1, 4, c, 3000, {0: 0, 1: 400, 2: 800}))
    for c in (0, 1, 2):
        blocks.append(block(1, 3, c, 6000, {0: 0, 1: 300, 2: 700}))
    raw = np.concatenate(blocks)
    ls = trace.launches(raw)
    assert [len(L["ctas"]) for L in ls] == [3, 4, 3]
    assert [L["grid"] for L in ls] == [3, 4, 3]
    kinds, span, n = trace.summarise(raw, sm_ghz=1.0)
    assert n == 3
    g = kinds["gemv"]
    assert g["launches"] == 2                                  # the first launch has no predecessor
    # second launch: released 400 ns after its entry, previous end at 1900
    assert abs(g["gap_us"] - np.median([(3400 - 1900) / 1e3, (6300 - 3800) / 1e3])) < 1e-9
    assert g["phases_us"]["1-2"] == round(np.median([0.4, 0.4]), 2)


def test_kind_change_starts_a_launch():
    raw = np.concatenate([block(1, 2, 0, 5, {0: 0, 1: 10}), block(2, 2, 1, 50, {0: 0, 1: 10}),
                          block(2, 2, 0, 60, {0: 0, 1: 10})])
    ls = trace.launches(raw)
    assert [(L["kind"], len(L["ctas"])) for L in ls] == [("gemv", 1), ("attn", 2)]
