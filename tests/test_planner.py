"""CPU: the decode planner's split choice against measured split sweeps.

The planner (eakv_b200/csrc/decode.cu) cuts every (cache, layer, KV head)
row into splits of whole pages and picks the split count from a makespan
model. This test calls the model's choice through the C-ABI (pure host
code, no kernel) for the BASELINE shapes and checks that the choice is one
whose measured step time, on one B200 with the tensor-core decode kernel, is
within 5 % of the best split count measured for that shape.

Each table maps a split count to the measured time of one decode launch in
microseconds (bench.py --splits N; cfg4/cfg5 full steps in ms). `lo` is the
fewest splits the precision cap allows (no split longer than 256 pages),
`hi` the most (two pages per split); per_sm is the number of CTAs of the
kernel resident on one of the 148 SMs (4 with 4 query heads per CTA, 3 with
8 at head_dim 128).
"""
import pytest

SMS = 148

SHAPES = [
    # name, rows (items), pages per row, lo, hi, per_sm, {splits: measured time}
    ("cfg1 MHA d128 S2048", 8, 32, 1, 16, 4, {2: 22.5, 4: 17.1, 8: 16.2, 16: 16.5}),
    ("cfg2 GQA 8:1 d64 S2048", 88, 32, 1, 16, 4, {2: 22.6, 3: 22.5, 4: 21.7, 8: 27.4, 16: 35.0}),
    ("cfg3 MHA d128 S8192", 1024, 128, 1, 64, 4,
     {1: 263.2, 2: 273.0, 3: 281.5, 4: 286.6, 5: 294.6, 6: 303.5, 8: 319.5, 9: 333.3,
      10: 342.6, 12: 360.0, 16: 387.1}),
    ("cfg4 one sequence", 256, 512, 2, 256, 4,
     {2: 276.0, 3: 295.8, 4: 258.0, 5: 275.2, 6: 270.1, 7: 277.5, 8: 268.5, 9: 270.7,
      11: 276.1, 16: 291.4, 19: 298.9, 23: 309.0, 32: 332.6, 37: 355.9}),
    ("cfg4 16 sequences", 4096, 512, 2, 256, 4, {2: 3512.2, 3: 3538.8, 4: 3571.9}),
    ("cfg5 4 sequences", 2560, 2048, 8, 1024, 3, {8: 12065.9, 10: 12076.7, 16: 12201.8}),
]


@pytest.mark.parametrize("name,items,pages,lo,hi,per_sm,measured", SHAPES,
                         ids=[s[0] for s in SHAPES])
def test_planner_picks_a_measured_best_split(name, items, pages, lo, hi, per_sm, measured):
    import eakv_b200 as E
    ns = E.choose_splits(items, pages, lo, hi, per_sm, SMS)
    assert lo <= ns <= hi
    assert ns in measured, f"{name}: chose {ns} splits, not among the measured {sorted(measured)}"
    best = min(measured.values())
    assert measured[ns] <= 1.05 * best, f"{name}: {ns} splits measured {measured[ns]}, best {best}"


def test_planner_bounds_and_degenerate_inputs():
    import eakv_b200 as E
    assert E.choose_splits(100, 1, 1, 1, 4, SMS) == 1
    assert E.choose_splits(100, 64, 5, 5, 4, SMS) == 5      # a single candidate
    assert E.choose_splits(100, 64, 3, 2, 4, SMS) == 3      # empty range: the lower bound
    assert E.choose_splits(0, 64, 1, 32, 4, SMS) >= 1


def _model_choice(items, max_pages, lo, hi, per_sm, sms):
    """The makespan model evaluated at every split count in [lo, hi] (the
    first of equal costs wins): the reference for the library's shortcut,
    which evaluates one count per split length and remembers recent answers."""
    best, ns = None, lo
    for k in range(lo, hi + 1):
        sp = -(-max_pages // k)
        n = -(-max_pages // sp)
        m = -(-(items * n) // sms)
        rounds = -(-m // per_sm)
        r = m - per_sm * (rounds - 1)
        c = (sp + 8.0) * ((rounds - 1) + (r / per_sm) ** (2.0 / 3.0))
        if best is None or c < best:
            best, ns = c, k
    return ns


def test_planner_shortcut_equals_the_full_scan():
    import random

    import eakv_b200 as E
    rnd = random.Random(7)
    cases = [(items, pages, 1, pages, per_sm)
             for items in (1, 8, 88, 256, 1024, 4096)
             for pages in (1, 2, 3, 7, 32, 129, 512, 2048)
             for per_sm in (1, 3, 4)]
    cases += [(rnd.randint(1, 20000), rnd.randint(1, 3000), 0, 0, rnd.randint(1, 8))
              for _ in range(300)]
    for items, pages, lo, hi, per_sm in cases:
        if hi == 0:
            lo = rnd.randint(1, pages)
            hi = rnd.randint(lo, pages)
        want = _model_choice(items, pages, lo, hi, per_sm, SMS)
        # twice: the second answer comes from the per-thread memo
        for _ in range(2):
            assert E.choose_splits(items, pages, lo, hi, per_sm, SMS) == want, \
                (items, pages, lo, hi, per_sm)
