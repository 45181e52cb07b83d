"""Work schedule of the fused collective kernel, checked on the host.

The kernel hands out tickets through `coll_schedule_item` (the same function
runs here through the extension).  Deadlock freedom with any number of
resident CTAs needs two properties, checked for every op, world size and lag:
the order is a permutation of the work items, and every item a rank waits for
(on itself or on a peer, which uses the same order) is handed out at an
earlier ticket.
"""

import pytest

from bitscom_b200 import _ext

C = _ext.require()

TWO_SHOT, ONE_SHOT, RS, AG = 0, 1, 2, 3


def phase_items(op, w):
    return {TWO_SHOT: (w, 1, w - 1), RS: (w, 1, 0), ONE_SHOT: (1, 1, 0), AG: (1, 0, w - 1)}[op]


def dependencies(op, w, IS, item):
    """Items (in phase-major numbering, on some rank) that `item` waits for."""
    a1, a2, a3 = phase_items(op, w)
    n1, n2 = a1 * IS, a2 * IS
    if item < n1:
        return []
    if item < n1 + n2:  # owner reduce of chunk c: phase 1 of chunk c on every rank
        c = item - n1
        return [c * a1 + k for k in range(a1)]
    c = (item - n1 - n2) // a3
    if a2:  # decode of a peer's reduced chunk: that owner's phase 2
        return [n1 + c]
    return [c]  # all-gather: the source's phase 1


@pytest.mark.parametrize("op", [TWO_SHOT, ONE_SHOT, RS, AG])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("IS,lag", [(1, 1), (5, 0), (5, 1), (5, 2), (37, 4), (37, 9), (37, 36), (37, 100), (64, 16)])
def test_schedule_is_a_permutation_and_dependencies_come_first(op, world, IS, lag):
    if op == AG and world == 1:
        pytest.skip("all-gather at world size 1 has no phase 3")
    order = C.coll_schedule(op, world, IS, lag)
    a1, a2, a3 = phase_items(op, world)
    total = (a1 + a2 + a3) * IS
    assert sorted(order) == list(range(total))
    pos = {item: t for t, item in enumerate(order)}
    for t, item in enumerate(order):
        for dep in dependencies(op, world, IS, item):
            assert pos[dep] < t, (op, world, IS, lag, item, dep)


@pytest.mark.parametrize("lag", [0, -3, 37, 1000])
def test_lag_zero_or_large_is_phase_major(lag):
    order = C.coll_schedule(TWO_SHOT, 8, 37, lag)
    assert order == list(range(len(order)))


def test_interleaving_starts_reduce_before_encode_ends():
    IS, lag, w = 64, 4, 8
    order = C.coll_schedule(TWO_SHOT, w, IS, lag)
    n1 = w * IS
    first_reduce = next(t for t, i in enumerate(order) if i >= n1)
    # Phase 2 of chunk 0 is handed out right after phase 1 of chunk `lag`.
    assert first_reduce == (lag + 1) * w
    assert order[first_reduce] == n1
    # The last ticket is a decode of the last chunk.
    assert order[-1] == len(order) - 1
