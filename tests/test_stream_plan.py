"""The multi-GPU streaming schedule (fenix_b200/stream.py) on the CPU: simulated over every rank, each
tile row of the grid runs exactly once, every chunk row is finalised by exactly one rank, and at
the moment it is finalised it holds the contributions of every tile row that reaches it (so the
composed result equals a one-GPU stream of the whole grid), no contribution falls below a
window's floor or past its end."""
import pytest

from oracle import oracle as orc
from fenix_b200.stream import T, row_ranges, stream_actions, stream_window


def simulate(D, P, ov, world, rows=None):
    zs = [int(v) for v in orc.tile_starts(D, P, ov)]
    rows = len(zs) if rows is None else rows
    win = stream_window(zs, rows, P, D, world)
    acts = [stream_actions(zs, rows, P, D, r, world) for r in range(world)]
    state = [{"floor": 0, "acc": {}} for _ in range(world)]
    for r in range(world):  # the lower band's chunk rows start below the floor set at creation
        if r > 0:
            state[r]["floor"] = zs[row_ranges(rows, world)[r][0]] // T
    exported, final, ran = {}, {}, []

    def phase(r, acts_r):
        st = state[r]
        for act in acts_r:
            k = act[0]
            if k == "row":
                zi = act[1]
                ran.append(zi)
                for p in range(zs[zi], min(zs[zi] + P, D)):
                    assert p >= st["floor"] * T, ("contribution below the floor", r, zi, p)
                    assert p < st["floor"] * T + win, ("contribution past the window", r, zi, p)
                    st["acc"].setdefault(p, set()).add(zi)
            elif k == "export":
                exported[r] = {p: set(st["acc"].get(p, set())) for p in range(act[1], act[1] + act[2])}
            elif k == "discard":
                for p in range(st["floor"] * T, act[1] * T):
                    st["acc"].pop(p, None)
                st["floor"] = max(st["floor"], act[1])
            elif k == "finalize":
                for p in range(st["floor"] * T, min(act[1] * T, D)):
                    assert p not in final, ("finalised twice", p)
                    final[p] = set(st["acc"].pop(p, set()))
                st["floor"] = max(st["floor"], act[1])
            elif k == "add":
                for p in range(act[1], act[1] + act[2]):
                    st["acc"].setdefault(p, set()).update(exported[r + 1][p])

    firsts = []
    for r in range(world):
        i = acts[r].index(("barrier",))
        firsts.append(i)
        phase(r, acts[r][:i])
    for r in range(world):
        phase(r, acts[r][firsts[r] + 1:])
    assert sorted(ran) == list(range(rows))
    top = D if rows == len(zs) else zs[rows] // T * T  # whole chunk rows that no unrun row reaches
    for p in range(top):
        want = {zi for zi in range(rows) if zs[zi] <= p < zs[zi] + P}
        assert final.get(p) == want, (p, final.get(p), want)
    return final


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8, 10])
def test_config5_grid(world):
    simulate(2048, 192, 0.5, world)  # 21 tile rows of 192^3 tiles, the out-of-core workload's grid


@pytest.mark.parametrize("D,P,ov,world", [(1024, 128, 0.5, 7), (1000, 128, 0.25, 3), (700, 192, 0.5, 2),
                                          (512, 64, 0.5, 6)])
def test_other_grids(D, P, ov, world):
    simulate(D, P, ov, world)


@pytest.mark.parametrize("world,rows", [(1, 5), (2, 6), (3, 7)])
def test_prefix_sample(world, rows):
    simulate(2048, 192, 0.5, world, rows)


def test_row_ranges_need_two_rows_each():
    assert row_ranges(21, 8) == [(0, 3), (3, 6), (6, 9), (9, 12), (12, 15), (15, 17), (17, 19), (19, 21)]
    with pytest.raises(ValueError):
        row_ranges(5, 3)
