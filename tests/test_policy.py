"""Runtime policy of the reference's llama.cpp integration (QUICKSTART.md:41-45):
budget as retention %, window, interval and sink; ramp stages 10/20/40/80/100;
and per-sequence cache lengths (README.md:92).  Host-only, no GPU."""
import numpy as np
import pytest

import tria_b200


def test_policy_schedule():
    p = tria_b200.Policy(budget_pct=75, window=512, interval=128, sink=4)
    due = []
    n_kv = 0
    for n_past in range(0, 2000):
        n_kv += 1
        prm = p.due(n_past, n_kv)
        if prm is not None:
            due.append((n_past, n_kv, prm.budget, prm.ramp_pct, prm.window, prm.sink, prm.cur_pos))
            n_kv = prm.budget                    # the cache shrinks to the budget (ramp aside)
    first = due[0]
    assert first[1] == 512 + 4 + 128 + 1          # first once n_kv > window + sink + interval
    assert [d[0] - due[0][0] for d in due[:4]] == [0, 128, 256, 384]
    assert [d[3] for d in due[:7]] == [10, 20, 40, 80, 100, 100, 100]
    for d in due:
        assert d[2] == max(1, d[1] * 75 // 100) and d[4] == 512 and d[5] == 4 and d[6] == d[0]


def test_policy_clamps_and_errors():
    p = tria_b200.Policy(budget_pct=0, window=-5, interval=0, sink=-1)
    assert (p.budget_pct, p.window, p.interval, p.sink) == (1, 0, 1, 0)
    with pytest.raises(tria_b200.TriaError):
        p.due(-1, 10)


def test_n_kv_per_seq():
    nk = np.array([5, 9, 3, 7, 0, 2], np.int32)
    seq = np.array([0, 0, 1, 1, 2, 2], np.int32)
    assert tria_b200.n_kv_per_seq(nk, seq, 3).tolist() == [9, 7, 2]
    with pytest.raises(tria_b200.TriaError):
        tria_b200.n_kv_per_seq(nk, np.array([0, 0, 1, 1, 2, 5], np.int32), 3)
