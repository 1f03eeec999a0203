"""Global budget across units (multi-sequence serving), host logic on CPU.

The orchestration in global_budget.py is run against a CPU stand-in for the
device calls (histogram, key count, select by key, key gather), in one
process and on two gloo ranks that each own a contiguous block of layers,
for both exchange protocols (three all-gathers, and one all-gather of
candidates with its fallback); the kept sets must equal the oracle's global
top-k with the (key desc, unit asc, row asc) rule, ties and NaN included.
"""
import os
import socket

import numpy as np
import pytest

import global_budget as gb
import oracle_py


class CpuBackend:
    """Stand-in for DeviceBackend on numpy keys: seq = {"keys": [unit arrays]}."""

    def histogram(self, seq, level, prefix):
        import torch
        h = np.zeros(gb.NBINS, np.int64)
        for k in seq["keys"]:
            k = np.asarray(k, np.uint32)
            if level == 0:
                np.add.at(h, (k >> 16).astype(np.int64), 1)
            else:
                sel = k[(k >> 16) == prefix]
                np.add.at(h, (sel & 0xFFFF).astype(np.int64), 1)
        return torch.from_numpy(h)

    def count(self, seq, key):
        import torch
        seq["_counts"] = np.array([int((np.asarray(k, np.uint32) == key).sum()) for k in seq["keys"]], np.int64)
        return torch.from_numpy(seq["_counts"])

    def histograms(self, seqs, level, prefixes):
        import torch
        return torch.stack([self.histogram(sq, level, p) for sq, p in zip(seqs, prefixes)])

    def rows(self, seq):
        return int(sum(len(k) for k in seq["keys"]))

    def candidates(self, seqs, key_mins, cap):
        """[n_seq, CAND_HEAD + cap] int64: the count, then the keys >= key_mins[s]."""
        import torch
        buf = np.zeros((len(seqs), gb.CAND_HEAD + cap), np.int64)
        for s, (sq, km) in enumerate(zip(seqs, key_mins)):
            c = np.concatenate([np.asarray(k, np.uint32) for k in sq["keys"]] + [np.zeros(0, np.uint32)])
            c = c[c >= np.uint32(km)].astype(np.int64)
            buf[s, 0] = c.size
            buf[s, gb.CAND_HEAD:gb.CAND_HEAD + min(c.size, cap)] = c[:cap]
        return torch.from_numpy(buf)

    @staticmethod
    def candidate_counts(g):
        return g[:, :, 0].numpy().astype(np.int64)

    @staticmethod
    def _gathered(g, counts, s):
        return {"keys": [g[r, s, gb.CAND_HEAD:gb.CAND_HEAD + int(counts[r, s])].numpy().astype(np.uint32)
                         for r in range(g.shape[0])]}

    def gathered_histograms(self, g, counts, level, prefixes):
        return self.histograms([self._gathered(g, counts, s) for s in range(g.shape[1])], level, prefixes)

    def gathered_ties(self, g, counts, keys):
        out = np.zeros((g.shape[0], g.shape[1]), np.int64)
        for s in range(g.shape[1]):
            for r, k in enumerate(self._gathered(g, counts, s)["keys"]):
                out[r, s] = int((k == np.uint32(keys[s])).sum())
        return out

    def select(self, seq, key, tie_allow):
        kept, before = [], 0
        for k, c in zip(seq["keys"], seq["_counts"]):
            k = np.asarray(k, np.uint32)
            allow = max(0, min(tie_allow - before, int(c)))
            eq = np.flatnonzero(k == key)[:allow]
            kept.append(np.sort(np.concatenate([np.flatnonzero(k > key), eq])))
            before += int(c)
        seq["kept"] = kept


def _make_seq_keys(rng, n_units, lo, hi, heavy_ties):
    keys = []
    for _ in range(n_units):
        n = int(rng.integers(lo, hi + 1))
        x = rng.standard_normal(n).astype(np.float32)
        if heavy_ties:
            x = (np.round(x * 2) / 2).astype(np.float32)
            x[: n // 20] = np.nan
        keys.append(oracle_py.score_keys(x))
    return keys


def test_boundary_bin():
    h = np.zeros(gb.NBINS, np.int64)
    h[[10, 500, 65535]] = [5, 3, 2]
    assert gb.boundary_bin(h, 1) == (65535, 1)
    assert gb.boundary_bin(h, 2) == (65535, 2)
    assert gb.boundary_bin(h, 3) == (500, 1)
    assert gb.boundary_bin(h, 5) == (500, 3)
    assert gb.boundary_bin(h, 6) == (10, 1)
    assert gb.boundary_bin(h, 10) == (10, 5)


def test_boundary_bins_match_boundary_bin():
    """The batched (torch) search gives boundary_bin's answer on every row."""
    import torch
    rng = np.random.default_rng(0)
    h = np.zeros((5, gb.NBINS), np.int64)
    for s in range(5):
        idx = rng.integers(0, gb.NBINS, 40)
        np.add.at(h[s], idx, rng.integers(1, 50, 40))
    h[4, -1] = 7                                  # a key in the top bin
    needs = [1, int(h[1].sum()), int(h[2].sum()) // 2, 17, 3]
    got = gb.boundary_bins(torch.from_numpy(h), needs)
    assert got == [gb.boundary_bin(h[s], needs[s]) for s in range(5)]


def test_score_keys_match_the_library():
    import tria_b200
    x = np.array([0.0, -0.0, 1.5, -1.5, np.inf, -np.inf, np.nan, 1e-40, -1e-40], np.float32)
    assert [tria_b200.score_key(float(v)) for v in x] == oracle_py.score_keys(x).tolist()


PROTOCOLS = {
    "histograms": gb.global_select,
    "candidates": gb.global_select_candidates,
    "candidates-overflow": lambda *a: gb.global_select_candidates(*a, cap=8),     # always falls back
}


@pytest.mark.parametrize("protocol", sorted(PROTOCOLS))
@pytest.mark.parametrize("heavy_ties", [False, True])
def test_global_select_one_rank(heavy_ties, protocol):
    import torch
    rng = np.random.default_rng(3 + heavy_ties)
    seqs, ks = [], []
    for s in range(4):
        keys = _make_seq_keys(rng, 12, 0 if s == 3 else 50, 400, heavy_ties)
        seqs.append({"keys": keys})
        ks.append([0, 17, 900, 10**6][s])
    PROTOCOLS[protocol](seqs, ks, lambda t: t[None], CpuBackend(), 0)
    for sq, k in zip(seqs, ks):
        exp = oracle_py.global_select(sq["keys"], k)
        assert len(sq["kept"]) == len(exp)
        for a, b in zip(sq["kept"], exp):
            assert np.array_equal(a, b)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, protocol="histograms"):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        all_seqs = [_make_seq_keys(rng, 16, 1, 300, s % 2 == 1) for s in range(3)]   # 16 units = 4 layers x 4 heads
        ks = [100, 1234, 5000]
        per = 16 // world
        mine = [{"keys": keys[rank * per:(rank + 1) * per]} for keys in all_seqs]

        def gather(t):
            out = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(out, t.contiguous())
            return torch.stack(out)

        PROTOCOLS[protocol](mine, ks, gather, CpuBackend(), rank)
        q.put((rank, [[k.tolist() for k in sq["kept"]] for sq in mine], [[k.tolist() for k in x] for x in all_seqs], ks))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("protocol", sorted(PROTOCOLS))
def test_global_select_two_gloo_ranks(protocol):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, protocol)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    all_seqs, ks = res[0][2], res[0][3]
    for s, keys in enumerate(all_seqs):
        exp = oracle_py.global_select([np.array(k, np.uint32) for k in keys], ks[s])
        got = res[0][1][s] + res[1][1][s]
        assert len(got) == len(exp)
        for a, b in zip(got, exp):
            assert a == b.tolist()


def _dead_rank_main(rank, world, port, q, mode, dead):
    """One global-budget step on every rank, then rank `dead` leaves (exits,
    or stalls without joining the next step); the others run a second step
    and must get an error from their next gather, not hang."""
    import time
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    rng = np.random.default_rng(5)
    all_seqs = [_make_seq_keys(rng, 12, 1, 200, False) for _ in range(2)]
    per = 12 // world
    mine = [{"keys": keys[rank * per:(rank + 1) * per]} for keys in all_seqs]

    def gather(t):
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t.contiguous())
        return torch.stack(out)

    gb.global_select(mine, [50, 500], gather, CpuBackend(), rank)          # step 1: every rank
    def report(*msg):                          # flush before os._exit, which skips the queue's feeder
        q.put(msg)
        q.close()
        q.join_thread()

    if rank == dead:
        report(rank, "left", 0.0)
        if mode == "stall":
            time.sleep(60)                                                  # never joins step 2
        os._exit(0)
    t0 = time.monotonic()
    try:
        gb.global_select(mine, [50, 500], gather, CpuBackend(), rank)      # step 2: a peer is gone
        report(rank, "no error", time.monotonic() - t0)
    except Exception as e:                                                  # noqa: BLE001
        report(rank, "error: " + type(e).__name__, time.monotonic() - t0)
    os._exit(0)                                # no destroy_process_group with a peer gone


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_global_select_dead_rank_fails_fast(mode):
    """Failure detection on the collective path: a rank that exits or stops
    between steps makes every other rank's next step raise within the process
    group's timeout (4 s here) instead of waiting forever."""
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world, dead = 3, 2
    procs = [ctx.Process(target=_dead_rank_main, args=(r, world, port, q, mode, dead)) for r in range(world)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=90) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=5)
            if p.is_alive():
                p.kill()
                p.join()
    assert res[dead][1] == "left"
    for r in range(world):
        if r == dead:
            continue
        assert res[r][1].startswith("error"), res
        assert res[r][2] < 30.0, res                     # bounded by the group timeout, not a hang
    assert time.monotonic() - t0 < 120
