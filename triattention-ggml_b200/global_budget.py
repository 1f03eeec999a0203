"""Global budget across the (layer, kv-head) units of each sequence.

Multi-sequence serving evicts with one budget per sequence rather than a
fixed count per unit: sequence s keeps its best K_s rows over all of its
units, ranked by (key desc, unit asc, row asc), where key is the
order-preserving 32-bit key of the z-max score (include/triattention.h,
tria_score_key) and units are ordered (layer, kv-head).  The ranks of one
node each own a contiguous block of layers (rank order = layer order) and
agree on one threshold key per sequence through three all-gathers:

  1. 16-bit histograms of the keys' high halves -> the boundary bin b_s;
  2. 16-bit histograms of the low halves inside b_s -> the threshold key T_s
     and how many rows equal to T_s are still needed;
  3. each rank's count of rows equal to T_s -> how many of its own it keeps
     (rows equal to T_s go in unit order, so ranks holding earlier layers
     keep theirs first).

Every rank then keeps rows with key > T_s plus its share of the rows equal
to T_s, which makes the kept sets exactly the global top K_s.

global_select_candidates reaches the same kept sets with one all-gather: each
rank finds its own K_s-th largest key (steps 1-2 on its own rows), gathers
the scores at or above it (tria_key_gather), and every rank runs steps 1-3 on
the gathered candidates.  The global K_s-th key is never below a rank's own,
so the candidates hold every kept row and every row equal to the threshold.
If a rank has more candidates than the exchange buffer holds (many ties at
its own threshold), every rank sees that in the gathered counts and falls
back to global_select.

The arithmetic of the device path lives in the C ABI (tria_key_histogram,
tria_key_count, tria_select_key, tria_key_gather); this module is the host
orchestration, written against a small backend interface so that the same
code runs on the GPU with NCCL and, in tests, on CPU gloo ranks.
"""
from __future__ import annotations

import numpy as np

NBINS = 1 << 16
CAND_HEAD = 4        # header floats of a candidate row (count first); keeps the scores 16-byte aligned


def boundary_bin(hist, need):
    """Bin b (counting from the top) where the count of keys in bins >= b first
    reaches `need`, and how many of bin b's keys are needed.  `need` must be in
    [1, hist.sum()]."""
    h = np.asarray(hist, np.int64)
    from_top = np.cumsum(h[::-1])
    i = int(np.searchsorted(from_top, need))
    b = NBINS - 1 - i
    above = int(from_top[i] - h[b])
    return b, int(need - above)


def boundary_bins(hists, needs):
    """boundary_bin for every row of hists [n_seq, NBINS] at once (need >= 1),
    on the tensor's own device: only the (bin, need) pairs come back."""
    import torch
    h = hists.to(torch.int64)
    from_top = torch.cumsum(h.flip(1), dim=1)
    nd = torch.as_tensor(needs, dtype=torch.int64, device=h.device).reshape(-1, 1)
    i = torch.searchsorted(from_top, nd).clamp_(max=NBINS - 1)
    b = NBINS - 1 - i
    rest = nd - (from_top.gather(1, i) - h.gather(1, b))
    res = torch.cat([b, rest], 1).cpu().numpy()
    return [(int(x), int(y)) for x, y in res]


class DeviceBackend:
    """The GPU path: z-max scores on the device ([units][stride] fp32) of the
    units this rank owns for one sequence, processed through the C ABI.
    histograms() fills one preallocated [n_seq, NBINS] buffer for all
    sequences of a level, so a level costs one copy and one gather."""

    def __init__(self, device, stream=None):
        self.device = device
        self.stream = stream
        self._hbuf = None

    def histograms(self, seqs, level, prefixes):
        import torch
        import tria_b200
        n = len(seqs)
        if self._hbuf is None or self._hbuf.shape[0] < n:
            self._hbuf = torch.zeros((n, NBINS), dtype=torch.int32, device=self.device)
        h = self._hbuf[:n]
        h.zero_()
        for s, (sq, p) in enumerate(zip(seqs, prefixes)):
            tria_b200.key_histogram(sq["scores"], sq["stride"], sq["n_rows"], level, p, h[s], self.stream)
        return h

    def counts(self, seqs, keys):
        """count() for every sequence into one buffer; returns [n_seq] int64 totals."""
        import torch
        import tria_b200
        width = max(len(sq["n_rows"]) for sq in seqs)
        buf = torch.zeros((len(seqs), width), dtype=torch.int32, device=self.device)
        for s, (sq, key) in enumerate(zip(seqs, keys)):
            c = buf[s, :len(sq["n_rows"])]
            tria_b200.key_count(sq["scores"], sq["stride"], sq["n_rows"], key, c, self.stream)
            sq["_counts"] = c
        return buf.to(torch.int64).sum(1)

    def histogram(self, seq, level, prefix):
        import torch
        import tria_b200
        h = torch.zeros(NBINS, dtype=torch.int32, device=self.device)
        tria_b200.key_histogram(seq["scores"], seq["stride"], seq["n_rows"], level, prefix, h, self.stream)
        return h.to(torch.int64)

    def count(self, seq, key):
        import torch
        import tria_b200
        c = torch.zeros(len(seq["n_rows"]), dtype=torch.int32, device=self.device)
        tria_b200.key_count(seq["scores"], seq["stride"], seq["n_rows"], key, c, self.stream)
        seq["_counts"] = c
        return c.to(torch.int64)

    def select(self, seq, key, tie_allow):
        import tria_b200
        tria_b200.select_key(seq["scores"], seq["stride"], seq["n_rows"], key, seq["_counts"], tie_allow,
                             seq["kept_idx"], seq["kept_stride"], seq["n_kept"], self.stream)

    # ---- one exchange (global_select_candidates) ----

    def rows(self, seq):
        return int(np.asarray(seq["n_rows"], np.int64).sum())

    def candidates(self, seqs, key_mins, cap):
        """[n_seq, CAND_HEAD + cap] fp32: column 0 the candidate count, then the
        scores whose key is >= key_mins[s] (tria_key_gather)."""
        import torch
        import tria_b200
        buf = torch.zeros((len(seqs), CAND_HEAD + cap), dtype=torch.float32, device=self.device)
        cnt = torch.zeros(len(seqs), dtype=torch.int32, device=self.device)
        for s, (sq, k) in enumerate(zip(seqs, key_mins)):
            tria_b200.key_gather(sq["scores"], sq["stride"], sq["n_rows"], k, buf[s, CAND_HEAD:], cap,
                                 cnt[s:s + 1], self.stream)
        buf[:, 0] = cnt.to(torch.float32)
        return buf

    @staticmethod
    def candidate_counts(g):
        """Host [world, n_seq] candidate counts of the gathered buffers."""
        import torch
        return g[:, :, 0].to(torch.int64).cpu().numpy()

    def _gathered(self, g, counts, s):
        """Sequence s of the gathered buffers as `world` units of candidate scores."""
        world, n_seq, width = g.shape
        return {"scores": g[:, s, CAND_HEAD:], "stride": n_seq * width,
                "n_rows": np.minimum(counts[:, s], width - CAND_HEAD).astype(np.int32)}

    def gathered_histograms(self, g, counts, level, prefixes):
        return self.histograms([self._gathered(g, counts, s) for s in range(g.shape[1])], level, prefixes)

    def gathered_ties(self, g, counts, keys):
        """Host [world, n_seq]: each rank's candidates equal to keys[s]."""
        import torch
        import tria_b200
        world, n_seq = g.shape[0], g.shape[1]
        out = torch.zeros((n_seq, world), dtype=torch.int32, device=self.device)
        for s in range(n_seq):
            sq = self._gathered(g, counts, s)
            tria_b200.key_count(sq["scores"], sq["stride"], sq["n_rows"], keys[s], out[s], self.stream)
        return out.t().to(torch.int64).cpu().numpy()


def global_select(seqs, k_total, gather, backend, rank):
    """Keep the global top k_total[s] rows of every sequence s.

    seqs     per sequence, this rank's units (a dict the backend understands)
    k_total  per sequence, rows to keep over all ranks' units
    gather   all-gather over the ranks: tensor [...] -> tensor [world, ...]
    backend  DeviceBackend (or a CPU stand-in with the same methods)
    rank     this rank's position in layer order
    Returns per sequence (threshold key, rows equal to it kept by this rank).
    """
    import torch
    n_seq = len(seqs)

    def level_hists(level, prefixes):
        if hasattr(backend, "histograms"):
            return backend.histograms(seqs, level, prefixes)
        return torch.stack([backend.histogram(sq, level, p) for sq, p in zip(seqs, prefixes)])

    # 1. high halves (the bin search runs where the summed histograms are;
    #    the totals ride along in the same copy)
    g0 = gather(level_hists(0, [0] * n_seq)).to(torch.int64).sum(0)
    totals = g0.sum(1).cpu().numpy()
    ks = [min(int(k_total[s]), int(totals[s])) for s in range(n_seq)]
    live = [s for s in range(n_seq) if ks[s] > 0]
    bins, needs = [None] * n_seq, [0] * n_seq
    if live:
        for s, (b, need) in zip(live, boundary_bins(g0[live], [ks[s] for s in live])):
            bins[s], needs[s] = b, need
    # 2. low halves inside the boundary bins
    g1 = gather(level_hists(1, [b if b is not None else 0 for b in bins])).to(torch.int64).sum(0)
    keys, needs2 = [0xFFFFFFFF] * n_seq, [0] * n_seq   # dead sequences: nothing above the key, no ties allowed
    if live:
        for s, (t, need2) in zip(live, boundary_bins(g1[live], [needs[s] for s in live])):
            keys[s] = (bins[s] << 16) | t
            needs2[s] = need2
    # 3. rows equal to the threshold, in rank (layer) order
    if hasattr(backend, "counts"):
        ties = backend.counts(seqs, keys)
    else:
        ties = torch.stack([backend.count(sq, key).sum() for sq, key in zip(seqs, keys)])
    gt = gather(ties).cpu().numpy()              # [world, n_seq]
    out = []
    for s in range(n_seq):
        before = int(gt[:rank, s].sum())
        allow = max(0, min(needs2[s] - before, int(gt[rank, s])))
        backend.select(seqs[s], keys[s], allow)
        out.append((keys[s], allow))
    return out


def global_select_candidates(seqs, k_total, gather, backend, rank, cap=None):
    """global_select with one all-gather: same arguments and result.

    cap is the candidate buffer per sequence and rank (a multiple of 4,
    default max(k_total) + 4096); a rank with more candidates than that in
    any sequence makes every rank fall back to global_select.
    """
    import torch
    n_seq = len(seqs)
    if cap is None:
        cap = max([int(k) for k in k_total] + [0]) + 4096
    cap = (int(cap) + 3) & ~3

    # this rank's own K_s-th largest key: steps 1-2 on its own rows
    rows = [backend.rows(sq) for sq in seqs]
    kl = [min(int(k_total[s]), rows[s]) for s in range(n_seq)]
    key_min = [0] * n_seq                                  # 0: every row is a candidate
    part = [s for s in range(n_seq) if 0 < kl[s] < rows[s]]
    for s in range(n_seq):
        if kl[s] == 0:
            key_min[s] = 0xFFFFFFFF                        # above every score key: no candidate
    if part:
        sub = [seqs[s] for s in part]
        h0 = backend.histograms(sub, 0, [0] * len(part))
        b0 = boundary_bins(h0, [kl[s] for s in part])
        h1 = backend.histograms(sub, 1, [b for b, _ in b0])
        for s, (b, _), (t, _) in zip(part, b0, boundary_bins(h1, [need for _, need in b0])):
            key_min[s] = (b << 16) | t

    # the one exchange
    g = gather(backend.candidates(seqs, key_min, cap))     # [world, n_seq, CAND_HEAD + cap]
    counts = backend.candidate_counts(g)                   # host [world, n_seq]
    if (counts > cap).any():
        return global_select(seqs, k_total, gather, backend, rank)

    # steps 1-3 on the gathered candidates, the same on every rank
    totals = counts.sum(0)
    ks = [min(int(k_total[s]), int(totals[s])) for s in range(n_seq)]
    live = [s for s in range(n_seq) if ks[s] > 0]
    keys, needs2 = [0xFFFFFFFF] * n_seq, [0] * n_seq
    if live:
        gh0 = backend.gathered_histograms(g, counts, 0, [0] * n_seq)
        bins = [0] * n_seq
        needs = [0] * n_seq
        for s, (b, need) in zip(live, boundary_bins(gh0[live], [ks[s] for s in live])):
            bins[s], needs[s] = b, need
        gh1 = backend.gathered_histograms(g, counts, 1, bins)
        for s, (t, need2) in zip(live, boundary_bins(gh1[live], [needs[s] for s in live])):
            keys[s] = (bins[s] << 16) | t
            needs2[s] = need2
    ties = backend.gathered_ties(g, counts, keys)           # host [world, n_seq]
    out = []
    for s in range(n_seq):
        before = int(ties[:rank, s].sum())
        allow = max(0, min(needs2[s] - before, int(ties[rank, s])))
        backend.count(seqs[s], keys[s])                     # this rank's per-unit ties, for the selection
        backend.select(seqs[s], keys[s], allow)
        out.append((keys[s], allow))
    return out

