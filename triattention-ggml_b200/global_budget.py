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

The arithmetic of the device path lives in the C ABI (tria_key_histogram,
tria_key_count, tria_select_key); this module is the host orchestration,
written against a small backend interface so that the same code runs on the
GPU with NCCL and, in tests, on CPU gloo ranks.
"""
from __future__ import annotations

import numpy as np

NBINS = 1 << 16


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
