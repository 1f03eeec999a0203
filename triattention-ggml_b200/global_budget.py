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


class DeviceBackend:
    """The GPU path: z-max scores on the device ([units][stride] fp32) of the
    units this rank owns for one sequence, processed through the C ABI."""

    def __init__(self, device, stream=None):
        self.device = device
        self.stream = stream

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
    # 1. high halves
    h0 = torch.stack([backend.histogram(sq, 0, 0) for sq in seqs])
    g0 = gather(h0).sum(0).cpu().numpy()
    bins, needs = [], []
    for s in range(n_seq):
        total = int(g0[s].sum())
        k = min(int(k_total[s]), total)
        if k <= 0:
            bins.append(None)
            needs.append(0)
            continue
        b, need = boundary_bin(g0[s], k)
        bins.append(b)
        needs.append(need)
    # 2. low halves inside the boundary bins
    h1 = torch.stack([backend.histogram(sq, 1, b if b is not None else 0) for sq, b in zip(seqs, bins)])
    g1 = gather(h1).sum(0).cpu().numpy()
    keys, needs2 = [], []
    for s in range(n_seq):
        if bins[s] is None:
            keys.append(0xFFFFFFFF)              # nothing above it, no rows equal to it allowed
            needs2.append(0)
            continue
        t, need2 = boundary_bin(g1[s], needs[s])
        keys.append((bins[s] << 16) | t)
        needs2.append(need2)
    # 3. rows equal to the threshold, in rank (layer) order
    ties = torch.stack([backend.count(sq, key).sum() for sq, key in zip(seqs, keys)])
    gt = gather(ties).cpu().numpy()              # [world, n_seq]
    out = []
    for s in range(n_seq):
        before = int(gt[:rank, s].sum())
        allow = max(0, min(needs2[s] - before, int(gt[rank, s])))
        backend.select(seqs[s], keys[s], allow)
        out.append((keys[s], allow))
    return out
