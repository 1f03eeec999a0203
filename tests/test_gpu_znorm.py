"""GPU: the z-norm statistics kernel must be bit-identical to the reference's
sequential fp32 chains (triattention.c:227-238) on every input, including the
ones that defeat its chunked fast path (ties, binade crossings, mean ~ 0,
NaN/Inf, subnormals, overflow)."""
import numpy as np
import pytest

import tria_b200

pytestmark = pytest.mark.gpu


def _chains():
    rng = np.random.default_rng(2024)
    F = np.float32
    c = {
        "mean3": (rng.standard_normal(32768) * 4 + 3).astype(F),
        "mean0": (rng.standard_normal(32768) * 4).astype(F),
        "ties_quarter": (rng.integers(-50, 50, 20000) / 4).astype(F),
        "tiny_ties": (rng.integers(-3, 4, 20000) * 2.0 ** -24 + 1.0).astype(F),
        "wide": (rng.standard_normal(20000) * np.exp(rng.uniform(-20, 20, 20000))).astype(F),
        "squares": ((rng.standard_normal(20000) * 4).astype(F) ** 2).astype(F),
        "const": np.full(30000, 0.1, F),
        "halfulps": np.tile(F([2.0 ** 23, 0.5, 0.5, 1.5]), 4096),
        "neg": (-np.abs(rng.standard_normal(20000)) * 3).astype(F),
        "nan": np.where(np.arange(20000) == 5000, np.nan, rng.standard_normal(20000)).astype(F),
        "inf": np.where(np.arange(20000) == 300, np.inf, rng.standard_normal(20000)).astype(F),
        "overflow": np.full(1000, 3e38, F),
        "subnormal": (rng.standard_normal(5000) * 1e-40).astype(F),
        "zeros": np.zeros(4096, F),
        "alternating_big": np.tile(F([1e30, 1.0, -1e30, 1.0]), 2500),
        "n1": F([2.5]),
        "n2": F([1.0, 2.0 ** -30]),
        "n127": (rng.standard_normal(127) + 1).astype(F),
        "n65536": (rng.standard_normal(65536) * 3 + 1).astype(F),
        "n131072": (rng.standard_normal(131072) * 5 + 2).astype(F),
        "n100003": (rng.standard_normal(100003) * 0.01 + 1e4).astype(F),
        "scores_like": (rng.standard_normal(32768) * 4.6 + 3.2).astype(F),
    }
    for i in range(12):
        n = int(rng.integers(1, 40000))
        x = (rng.standard_normal(n) * float(np.exp(rng.uniform(-4, 4))) + float(rng.normal(0, 3))).astype(F)
        if i % 3 == 0:
            x = (np.round(x * 16) / 16).astype(F)
        c[f"rand{i}"] = x
    return c


def _same(a, b):
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


@pytest.mark.parametrize("copies", [1, 9])
def test_znorm_stats_bit_exact(oracle, copies):
    """copies=1: few chains (the whole-pass kernel); copies=9: 306 chains,
    more than two per SM (the window-by-window kernel)."""
    import torch
    base = _chains()
    chains = {f"{k}#{i}": v for i in range(copies) for k, v in base.items()}
    names = list(chains)
    stride = (max(x.size for x in chains.values()) + 63) // 64 * 64
    host = np.full((len(names), stride), np.nan, np.float32)
    n = np.zeros(len(names), np.int32)
    for i, k in enumerate(names):
        host[i, :chains[k].size] = chains[k]
        n[i] = chains[k].size
    dev = torch.device("cuda:0")
    x = torch.from_numpy(host).to(dev)
    out = torch.zeros((len(names), 2), dtype=torch.float32, device=dev)
    tria_b200.znorm_stats(x, stride, n, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    bad = []
    for i, k in enumerate(names):
        m, s = oracle.znorm_stats(chains[k])
        exp = np.array([m, s], np.float32)
        if not _same(got[i], exp).all():
            bad.append((k, got[i].tolist(), exp.tolist()))
    assert not bad, bad


def test_znorm_stats_repeatable(oracle):
    """A second launch over different data is not affected by the first."""
    import torch
    rng = np.random.default_rng(7)
    dev = torch.device("cuda:0")
    for trial in range(2):
        x = (rng.standard_normal((40, 8192)) * (trial + 1) + trial).astype(np.float32)
        n = rng.integers(1, 8193, 40).astype(np.int32)
        out = torch.zeros((40, 2), device=dev)
        tria_b200.znorm_stats(torch.from_numpy(x).to(dev), 8192, n, out)
        got = out.cpu().numpy()
        for i in range(40):
            m, s = oracle.znorm_stats(x[i, :n[i]])
            assert got[i, 0] == m and got[i, 1] == s, (trial, i)
