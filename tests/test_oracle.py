"""CPU tests: pin the oracle against the reference's golden vectors and the
compiled reference C, and check the select/compact restatement against an
independent numpy formulation."""
import os

import numpy as np
import pytest

import oracle_py
import workloads
from conftest import GOLDEN


def _rel(a, e, floor=1e-6):
    return np.abs(a - e) / np.maximum(np.abs(e), floor)


# ---------------- scoring pins ----------------

@pytest.mark.parametrize("name", ["kat_single_synth_L1H3.bin", "kat_single_qwen3-8b_L3H5.bin"])
def test_atan2_form_matches_reference_python_golden(oracle, name):
    """triattention_score_ref.c:162-180 criterion: max rel err < 1e-3."""
    d = oracle_py.read_kat_single(os.path.join(GOLDEN, name))
    out = oracle.score_keys_atan2(d["k_re"], d["k_im"], d["qmr"], d["qmi"], d["qam"],
                                  d["omega"], d["key_pos"], d["cur_pos"])
    assert _rel(out, d["expected"]).max() < 1e-3


def test_table_form_matches_reference_python_golden(oracle, synth_stats_path):
    """triattention.c's single-head path vs the Python exporter: the two reference
    formulations differ by fp32 phase rounding (<= 1e-3 abs, score std ~4.6)."""
    d = oracle_py.read_kat_single(os.path.join(GOLDEN, "kat_single_synth_L1H3.bin"))
    st = oracle.load(synth_stats_path)
    try:
        out = oracle.score_single_head(st, 1, 3, d["k_re"], d["k_im"], d["key_pos"], d["cur_pos"])
    finally:
        oracle.free(st)
    assert np.abs(out - d["expected"]).max() < 2e-3


def test_gqa_matches_reference_python_golden(oracle, synth_stats_path):
    """test_tria_gqa.c:35-45 criterion (rel < 1e-2; Python uses the unbiased std)."""
    d = oracle_py.read_kat_gqa(os.path.join(GOLDEN, "kat_gqa_synth_L1KV2.bin"))
    st = oracle.load(synth_stats_path)
    try:
        out = oracle.score_kv_head(st, d["k_re"], d["k_im"], d["key_pos"], d["cur_pos"], 1, 2)
    finally:
        oracle.free(st)
    denom = np.where(np.abs(d["expected"]) > 1e-6, np.abs(d["expected"]), 1.0)
    assert (np.abs(out - d["expected"]) / denom).max() < 1e-2


@pytest.mark.parametrize("name", ["refc_synth_L1KV2_n300.bin", "refc_synth_L0KV1_n512.bin"])
def test_bit_exact_vs_compiled_reference_fixture(oracle, synth_stats_path, name):
    d = oracle_py.read_refc(os.path.join(GOLDEN, name))
    st = oracle.load(synth_stats_path)
    try:
        out = oracle.score_kv_head(st, d["k_re"], d["k_im"], d["key_pos"], d["cur_pos"],
                                   d["layer"], d["kv_head"])
    finally:
        oracle.free(st)
    assert np.array_equal(out.view(np.uint32), d["expected"].view(np.uint32))


def test_bit_exact_vs_live_reference(oracle, reflib, tmp_path):
    """Random geometry (gqa 5, hd 64) through both the oracle and the compiled reference."""
    path = str(tmp_path / "s.tria")
    workloads.write_tria(path, 3, 10, 2, 64, rope_theta=1e7, seed=3,
                         scales=np.array([1.0, 0.5, 1.5], np.float32))
    st, rs = oracle.load(path), reflib.load(path)
    try:
        rng = np.random.default_rng(5)
        for layer, kvh, n, cur in [(0, 0, 1, 1), (2, 1, 257, 100000), (1, 1, 64, 64)]:
            k = workloads.fp32_keys(n, 64, seed=layer + 10 * kvh)[0]
            re, im = workloads.split_halves(k)
            pos = np.sort(rng.choice(cur, size=n, replace=False)).astype(np.int32)
            a = oracle.score_kv_head(st, re, im, pos, cur, layer, kvh)
            b = reflib.score_kv_head(rs, re, im, pos, cur, layer, kvh)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    finally:
        oracle.free(st)
        reflib.free(rs)


def test_reference_kat_tools_pass_on_fixtures():
    """The reference's own C KAT drivers accept the committed fixtures."""
    import subprocess
    ref = os.path.join(oracle_py.HERE, "_ref")
    if not os.path.exists(os.path.join(ref, "test_tria_gqa")):
        pytest.skip("reference tools not built")
    r = subprocess.run([os.path.join(ref, "triattention_score_ref"),
                        os.path.join(GOLDEN, "kat_single_synth_L1H3.bin")], capture_output=True)
    assert r.returncode == 0 and b"PASS" in r.stdout
    r = subprocess.run([os.path.join(ref, "test_tria_gqa"), os.path.join(GOLDEN, "synth_l2h8kv4.tria"),
                        os.path.join(GOLDEN, "kat_gqa_synth_L1KV2.bin"), "1", "2"], capture_output=True)
    assert r.returncode == 0 and b"PASS" in r.stdout


def test_znorm_is_sequential_fp32(oracle):
    """triattention.c:228-238: sequential fp32 sums (not pairwise, not double)."""
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(4097) * 3 + 10).astype(np.float32)
    s = np.float32(0)
    for v in x:
        s = np.float32(s + v)
    mean = np.float32(s / np.float32(x.size))
    var = np.float32(0)
    for v in x:
        d = np.float32(v - mean)
        var = np.float32(var + np.float32(d * d))
    sd = np.float32(np.sqrt(np.float32(var / np.float32(x.size))))
    m2, s2 = oracle.znorm_stats(x)
    assert m2 == mean and s2 == sd


def test_znorm_std_clamp(oracle):
    m, s = oracle.znorm_stats(np.full(10, 2.5, np.float32))
    assert m == np.float32(2.5) and s == np.float32(1e-6)


# ---------------- selection / budget pins ----------------

def _np_select(scores, keep, pos=None, cur_pos=0, window=0, sink=0):
    keys = np.array([_key(x) for x in scores], np.uint64)
    if pos is not None:
        prot = ((sink > 0) & (pos < sink)) | ((window > 0) & (pos >= cur_pos - window))
        keys = np.where(prot, np.uint64(0xFFFFFFFF), keys)
        keep = max(keep, int(prot.sum()))
    keep = min(max(keep, 0), scores.size)
    order = np.lexsort((np.arange(scores.size), -keys.astype(np.int64)))
    return np.sort(order[:keep]).astype(np.int32)


def _key(x):
    x = np.float32(x)
    if np.isnan(x):
        return 0
    if x == 0:
        x = np.float32(0)
    u = int(np.array(x, np.float32).view(np.uint32))
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def test_score_key_order(oracle):
    vals = [-np.inf, -1e30, -1.5, -1e-40, -0.0, 0.0, 1e-40, 1.0, 3e38, np.inf]
    keys = [oracle.score_key(v) for v in vals]
    assert keys == sorted(keys)
    assert oracle.score_key(-0.0) == oracle.score_key(0.0)
    assert oracle.score_key(float("nan")) == 0


@pytest.mark.parametrize("seed", range(6))
def test_select_matches_numpy_lexsort(oracle, seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 3000))
    scores = rng.standard_normal(n).astype(np.float32)
    if seed % 2:   # heavy ties, signed zeros, NaN
        scores = np.round(scores * 2).astype(np.float32) / 2
        scores[rng.integers(0, n, 5)] = -0.0
        scores[rng.integers(0, n, 3)] = np.nan
    keep = int(rng.integers(0, n + 2))
    pos = np.arange(n, dtype=np.int32)
    window = int(rng.integers(0, 50)) if seed >= 3 else 0
    sink = int(rng.integers(0, 10)) if seed >= 3 else 0
    got = oracle.select(scores, keep, pos, n, window, sink)
    exp = _np_select(scores, keep, pos, n, window, sink)
    assert np.array_equal(got, exp)


def test_select_all_equal_keeps_lowest_rows(oracle):
    got = oracle.select(np.zeros(100, np.float32), 7)
    assert np.array_equal(got, np.arange(7))


def test_keep_count_ramp_sequence(oracle):
    """The ramp 10->20->40->80->100% over five steps, 128 rows appended between steps,
    from 65536 rows to a 512-token budget."""
    n, seq = 65536, []
    for pct in (10, 20, 40, 80, 100):
        k = oracle.keep_count(n, 512, pct)
        assert k == workloads.layer_keep(n, 512, pct)
        seq.append(k)
        n = k + 128
    assert seq == [59034, 47432, 28741, 6184, 512]
    assert oracle.keep_count(100, 512, 100) == 100
    assert oracle.keep_count(32768, 3932, 100) == 3932


def test_layer_budget_matches_reference_inline(oracle):
    for scale, base in [(1.0, 3932), (0.9, 512), (1.063, 512), (0.0, 10), (1e-9, 5)]:
        assert oracle.layer_budget(scale, base) == workloads.layer_budget(scale, base)
        assert oracle.layer_budget(scale, base) >= 1


# ---------------- formats / compaction ----------------

def test_half_to_float_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    exp = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib.oracle_half_to_float(int(v)) for v in h[::97]], np.float32)
    e = exp[::97]
    same = (got.view(np.uint32) == e.view(np.uint32)) | (np.isnan(got) & np.isnan(e))
    assert same.all()


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_row_to_split_matches_numpy(oracle, type_id):
    hd = 128
    cache = (workloads.f16_cache(1, 9, 2, hd, seed=1) if type_id == workloads.TYPE_F16
             else workloads.q8_0_cache(1, 9, 2, hd, seed=1))
    rb = workloads.row_bytes(type_id, hd)
    rows = np.ascontiguousarray(cache[0, :, rb:2 * rb])     # head 1
    re_np, im_np = workloads.rows_to_split(type_id, rows, hd)
    for r in range(9):
        re, im = oracle.row_to_split(type_id, np.ascontiguousarray(rows[r]), hd)
        assert np.array_equal(re, re_np[r]) and np.array_equal(im, im_np[r])


def test_compact_rows_stable_gather(oracle):
    rng = np.random.default_rng(0)
    src = rng.integers(0, 255, (50, 40), dtype=np.uint8)
    dst = np.zeros_like(src)
    idx = np.sort(rng.choice(50, 17, replace=False)).astype(np.int32)
    oracle.compact_rows(src, 40, dst, 40, 24, idx)
    assert np.array_equal(dst[:17, :24], src[idx, :24])
    assert not dst[17:].any() and not dst[:, 24:].any()


def test_cpu_step_matches_per_unit_pipeline(oracle, synth_stats_path):
    """Threaded CPU step == dequantise -> score -> select -> compact per unit."""
    st = oracle.load(synth_stats_path)
    try:
        L, KV, hd, n, cur = 2, 4, 128, 96, 96
        rb = workloads.row_bytes(1, hd)
        K = workloads.f16_cache(L, n, KV, hd, seed=2)
        V = workloads.f16_cache(L, n, KV, hd, seed=3)
        Ko, Vo = np.zeros_like(K), np.zeros_like(V)
        pos = np.tile(np.arange(n, dtype=np.int32), (L, KV, 1)).copy()
        pos_o = np.zeros_like(pos)
        units = []
        for l in range(L):
            for h in range(KV):
                units.append(oracle_py.OracleUnit(
                    l, h, n, 20 + l, K[l, :, h * rb:].ctypes.data, V[l, :, h * rb:].ctypes.data,
                    Ko[l, :, h * rb:].ctypes.data, Vo[l, :, h * rb:].ctypes.data,
                    pos[l, h].ctypes.data, pos_o[l, h].ctypes.data, 0))
        assert oracle.cpu_step(oracle.score_fn_ptr, st, 1, hd, KV * rb, units, cur, n_threads=3) == 0
        for u in units:
            l, h = u.layer, u.kv_head
            re, im = workloads.rows_to_split(1, np.ascontiguousarray(K[l, :, h * rb:(h + 1) * rb]), hd)
            sc = oracle.score_kv_head(st, re, im, pos[l, h], cur, l, h)
            idx = oracle.select(sc, 20 + l, pos[l, h], cur)
            assert u.n_kept == idx.size
            assert np.array_equal(Ko[l, :idx.size, h * rb:(h + 1) * rb], K[l, idx, h * rb:(h + 1) * rb])
            assert np.array_equal(Vo[l, :idx.size, h * rb:(h + 1) * rb], V[l, idx, h * rb:(h + 1) * rb])
            assert np.array_equal(pos_o[l, h, :idx.size], pos[l, h, idx])
    finally:
        oracle.free(st)
