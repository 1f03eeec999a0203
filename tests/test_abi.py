"""CPU tests of the C ABI: the product library loads, exports every symbol the
header declares, loads TRIA files exactly like the reference (and rejects
malformed ones), and fails loudly (no CPU fallback) where no GPU exists."""
import ctypes as C
import os
import struct

import numpy as np
import pytest

import tria_b200
import workloads
from conftest import GOLDEN


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(tria_b200.LIB_PATH):
        tria_b200.build()
    return tria_b200.lib()


def test_exports_every_header_symbol(L):
    names = tria_b200.exported_symbols_in_header()
    assert {"tria_load", "tria_free", "tria_score_kv_head", "tria_ctx_create", "tria_evict",
            "tria_score", "tria_select", "tria_compact", "tria_get_n_kv"} <= set(names)
    for n in names:
        assert hasattr(L, n), n


def test_checked_build_exports_the_same_symbols(L):
    """The checked build (make checked) is the same ABI with bounds checks in
    its kernels; it says so through tria_checked_build, the product does not."""
    if not os.path.exists(tria_b200.CHECKED_LIB_PATH):
        tria_b200.build()
    CL = C.CDLL(tria_b200.CHECKED_LIB_PATH)
    for n in tria_b200.exported_symbols_in_header():
        assert hasattr(CL, n), n
    assert CL.tria_checked_build() == 1
    assert L.tria_checked_build() == (1 if tria_b200.LIB_PATH == tria_b200.CHECKED_LIB_PATH else 0)


def test_no_oracle_or_reference_symbols_in_product(L):
    """The product never links the checker."""
    for n in ("oracle_score_kv_head", "oracle_select", "score_keys", "tria_score_ref_main"):
        with pytest.raises(AttributeError):
            getattr(L, n)


def _fields(st):
    s = st.contents
    fc = s.freq_count
    out = dict(L=s.num_layers, H=s.num_heads, KV=s.num_kv_heads, hd=s.head_dim, fc=fc,
               theta=s.rope_theta, ascale=s.attn_scale,
               scales=np.ctypeslib.as_array(s.layer_budget_scales, (s.num_layers,)).copy(),
               omega=np.ctypeslib.as_array(s.omega, (fc,)).copy())
    heads = []
    for h in range(s.num_layers * s.num_heads):
        hs = s.heads[h]
        heads.append(np.stack([np.ctypeslib.as_array(getattr(hs, f), (fc,)).copy()
                               for f in ("q_mean_real", "q_mean_imag", "q_abs_mean", "qma")]))
    out["heads"] = np.stack(heads)
    return out


def test_load_matches_reference_loader(L, reflib, synth_stats_path):
    st = tria_b200.load(synth_stats_path)
    rs = reflib.load(synth_stats_path)
    assert st and rs
    try:
        a = _fields(st)
        b = _fields(C.cast(C.c_void_p(rs), C.POINTER(tria_b200.Stats)))
        for k in a:
            if isinstance(a[k], np.ndarray):
                assert np.array_equal(a[k].view(np.uint32) if a[k].dtype == np.float32 else a[k],
                                      b[k].view(np.uint32) if b[k].dtype == np.float32 else b[k]), k
            else:
                assert a[k] == b[k], k
    finally:
        tria_b200.free(st)
        reflib.free(rs)


def test_load_v1_defaults_scales(tmp_path):
    p = str(tmp_path / "v1.tria")
    workloads.write_tria(p, 3, 4, 2, 32, version=1, seed=1)
    st = tria_b200.load(p)
    assert st
    try:
        f = _fields(st)
        assert f["L"] == 3 and np.all(f["scales"] == 1.0)
    finally:
        tria_b200.free(st)


def _corrupt(tmp_path, name, mutate):
    src = open(os.path.join(GOLDEN, "synth_l2h8kv4.tria"), "rb").read()
    p = str(tmp_path / name)
    open(p, "wb").write(mutate(bytearray(src)))
    return p


@pytest.mark.parametrize("name,mutate", [
    ("magic", lambda b: b"XXXX" + b[4:]),
    ("version", lambda b: b[:4] + struct.pack("<I", 3) + b[8:]),
    ("truncated", lambda b: b[:-1]),
    ("overlong", lambda b: b + b"\0"),
    ("header_only", lambda b: b[:64]),
    ("short_header", lambda b: b[:20]),
    ("fc_mismatch", lambda b: b[:24] + struct.pack("<I", 63) + b[28:]),
    ("gqa_mismatch", lambda b: b[:16] + struct.pack("<I", 3) + b[20:]),
    ("zero_layers", lambda b: b[:8] + struct.pack("<I", 0) + b[12:]),
])
def test_load_rejects_malformed(tmp_path, name, mutate):
    assert tria_b200.load(_corrupt(tmp_path, name, mutate)) is None
    assert tria_b200.last_error().startswith("tria_load")


def test_load_missing_file(tmp_path):
    assert tria_b200.load(str(tmp_path / "nope.bin")) is None


def test_free_null_is_safe(L):
    L.tria_free(None)


def test_layer_budget_inline(synth_stats_path):
    st = tria_b200.load(synth_stats_path)
    try:
        assert tria_b200.layer_budget(st, 0, 512) == workloads.layer_budget(0.9, 512) == 460
        assert tria_b200.layer_budget(st, 1, 3932) == workloads.layer_budget(1.1, 3932)
    finally:
        tria_b200.free(st)


def test_status_strings(L):
    for s in range(-6, 1):
        assert L.tria_status_str(s)


def test_no_gpu_fails_loudly(synth_stats_path):
    """Without a GPU the device path reports an error; the reference-signature
    call writes NaN instead of silently computing on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    st = tria_b200.load(synth_stats_path)
    try:
        with pytest.raises(tria_b200.TriaError) as ei:
            tria_b200.Context(st, 0)
        assert ei.value.status == tria_b200.ERR_NO_DEVICE
        d = workloads.fp32_keys(16, 128, seed=0)[0]
        re, im = workloads.split_halves(d)
        out = tria_b200.score_kv_head(st, re, im, np.arange(16, dtype=np.int32), 16, 0, 0)
        assert np.isnan(out).all()
    finally:
        tria_b200.free(st)


def test_select_noalloc_rejects_bad_sizes_on_the_host(L):
    """Argument checks of tria_select_noalloc run before any CUDA call (no
    device needed, nothing launched): a negative or over-int32 position
    stride and a unit count above TRIA_NOALLOC_MAX_UNITS are refused."""
    units, n = 4, 100
    nr = np.full(units, n, np.int32)
    keep = np.full(units, 10, np.int32)
    fake = 256                                   # never dereferenced: the checks fail first
    for stride in (-1, 1 << 31):
        r = L.tria_select_noalloc(fake, n, nr.ctypes.data, keep.ctypes.data, units, fake, stride, n, 8, 0,
                                  fake, n, fake, None)
        assert r == tria_b200.ERR_INVALID, stride
        assert "pos_stride" in tria_b200.last_error()
    big = 2049
    nr2 = np.full(big, 1, np.int32)
    keep2 = np.ones(big, np.int32)
    r = L.tria_select_noalloc(fake, 1, nr2.ctypes.data, keep2.ctypes.data, big, None, 0, 1, 0, 0,
                              fake, 1, fake, None)
    assert r == tria_b200.ERR_INVALID and "units" in tria_b200.last_error()
