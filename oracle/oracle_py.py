"""ctypes binding of the CPU oracle (liboracle.so) and of the compiled reference
(_ref/libtria_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product library.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtria_ref.so")
REF_SRC = os.environ.get("TRIA_REF_SRC", "")      # the reference source tree, when it is present

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build(ref: bool = True, ref_src: str = "") -> None:
    """Compile liboracle.so, and _ref/ when the reference sources are given
    (ref_src, else the environment variable TRIA_REF_SRC) and present."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    src = ref_src or REF_SRC
    if ref and src and os.path.exists(os.path.join(src, "triattention.c")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={src}"], check=True)
        if os.path.exists(os.path.join(os.path.dirname(HERE), "triattention-ggml_b200", "libtriattention_b200.so")):
            subprocess.run(["make", "-s", "-C", HERE, "dropin", f"REF={src}"], check=True)


def dropin_tool(name: str) -> str:
    """Path of a reference C driver (test_tria_gqa, test_tria_lib, bench_tria)
    compiled unmodified against the product header and library."""
    return os.path.join(HERE, "_ref", "dropin_" + name)


def ref_tool(name: str) -> str:
    """Path of a reference C driver compiled against the reference itself."""
    return os.path.join(HERE, "_ref", name)


class OracleUnit(C.Structure):
    _fields_ = [("layer", C.c_int32), ("kv_head", C.c_int32), ("n", C.c_int32),
                ("keep", C.c_int32), ("k_src", C.c_void_p), ("v_src", C.c_void_p),
                ("k_dst", C.c_void_p), ("v_dst", C.c_void_p), ("pos_src", C.c_void_p),
                ("pos_dst", C.c_void_p), ("n_kept", C.c_int32)]


SCORE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                       C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        L = self.lib = C.CDLL(path)
        L.oracle_load.restype = C.c_void_p
        L.oracle_load.argtypes = [C.c_char_p]
        L.oracle_free.argtypes = [C.c_void_p]
        L.oracle_score_kv_head.argtypes = [C.c_void_p, _f32p, _f32p, _i32p, C.c_int, C.c_int,
                                           C.c_int, C.c_int, _f32p]
        L.oracle_score_single_head.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p, _i32p,
                                               C.c_int, C.c_int, _f32p]
        L.oracle_znorm_stats.argtypes = [_f32p, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_float)]
        L.oracle_score_keys_atan2.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i32p,
                                              C.c_int, C.c_int, C.c_int, _f32p]
        L.oracle_score_key.restype = C.c_uint32
        L.oracle_score_key.argtypes = [C.c_float]
        L.oracle_keep_count.argtypes = [C.c_int, C.c_int, C.c_int]
        L.oracle_layer_budget.argtypes = [C.c_float, C.c_int]
        L.oracle_select.argtypes = [_f32p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _i32p]
        L.oracle_count_protected.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.oracle_compact_rows.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int,
                                          _i32p, C.c_int]
        L.oracle_row_to_split.argtypes = [C.c_int, C.c_void_p, C.c_int, _f32p, _f32p]
        L.oracle_half_to_float.restype = C.c_float
        L.oracle_half_to_float.argtypes = [C.c_uint16]
        L.oracle_cpu_step.argtypes = [SCORE_FN, C.c_void_p, C.c_int, C.c_int, C.c_int64,
                                      C.POINTER(OracleUnit), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        self.score_fn_ptr = C.cast(L.oracle_score_kv_head, C.c_void_p).value

    # --- stats ---
    def load(self, path: str) -> int:
        return self.lib.oracle_load(path.encode()) or 0

    def free(self, st: int) -> None:
        self.lib.oracle_free(st)

    # --- scoring ---
    def score_kv_head(self, st, k_re, k_im, key_pos, cur_pos, layer, kv_head):
        n = int(key_pos.shape[0])
        out = np.zeros(max(n, 1), np.float32)
        self.lib.oracle_score_kv_head(st, _c(k_re), _c(k_im), _ci(key_pos), cur_pos, n,
                                      layer, kv_head, out)
        return out[:n]

    def score_single_head(self, st, layer, q_head, k_re, k_im, key_pos, cur_pos):
        n = int(key_pos.shape[0])
        out = np.zeros(max(n, 1), np.float32)
        self.lib.oracle_score_single_head(st, layer, q_head, _c(k_re), _c(k_im), _ci(key_pos),
                                          cur_pos, n, out)
        return out[:n]

    def znorm_stats(self, raw):
        m, s = C.c_float(), C.c_float()
        self.lib.oracle_znorm_stats(_c(raw), int(raw.shape[0]), C.byref(m), C.byref(s))
        return np.float32(m.value), np.float32(s.value)

    def score_keys_atan2(self, k_re, k_im, qmr, qmi, qam, omega, key_pos, cur_pos):
        n, fc = k_re.shape
        out = np.zeros(n, np.float32)
        self.lib.oracle_score_keys_atan2(_c(k_re), _c(k_im), _c(qmr), _c(qmi), _c(qam), _c(omega),
                                         _ci(key_pos), cur_pos, fc, n, out)
        return out

    # --- selection ---
    def score_key(self, x: float) -> int:
        return int(self.lib.oracle_score_key(x))

    def keep_count(self, n, layer_budget, ramp_pct):
        return int(self.lib.oracle_keep_count(n, layer_budget, ramp_pct))

    def layer_budget(self, scale, base):
        return int(self.lib.oracle_layer_budget(scale, base))

    def count_protected(self, pos, cur_pos, window, sink):
        return int(self.lib.oracle_count_protected(_ci(pos), int(pos.shape[0]), cur_pos, window, sink))

    def select(self, scores, keep, pos=None, cur_pos=0, window=0, sink=0):
        n = int(scores.shape[0])
        idx = np.zeros(max(n, 1), np.int32)
        pp = None
        if pos is not None:
            pos = _ci(pos)
            pp = pos.ctypes.data
        k = self.lib.oracle_select(_c(scores), pp, n, keep, cur_pos, window, sink, idx)
        return idx[:k].copy()

    # --- compaction / formats ---
    def compact_rows(self, src, src_stride, dst, dst_stride, row_bytes, kept_idx):
        self.lib.oracle_compact_rows(src.ctypes.data, src_stride, dst.ctypes.data, dst_stride,
                                     row_bytes, _ci(kept_idx), int(kept_idx.shape[0]))

    def row_to_split(self, type_id, row, head_dim):
        fc = head_dim // 2
        re, im = np.zeros(fc, np.float32), np.zeros(fc, np.float32)
        rc = self.lib.oracle_row_to_split(type_id, row.ctypes.data, head_dim, re, im)
        assert rc == 0
        return re, im

    def cpu_step(self, score_fn_ptr, st, type_id, head_dim, row_stride, units, cur_pos,
                 window=0, sink=0, n_threads=1):
        arr = (OracleUnit * len(units))(*units)
        rc = self.lib.oracle_cpu_step(SCORE_FN(score_fn_ptr), st, type_id, head_dim, row_stride,
                                      arr, len(units), cur_pos, window, sink, n_threads)
        for i, u in enumerate(units):
            u.n_kept = arr[i].n_kept
        return rc


class RefLib:
    """The reference's own triattention.c, compiled unmodified into _ref/."""

    def __init__(self, path: str = REF_SO):
        L = self.lib = C.CDLL(path)
        L.tria_load.restype = C.c_void_p
        L.tria_load.argtypes = [C.c_char_p]
        L.tria_free.argtypes = [C.c_void_p]
        L.tria_score_kv_head.argtypes = [C.c_void_p, _f32p, _f32p, _i32p, C.c_int, C.c_int,
                                         C.c_int, C.c_int, _f32p]
        L.score_keys.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i32p,
                                 C.c_int, C.c_int, C.c_int, _f32p]
        self.score_fn_ptr = C.cast(L.tria_score_kv_head, C.c_void_p).value

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def load(self, path: str) -> int:
        return self.lib.tria_load(path.encode()) or 0

    def free(self, st: int) -> None:
        self.lib.tria_free(st)

    def score_kv_head(self, st, k_re, k_im, key_pos, cur_pos, layer, kv_head):
        n = int(key_pos.shape[0])
        out = np.zeros(max(n, 1), np.float32)
        self.lib.tria_score_kv_head(st, _c(k_re), _c(k_im), _ci(key_pos), cur_pos, n,
                                    layer, kv_head, out)
        return out[:n]

    def score_keys(self, k_re, k_im, qmr, qmi, qam, omega, key_pos, cur_pos):
        n, fc = k_re.shape
        out = np.zeros(n, np.float32)
        self.lib.score_keys(_c(k_re), _c(k_im), _c(qmr), _c(qmi), _c(qam), _c(omega),
                            _ci(key_pos), cur_pos, fc, n, out)
        return out


def _c(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ci(a):
    return np.ascontiguousarray(a, dtype=np.int32)


# --- golden fixture readers (formats of the reference's exporters) ---

def read_kat_single(path):
    """triattention_export_test.py format (triattention_score_ref.c:108-121)."""
    b = open(path, "rb").read()
    fc, n, cur = np.frombuffer(b[:12], "<i4")
    off = 12
    def take(cnt, dt):
        nonlocal off
        a = np.frombuffer(b[off:off + 4 * cnt], dt).copy()
        off += 4 * cnt
        return a
    qmr, qmi, qam, omega = (take(fc, "<f4") for _ in range(4))
    key_pos = take(n, "<i4")
    k_re = take(n * fc, "<f4").reshape(n, fc)
    k_im = take(n * fc, "<f4").reshape(n, fc)
    expected = take(n, "<f4")
    return dict(fc=int(fc), n=int(n), cur_pos=int(cur), qmr=qmr, qmi=qmi, qam=qam, omega=omega,
                key_pos=key_pos.astype(np.int32), k_re=k_re, k_im=k_im, expected=expected)


def read_kat_gqa(path):
    """triattention_export_test_gqa.py format (test_tria_gqa.c:17-30)."""
    b = open(path, "rb").read()
    fc, n, cur, gqa = np.frombuffer(b[:16], "<i4")
    off = 16
    key_pos = np.frombuffer(b[off:off + 4 * n], "<i4").astype(np.int32); off += 4 * n
    k_re = np.frombuffer(b[off:off + 4 * n * fc], "<f4").reshape(n, fc).copy(); off += 4 * n * fc
    k_im = np.frombuffer(b[off:off + 4 * n * fc], "<f4").reshape(n, fc).copy(); off += 4 * n * fc
    expected = np.frombuffer(b[off:off + 4 * n], "<f4").copy()
    return dict(fc=int(fc), n=int(n), cur_pos=int(cur), gqa=int(gqa), key_pos=key_pos,
                k_re=k_re, k_im=k_im, expected=expected)


def read_refc(path):
    """make_golden.py's record of the compiled reference C tria_score_kv_head."""
    b = open(path, "rb").read()
    fc, n, cur, layer, kvh = (int(x) for x in np.frombuffer(b[:20], "<i4"))
    off = 20
    key_pos = np.frombuffer(b[off:off + 4 * n], "<i4").astype(np.int32); off += 4 * n
    k_re = np.frombuffer(b[off:off + 4 * n * fc], "<f4").reshape(n, fc).copy(); off += 4 * n * fc
    k_im = np.frombuffer(b[off:off + 4 * n * fc], "<f4").reshape(n, fc).copy(); off += 4 * n * fc
    expected = np.frombuffer(b[off:off + 4 * n], "<f4").copy()
    return dict(fc=fc, n=n, cur_pos=cur, layer=layer, kv_head=kvh, key_pos=key_pos,
                k_re=k_re, k_im=k_im, expected=expected)


# ---------------- global budget (multi-sequence) rule ----------------

def score_keys(x):
    """Order-preserving uint32 keys of fp32 scores, NaN lowest and -0 == +0
    (the key oracle_score_key computes one value at a time)."""
    x = np.asarray(x, np.float32).copy()
    x[x == 0] = 0.0
    u = x.view(np.uint32)
    k = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    k[np.isnan(x)] = 0
    return k


def global_select(keys_by_unit, k):
    """The global-budget rule: keys_by_unit lists one uint32 key array per unit
    in (layer, kv-head) order; returns per unit the kept row indices
    (ascending) of the top k rows by (key desc, unit asc, row asc)."""
    if not keys_by_unit:
        return []
    allk = np.concatenate([np.asarray(x, np.uint32) for x in keys_by_unit])
    unit = np.concatenate([np.full(len(x), i, np.int64) for i, x in enumerate(keys_by_unit)])
    row = np.concatenate([np.arange(len(x), dtype=np.int64) for x in keys_by_unit])
    order = np.lexsort((row, unit, -allk.astype(np.int64)))
    top = order[:max(0, min(k, allk.size))]
    return [np.sort(row[top][unit[top] == i]) for i in range(len(keys_by_unit))]
