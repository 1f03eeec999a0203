"""ctypes binding of libtriattention_b200.so (include/triattention.h).

The reference's Python side reimplements the scoring math in torch
(triattention_common.py); this module instead calls the C ABI, so the
Python validate/score scripts can drive the B200 kernels directly:

    st = tria_b200.load("stats.bin")                  # tria_load
    out = tria_b200.score_kv_head(st, k_re, k_im, key_pos, cur_pos, layer, kvh)
    ctx = tria_b200.Context(st, device=0)             # device path
    ctx.evict(src_view, dst_view, n_rows, params, stream)

There is no CPU fallback: if the shared library is missing this module
raises on import of the library, and every device call reports the CUDA
status it got.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
CHECKED_LIB_PATH = os.path.join(HERE, "libtriattention_b200_checked.so")
# TRIA_B200_LIB=checked loads the checked build (bounds checks in every kernel,
# TRIA_ERR_BOUNDS) instead of the product library
LIB_PATH = CHECKED_LIB_PATH if os.environ.get("TRIA_B200_LIB") == "checked" else \
    os.path.join(HERE, "libtriattention_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "triattention.h")
HEADERS = [HEADER, os.path.join(os.path.dirname(HERE), "include", "triattention_ggml.h")]

TYPE_F16 = 1
TYPE_Q8_0 = 8

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_NOMEM = -3
ERR_POSITION = -4
ERR_UNSUPPORTED = -5
ERR_NO_DEVICE = -6
ERR_TIMEOUT = -7
ERR_BOUNDS = -8


class TriaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


class HeadStats(C.Structure):
    _fields_ = [("q_mean_real", C.POINTER(C.c_float)), ("q_mean_imag", C.POINTER(C.c_float)),
                ("q_abs_mean", C.POINTER(C.c_float)), ("qma", C.POINTER(C.c_float))]


class Stats(C.Structure):
    """struct tria_stats (triattention.h:38-50 of the reference)."""
    _fields_ = [("num_layers", C.c_uint32), ("num_heads", C.c_uint32), ("num_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("freq_count", C.c_uint32), ("rope_theta", C.c_float),
                ("attn_scale", C.c_float), ("layer_budget_scales", C.POINTER(C.c_float)),
                ("omega", C.POINTER(C.c_float)), ("heads", C.POINTER(HeadStats))]


class KvView(C.Structure):
    """struct tria_kv_view."""
    _fields_ = [("type", C.c_int32), ("n_layer", C.c_int32), ("layer0", C.c_int32),
                ("n_head_kv", C.c_int32), ("head0", C.c_int32), ("n_cells", C.c_int32),
                ("cell_stride", C.c_int64), ("head_stride", C.c_int64),
                ("k", C.POINTER(C.c_void_p)), ("v", C.POINTER(C.c_void_p)),
                ("pos", C.c_void_p), ("pos_shared", C.c_int32), ("flags", C.c_int32)]


VIEW_POST_ROPE = 1      # TRIA_VIEW_POST_ROPE


class GgmlTensor(C.Structure):
    """struct tria_ggml_tensor: the ggml_tensor fields the bridge reads."""
    _fields_ = [("type", C.c_int32), ("reserved", C.c_int32), ("ne", C.c_int64 * 4),
                ("nb", C.c_size_t * 4), ("data", C.c_void_p)]


class GgmlCache(C.Structure):
    """struct tria_ggml_cache."""
    _fields_ = [("k", C.POINTER(C.POINTER(GgmlTensor))), ("v", C.POINTER(C.POINTER(GgmlTensor))),
                ("n_layer", C.c_int32), ("layer0", C.c_int32), ("n_head_kv", C.c_int32),
                ("head_dim", C.c_int32), ("pos", C.c_void_p), ("pos_shared", C.c_int32),
                ("flags", C.c_int32)]


def ggml_tensor(type_id, ne0, ne1, nb1, data, elem=None):
    """A 2-D ggml tensor descriptor [ne0, ne1] with rows nb1 bytes apart."""
    t = GgmlTensor()
    t.type = int(type_id)
    t.ne[:] = [int(ne0), int(ne1), 1, 1]
    e = elem if elem is not None else (2 if type_id == TYPE_F16 else 34)
    t.nb[:] = [e, int(nb1), int(nb1) * int(ne1), int(nb1) * int(ne1)]
    t.data = _ptr(data)
    return t


def ggml_cache(k_tensors, v_tensors, n_head_kv, head_dim, pos, layer0=0, pos_shared=False, flags=0):
    """A GgmlCache over lists of GgmlTensor; keeps its arrays alive."""
    nl = len(k_tensors)
    karr = (C.POINTER(GgmlTensor) * nl)(*[C.pointer(t) for t in k_tensors])
    varr = (C.POINTER(GgmlTensor) * nl)(*[C.pointer(t) for t in v_tensors]) if v_tensors is not None else None
    c = GgmlCache(C.cast(karr, C.POINTER(C.POINTER(GgmlTensor))),
                  C.cast(varr, C.POINTER(C.POINTER(GgmlTensor))) if varr is not None else None,
                  nl, int(layer0), int(n_head_kv), int(head_dim), _ptr(pos), 1 if pos_shared else 0, int(flags))
    c._keep = (karr, varr, k_tensors, v_tensors, pos)
    return c


def ggml_view(cache):
    """tria_ggml_view: (status, KvView) without raising."""
    nl = cache.n_layer
    kp, vp = (C.c_void_p * nl)(), (C.c_void_p * nl)()
    v = KvView()
    r = lib().tria_ggml_view(C.byref(cache), C.byref(v), kp, vp)
    v._keep = (kp, vp, cache)
    return r, v


class EvictParams(C.Structure):
    """struct tria_evict_params."""
    _fields_ = [("cur_pos", C.c_int32), ("budget", C.c_int32), ("ramp_pct", C.c_int32),
                ("window", C.c_int32), ("sink", C.c_int32), ("reserved", C.c_int32)]


class Policy(C.Structure):
    """struct tria_policy: the reference runtime's eviction schedule."""
    _fields_ = [("budget_pct", C.c_int32), ("window", C.c_int32), ("interval", C.c_int32),
                ("sink", C.c_int32), ("step", C.c_int32), ("next_pos", C.c_int32)]

    def __init__(self, budget_pct=75, window=512, interval=128, sink=0):
        super().__init__()
        lib().tria_policy_init(C.byref(self), int(budget_pct), int(window), int(interval), int(sink))

    def due(self, n_past: int, n_kv: int):
        """EvictParams when an eviction is due at n_past with n_kv cached rows, else None."""
        out = EvictParams()
        r = lib().tria_policy_due(C.byref(self), int(n_past), int(n_kv), C.byref(out))
        if r < 0:
            check(r)
        return out if r == 1 else None


def n_kv_per_seq(n_kept, seq_of_unit, n_seq):
    """tria_n_kv_per_seq: per-sequence maximum of the kept counts."""
    nk = np.ascontiguousarray(n_kept, np.int32)
    so = np.ascontiguousarray(seq_of_unit, np.int32)
    out = np.zeros(n_seq, np.int32)
    check(lib().tria_n_kv_per_seq(nk.ctypes.data, so.ctypes.data, int(nk.shape[0]), int(n_seq), out.ctypes.data))
    return out


def build() -> str:
    """Compile the library (and the checked build) in-tree (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-j4", "-C", HERE, "all", "checked"], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `make -C {HERE}`")
        L = C.CDLL(LIB_PATH)
        L.tria_load.restype = C.POINTER(Stats)
        L.tria_load.argtypes = [C.c_char_p]
        L.tria_free.argtypes = [C.POINTER(Stats)]
        L.tria_score_kv_head.argtypes = [C.POINTER(Stats), C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.tria_status_str.restype = C.c_char_p
        L.tria_status_str.argtypes = [C.c_int]
        L.tria_last_error.restype = C.c_char_p
        L.tria_ctx_create.argtypes = [C.POINTER(Stats), C.c_int, C.POINTER(C.c_void_p)]
        L.tria_ctx_destroy.argtypes = [C.c_void_p]
        L.tria_score.argtypes = [C.c_void_p, C.POINTER(KvView), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
        L.tria_select.argtypes = [C.c_void_p, C.POINTER(KvView), C.c_void_p, C.c_void_p,
                                  C.POINTER(EvictParams), C.c_void_p, C.c_void_p, C.c_void_p]
        L.tria_compact.argtypes = [C.c_void_p, C.POINTER(KvView), C.POINTER(KvView), C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p]
        L.tria_evict.argtypes = [C.c_void_p, C.POINTER(KvView), C.POINTER(KvView), C.c_void_p,
                                 C.POINTER(EvictParams), C.c_void_p, C.c_void_p]
        L.tria_get_n_kv.argtypes = [C.c_void_p, C.c_void_p, C.c_int32]
        L.tria_evict_host.argtypes = [C.c_void_p, C.POINTER(KvView), C.POINTER(KvView), C.c_void_p,
                                      C.POINTER(EvictParams), C.c_void_p]
        L.tria_ctx_set_timing.argtypes = [C.c_void_p, C.c_int]
        L.tria_ctx_stage_ms.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.tria_ctx_launches.restype = C.c_int64
        L.tria_ctx_launches.argtypes = [C.c_void_p]
        L.tria_ctx_check.argtypes = [C.c_void_p, C.c_void_p]
        L.tria_ggml_view.argtypes = [C.POINTER(GgmlCache), C.POINTER(KvView), C.c_void_p, C.c_void_p]
        L.tria_ggml_evict.argtypes = [C.c_void_p, C.POINTER(GgmlCache), C.POINTER(GgmlCache), C.c_void_p,
                                      C.POINTER(EvictParams), C.c_void_p]
        L.tria_ctx_set_wait_limit.argtypes = [C.c_void_p, C.c_int64]
        L.tria_ctx_set_select_split.argtypes = [C.c_void_p, C.c_int32]
        L.tria_key_gather.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_uint32,
                                      C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
        L.tria_checked_build.argtypes = []
        L.tria_select_noalloc.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int32,
                                          C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                          C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
        L.tria_znorm_stats.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]
        L.tria_policy_init.restype = None
        L.tria_policy_init.argtypes = [C.POINTER(Policy), C.c_int32, C.c_int32, C.c_int32, C.c_int32]
        L.tria_policy_due.argtypes = [C.POINTER(Policy), C.c_int32, C.c_int32, C.POINTER(EvictParams)]
        L.tria_n_kv_per_seq.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]
        L.tria_score_key.restype = C.c_uint32
        L.tria_score_key.argtypes = [C.c_float]
        L.tria_key_histogram.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_uint32,
                                         C.c_void_p, C.c_void_p]
        L.tria_key_count.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_uint32, C.c_void_p,
                                     C.c_void_p]
        L.tria_select_key.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_uint32, C.c_void_p,
                                      C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]
        L.tria_score_kv_head_dev.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                             C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]
        _lib = L
    return _lib


def exported_symbols_in_header(paths=None):
    """Names of every function the public headers declare with TRIA_API."""
    names = set()
    for path in paths or HEADERS:
        txt = open(path).read()
        names |= set(re.findall(r"TRIA_API\s+[^;(]*?\b(tria_\w+)\s*\(", txt))
    return sorted(names)


def last_error() -> str:
    return lib().tria_last_error().decode()


def check(status: int) -> None:
    if status != OK:
        raise TriaError(status, f"{lib().tria_status_str(status).decode()}: {last_error()}")


# ---------------- reference API ----------------

def load(path: str):
    """tria_load: returns a ctypes pointer to Stats (falsy on failure)."""
    p = lib().tria_load(os.fsencode(path))
    return p if p else None


def free(stats) -> None:
    if stats:
        lib().tria_free(stats)


def score_kv_head(stats, k_re, k_im, key_pos, cur_pos, layer, kv_head):
    """tria_score_kv_head on host arrays (fp32 [n, fc] halves, int32 positions)."""
    k_re = np.ascontiguousarray(k_re, np.float32)
    k_im = np.ascontiguousarray(k_im, np.float32)
    key_pos = np.ascontiguousarray(key_pos, np.int32)
    n = int(key_pos.shape[0])
    out = np.empty(max(n, 1), np.float32)
    lib().tria_score_kv_head(stats, k_re.ctypes.data, k_im.ctypes.data, key_pos.ctypes.data,
                             int(cur_pos), n, int(layer), int(kv_head), out.ctypes.data)
    return out[:n]


def layer_budget(stats, layer, base_budget):
    """tria_layer_budget (the header's static inline, restated for Python)."""
    scale = np.float32(stats.contents.layer_budget_scales[layer])
    b = int(np.float32(np.float32(base_budget) * scale))
    return b if b > 0 else 1


# ---------------- device path ----------------

NOALLOC_MAX_KEYS = 1 << 20


def znorm_stats(x, stride, n, mean_std, stream=None):
    """tria_znorm_stats: exact (mean, std) of each row of device array x."""
    nn = np.ascontiguousarray(n, np.int32)
    check(lib().tria_znorm_stats(_ptr(x), int(stride), nn.ctypes.data, int(nn.shape[0]),
                                 _ptr(mean_std), _stream(stream)))


def checked_build() -> bool:
    """tria_checked_build: True when the loaded library is the checked build."""
    return bool(lib().tria_checked_build())


def score_key(x: float) -> int:
    """tria_score_key: the order-preserving 32-bit key of a score."""
    return int(lib().tria_score_key(float(x)))


def key_histogram(scores, score_stride, n_rows, level, prefix, hist, stream=None):
    """tria_key_histogram: add the 16-bit bins of the keys of device `scores`
    ([units][score_stride]) to device `hist` [65536] uint32."""
    nr = np.ascontiguousarray(n_rows, np.int32)
    check(lib().tria_key_histogram(_ptr(scores), int(score_stride), nr.ctypes.data, int(nr.shape[0]),
                                   int(level), int(prefix), _ptr(hist), _stream(stream)))


def key_gather(scores, score_stride, n_rows, key_min, out, cap, count, stream=None):
    """tria_key_gather: scores of the units' rows with key >= key_min into
    device `out` [cap]; device `count` [1] int32 gets how many there were."""
    nr = np.ascontiguousarray(n_rows, np.int32)
    check(lib().tria_key_gather(_ptr(scores), int(score_stride), nr.ctypes.data, int(nr.shape[0]),
                                int(key_min), _ptr(out), int(cap), _ptr(count), _stream(stream)))


def key_count(scores, score_stride, n_rows, key, counts, stream=None):
    """tria_key_count: per-unit counts of rows whose key equals `key`."""
    nr = np.ascontiguousarray(n_rows, np.int32)
    check(lib().tria_key_count(_ptr(scores), int(score_stride), nr.ctypes.data, int(nr.shape[0]),
                               int(key), _ptr(counts), _stream(stream)))


def select_key(scores, score_stride, n_rows, key, counts, tie_allow, kept_idx, kept_stride, n_kept, stream=None):
    """tria_select_key: keep rows with key > `key` and the first `tie_allow`
    rows equal to it (unit order), kept indices ascending per unit."""
    nr = np.ascontiguousarray(n_rows, np.int32)
    check(lib().tria_select_key(_ptr(scores), int(score_stride), nr.ctypes.data, int(nr.shape[0]), int(key),
                                _ptr(counts), int(tie_allow), _ptr(kept_idx), int(kept_stride), _ptr(n_kept),
                                _stream(stream)))


def select_noalloc(scores, score_stride, n_rows, keep, kept_idx, kept_stride, n_kept,
                   pos=None, pos_stride=0, cur_pos=0, window=0, sink=0, stream=None):
    """tria_select_noalloc: rank device scores with no allocation (fixed static
    scratch of NOALLOC_MAX_KEYS keys; see the header)."""
    nr = np.ascontiguousarray(n_rows, np.int32)
    kp = np.ascontiguousarray(keep, np.int32)
    assert nr.shape == kp.shape
    check(lib().tria_select_noalloc(_ptr(scores), int(score_stride), nr.ctypes.data, kp.ctypes.data,
                                    int(nr.shape[0]), _ptr(pos), int(pos_stride), int(cur_pos),
                                    int(window), int(sink), _ptr(kept_idx), int(kept_stride),
                                    _ptr(n_kept), _stream(stream)))

def _ptr(x) -> int:
    """Device pointer of a torch tensor or an int."""
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def make_view(type_id, k_layers, v_layers, pos, n_cells, cell_stride, head_stride,
              n_head_kv, layer0=0, head0=0, pos_shared=False, flags=0):
    """Build a KvView; k_layers / v_layers are lists of torch tensors or device pointers.
    The returned view keeps its pointer arrays alive."""
    nl = len(k_layers)
    karr = (C.c_void_p * nl)(*[_ptr(t) for t in k_layers])
    varr = (C.c_void_p * nl)(*[_ptr(t) for t in v_layers]) if v_layers is not None else None
    v = KvView(type_id, nl, layer0, n_head_kv, head0, n_cells, cell_stride, head_stride,
               C.cast(karr, C.POINTER(C.c_void_p)),
               C.cast(varr, C.POINTER(C.c_void_p)) if varr is not None else None,
               _ptr(pos), 1 if pos_shared else 0, int(flags))
    v._keep = (karr, varr, k_layers, v_layers, pos)
    return v


class Context:
    def __init__(self, stats, device: int = 0):
        h = C.c_void_p()
        check(lib().tria_ctx_create(stats, device, C.byref(h)))
        self.h = h
        self.stats = stats

    def close(self):
        if self.h:
            lib().tria_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _rows(n_rows):
        a = np.ascontiguousarray(n_rows, np.int32)
        return a, a.ctypes.data

    def score(self, view, n_rows, cur_pos, scores, stream=None):
        a, p = self._rows(n_rows)
        check(lib().tria_score(self.h, C.byref(view), p, int(cur_pos), _ptr(scores), _stream(stream)))

    def select(self, view, n_rows, scores, params, kept_idx, n_kept, stream=None):
        a, p = self._rows(n_rows)
        check(lib().tria_select(self.h, C.byref(view), p, _ptr(scores), C.byref(params),
                                _ptr(kept_idx), _ptr(n_kept), _stream(stream)))

    def compact(self, src, dst, n_rows, kept_idx, n_kept, stream=None):
        a, p = self._rows(n_rows)
        check(lib().tria_compact(self.h, C.byref(src), C.byref(dst), p, _ptr(kept_idx),
                                 _ptr(n_kept), _stream(stream)))

    def evict(self, src, dst, n_rows, params, n_kept_out=None, stream=None):
        a, p = self._rows(n_rows)
        check(lib().tria_evict(self.h, C.byref(src), C.byref(dst), p, C.byref(params),
                               _ptr(n_kept_out), _stream(stream)))

    def ggml_evict(self, src, dst, n_rows, params, stream=None):
        """tria_ggml_evict: one step on ggml-described caches (GgmlCache)."""
        a, p = self._rows(n_rows)
        check(lib().tria_ggml_evict(self.h, C.byref(src), C.byref(dst), p, C.byref(params), _stream(stream)))

    def evict_host(self, src, dst, n_rows, params, stream=None):
        """tria_evict_host: src/dst views over page-locked host buffers."""
        a, p = self._rows(n_rows)
        check(lib().tria_evict_host(self.h, C.byref(src), C.byref(dst), p, C.byref(params), _stream(stream)))

    def get_n_kv(self, units: int = 0):
        buf = np.zeros(max(units, 1), np.int32)
        r = lib().tria_get_n_kv(self.h, buf.ctypes.data if units else None, units)
        if r < 0:
            check(r)
        return r, buf[:units]

    def set_timing(self, on: bool = True):
        check(lib().tria_ctx_set_timing(self.h, 1 if on else 0))

    STAGES = ("table", "score", "znorm", "select", "compact")

    def stage_ms(self):
        """Device ms per stage of the last timed evict: dict stage -> ms."""
        buf = np.zeros(5, np.float32)
        k = lib().tria_ctx_stage_ms(self.h, buf.ctypes.data, 5)
        if k < 0:
            check(k)
        return {n: float(buf[i]) for i, n in enumerate(self.STAGES[:k])}

    def launches(self) -> int:
        return int(lib().tria_ctx_launches(self.h))

    def check(self, stream=None):
        """tria_ctx_check: raise TriaError if a kernel of this context reported a
        bad position or a pipeline timeout since the last check."""
        check(lib().tria_ctx_check(self.h, _stream(stream)))

    def set_wait_limit(self, cycles: int = 0):
        """tria_ctx_set_wait_limit (timeout-path tests): 0 restores the default."""
        check(lib().tria_ctx_set_wait_limit(self.h, int(cycles)))

    def set_select_split(self, max_ctas: int = 0):
        """tria_ctx_set_select_split: CTAs per unit in selection (0 automatic, 1 one block)."""
        check(lib().tria_ctx_set_select_split(self.h, int(max_ctas)))

    def score_kv_head_dev(self, k_re, k_im, key_pos, cur_pos, n, layer, kv_head, out, stream=None):
        check(lib().tria_score_kv_head_dev(self.h, _ptr(k_re), _ptr(k_im), _ptr(key_pos), int(cur_pos),
                                           int(n), int(layer), int(kv_head), _ptr(out), _stream(stream)))
