"""CPU tests of the ggml bridge's cache description (include/triattention_ggml.h).

tria_ggml_view maps llama.cpp's per-layer KV tensors (ggml shape [head_dim *
n_head_kv, kv_size], row stride nb[1] per cell) to a tria_kv_view and rejects
tensors that do not have that layout; it touches no memory and needs no GPU,
so fake data addresses serve here.
"""
import pytest

import tria_b200
import workloads

KV, HD, CELLS = 8, 128, 1000


def _layers(type_id=workloads.TYPE_F16, n=3, cells=CELLS, pad=0, base=0x10000):
    rb = workloads.row_bytes(type_id, HD)
    cell = KV * rb + pad
    ks = [tria_b200.ggml_tensor(type_id, HD * KV, cells, cell, base + 0x1000000 * l) for l in range(n)]
    vs = [tria_b200.ggml_tensor(type_id, HD * KV, cells, cell, base + 0x8000000 + 0x1000000 * l) for l in range(n)]
    return ks, vs, cell, rb


@pytest.mark.parametrize("type_id", [workloads.TYPE_F16, workloads.TYPE_Q8_0])
def test_view_of_llama_layout(type_id):
    ks, vs, cell, rb = _layers(type_id, pad=64)
    c = tria_b200.ggml_cache(ks, vs, KV, HD, 0x5000, layer0=7, pos_shared=True, flags=tria_b200.VIEW_POST_ROPE)
    r, v = tria_b200.ggml_view(c)
    assert r == tria_b200.OK, tria_b200.last_error()
    assert (v.type, v.n_layer, v.layer0, v.n_head_kv, v.head0, v.n_cells) == (type_id, 3, 7, KV, 0, CELLS)
    assert v.cell_stride == cell and v.head_stride == rb
    assert [v.k[i] for i in range(3)] == [t.data for t in ks]
    assert [v.v[i] for i in range(3)] == [t.data for t in vs]
    assert v.pos == 0x5000 and v.pos_shared == 1 and v.flags == tria_b200.VIEW_POST_ROPE


def test_view_without_v():
    ks, _, _, _ = _layers()
    r, v = tria_b200.ggml_view(tria_b200.ggml_cache(ks, None, KV, HD, 0x5000))
    assert r == tria_b200.OK and not v.v


def _expect(cache, status, words):
    r, _ = tria_b200.ggml_view(cache)
    assert r == status, (r, tria_b200.last_error())
    msg = tria_b200.last_error()
    for w in words:
        assert w in msg, msg


def test_view_rejects_bad_layouts():
    ks, vs, cell, _ = _layers()
    bad = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV - 2, CELLS, cell, 0x9000)
    _expect(tria_b200.ggml_cache([ks[0], bad, ks[2]], vs, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["k[1]", "ne[0]"])
    q = tria_b200.ggml_tensor(workloads.TYPE_Q8_0, HD * KV, CELLS, KV * 136, 0x9000)
    _expect(tria_b200.ggml_cache([ks[0], q, ks[2]], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["k[1]", "type"])
    other = tria_b200.ggml_tensor(0, HD * KV, CELLS, cell, 0x9000)                  # GGML_TYPE_F32
    _expect(tria_b200.ggml_cache([other], None, KV, HD, 0x5000), tria_b200.ERR_UNSUPPORTED, ["type 0"])
    short = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS - 1, cell, 0x9000)
    _expect(tria_b200.ggml_cache([ks[0], short], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["cells"])
    tight = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS, cell - 2, 0x9000)
    _expect(tria_b200.ggml_cache([tight], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["nb[1]"])
    strided = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS, cell, 0x9000, elem=4)
    _expect(tria_b200.ggml_cache([strided], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["nb[0]"])
    cube = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS, cell, 0x9000)
    cube.ne[2] = 2
    _expect(tria_b200.ggml_cache([cube], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["2-D"])
    wide_v = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS, cell + 64, 0x9000)
    _expect(tria_b200.ggml_cache([ks[0]], [wide_v], KV, HD, 0x5000), tria_b200.ERR_INVALID, ["cell stride"])
    odd = tria_b200.ggml_tensor(workloads.TYPE_Q8_0, 48 * KV, CELLS, 48 * KV, 0x9000)  # head_dim 48: 1.5 blocks
    _expect(tria_b200.ggml_cache([odd], None, KV, 48, 0x5000), tria_b200.ERR_INVALID, ["nb[1]"])
    nodata = tria_b200.ggml_tensor(workloads.TYPE_F16, HD * KV, CELLS, cell, 0)
    _expect(tria_b200.ggml_cache([nodata], None, KV, HD, 0x5000), tria_b200.ERR_INVALID, ["no data"])
