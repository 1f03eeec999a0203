"""GPU: a pipeline wait that gives up is reported, not lost.

Every wait of the warp-specialised scoring kernel is bounded; when one gives
up the kernel sets a timeout bit, stops issuing work, waits (with the default
bound) for the copies it already issued and returns.  These tests shorten the
bound through the fault-injection hook tria_ctx_set_wait_limit to a few
dozen cycles, so the first wait on a TMA stage runs out long before its copy
lands: nothing faults or hangs, the step reports TRIA_ERR_TIMEOUT through
tria_get_n_kv (tria_evict) or tria_ctx_check (separate stages), and the same
context then runs a normal step whose result equals a fresh context's.
"""
import numpy as np
import pytest

import tria_b200
import workloads

pytestmark = pytest.mark.gpu

L, H, KV, HD, N = 2, 32, 8, 128, 2048
SHORT_WAIT = 32          # cycles: far below the latency of any bulk copy


@pytest.fixture
def setup(torch_dev, tmp_path):
    import devcache
    path = workloads.write_tria(str(tmp_path / "t.tria"), L, H, KV, HD, seed=5)
    st = tria_b200.load(path)
    src = devcache.DeviceCache(workloads.TYPE_F16, L, KV, HD, N, torch_dev)
    src.fill_synthetic(seed=3)
    yield st, src
    tria_b200.free(st)


def _evict(ctx, src, dst, shared, params):
    ctx.evict(src.view(shared_pos=shared), dst.view(), np.full(L * KV, N, np.int32), params)
    return ctx.get_n_kv(L * KV)


@pytest.mark.parametrize("shared", [True, False])     # staged table rows / rows read from L2
def test_timeout_surfaces_through_get_n_kv(setup, torch_dev, shared):
    import devcache
    import torch
    st, src = setup
    params = tria_b200.EvictParams(N, 256, 100, 0, 0, 0)
    ctx = tria_b200.Context(st, 0)
    ref_ctx = tria_b200.Context(st, 0)
    try:
        dst = devcache.DeviceCache(workloads.TYPE_F16, L, KV, HD, N, torch_dev)
        ctx.set_wait_limit(SHORT_WAIT)
        with pytest.raises(tria_b200.TriaError) as ei:
            _evict(ctx, src, dst, shared, params)
        assert ei.value.status == tria_b200.ERR_TIMEOUT
        assert "gave up" in str(ei.value)
        # the status was cleared and the context still works with the default bound
        ctx.set_wait_limit(0)
        mx, counts = _evict(ctx, src, dst, shared, params)
        ref_dst = devcache.DeviceCache(workloads.TYPE_F16, L, KV, HD, N, torch_dev)
        mx_r, counts_r = _evict(ref_ctx, src, ref_dst, shared, params)
        assert mx == mx_r and np.array_equal(counts, counts_r)
        torch.cuda.synchronize()
        for l in range(L):
            m = int(counts[l * KV])
            assert torch.equal(dst.k[l, :m], ref_dst.k[l, :m])
            assert torch.equal(dst.pos[l, :, :m], ref_dst.pos[l, :, :m])
    finally:
        ctx.close()
        ref_ctx.close()


def test_timeout_surfaces_through_ctx_check(setup, torch_dev):
    import torch
    st, src = setup
    ctx = tria_b200.Context(st, 0)
    try:
        scores = torch.empty((L * KV, N), dtype=torch.float32, device=torch_dev)
        ctx.check()                                       # nothing reported yet
        ctx.set_wait_limit(SHORT_WAIT)
        ctx.score(src.view(shared_pos=True), np.full(L * KV, N, np.int32), N, scores)
        with pytest.raises(tria_b200.TriaError) as ei:
            ctx.check()
        assert ei.value.status == tria_b200.ERR_TIMEOUT
        ctx.check()                                       # cleared by the first check
        ctx.set_wait_limit(0)
        ctx.score(src.view(shared_pos=True), np.full(L * KV, N, np.int32), N, scores)
        ctx.check()
        assert torch.isfinite(scores).all()
    finally:
        ctx.close()
