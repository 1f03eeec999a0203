"""Device-resident KV caches in llama.cpp's layout, for tests and bench.py.

torch is used only as the device allocator and for seeded fills; the
eviction step itself runs in libtriattention_b200.so.

Layout per layer: K and V are [n_cells, n_head_kv * row_bytes] uint8, so a
(layer, kv-head) row sits at cell*cell_stride + head*row_bytes; positions
are int32 [n_layer, n_head_kv, n_cells] (per head after a compaction) or a
shared [n_cells] array for a fresh cache.
"""
from __future__ import annotations

import numpy as np
import torch

import tria_b200
import workloads


class DeviceCache:
    def __init__(self, type_id, n_layer, n_head_kv, head_dim, n_cells, device, with_v=True,
                 layer0=0, head0=0):
        self.type_id, self.n_layer, self.n_head_kv = type_id, n_layer, n_head_kv
        self.head_dim, self.n_cells, self.layer0, self.head0 = head_dim, n_cells, layer0, head0
        self.rb = workloads.row_bytes(type_id, head_dim)
        self.device = torch.device(device)
        shape = (n_layer, n_cells, n_head_kv * self.rb)
        self.k = torch.zeros(shape, dtype=torch.uint8, device=self.device)
        self.v = torch.zeros(shape, dtype=torch.uint8, device=self.device) if with_v else None
        self.pos = torch.zeros((n_layer, n_head_kv, n_cells), dtype=torch.int32, device=self.device)
        self.pos_shared = None

    @property
    def cell_stride(self):
        return self.n_head_kv * self.rb

    def view(self, shared_pos: bool = False) -> tria_b200.KvView:
        pos = self.pos_shared if shared_pos else self.pos
        return tria_b200.make_view(self.type_id, [self.k[l] for l in range(self.n_layer)],
                                   [self.v[l] for l in range(self.n_layer)] if self.v is not None else None,
                                   pos, self.n_cells, self.cell_stride, self.rb, self.n_head_kv,
                                   self.layer0, self.head0, pos_shared=shared_pos)

    def unit_rows(self, which, l, h, n):
        """Bytes of the first n rows of (layer l, head h) as a host [n, rb] array."""
        t = self.k if which == "k" else self.v
        return t[l, :n, h * self.rb:(h + 1) * self.rb].cpu().numpy()

    # ---- fills ----
    def fill_from_host(self, k_bytes, v_bytes=None, pos=None, pos_shared=None):
        self.k.copy_(torch.from_numpy(np.ascontiguousarray(k_bytes)))
        if v_bytes is not None and self.v is not None:
            self.v.copy_(torch.from_numpy(np.ascontiguousarray(v_bytes)))
        if pos is not None:
            self.pos.copy_(torch.from_numpy(np.ascontiguousarray(pos, np.int32)))
        if pos_shared is not None:
            self.pos_shared = torch.from_numpy(np.ascontiguousarray(pos_shared, np.int32)).to(self.device)

    def fill_synthetic(self, seed=0, outlier_p=0.01, n_rows=None):
        """Seeded device-side fill with the bench distributions (see workloads.py)."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        hd, KV = self.head_dim, self.n_head_kv
        n = self.n_cells if n_rows is None else n_rows
        for t in (self.k, self.v):
            if t is None:
                continue
            for l in range(self.n_layer):
                x = torch.randn((n, KV, hd), generator=g, device=self.device, dtype=torch.float32)
                if self.type_id == workloads.TYPE_F16:
                    mask = torch.rand((1, KV, hd), generator=g, device=self.device) < outlier_p
                    x = torch.where(mask, x * 8.0, x)
                    t[l, :n].copy_(x.half().view(torch.uint8).reshape(n, -1))
                else:
                    t[l, :n].copy_(quantize_q8_0_torch(x).reshape(n, -1))
        ar = torch.arange(self.n_cells, dtype=torch.int32, device=self.device)
        self.pos.copy_(ar.expand(self.n_layer, self.n_head_kv, -1))
        self.pos_shared = ar.clone()


def quantize_q8_0_torch(x: torch.Tensor) -> torch.Tensor:
    """ggml q8_0 on the device: [..., hd] f32 -> [..., hd/32*34] uint8."""
    shp = x.shape
    xb = x.reshape(-1, 32)
    d = xb.abs().amax(dim=1) / 127.0
    inv = torch.where(d > 0, 1.0 / torch.where(d > 0, d, torch.ones_like(d)), torch.zeros_like(d))
    q = torch.clamp(torch.round(xb * inv[:, None]), -127, 127).to(torch.int8)
    blk = torch.cat([d.half().view(torch.uint8).reshape(-1, 2), q.view(torch.uint8)], dim=1)
    return blk.reshape(*shp[:-1], shp[-1] // 32 * workloads.Q8_0_BLOCK)
