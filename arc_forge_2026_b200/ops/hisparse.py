"""HiSparse KV offload for QSA serving (``csrc/hisparse.cu``): every finalised page of every QSA layer lives in a
pinned, device-mapped host pool; per session and layer the GPU holds a ring of ``R`` recent pages (this cycle's
tokens are written there) and ``C`` cache slots that the fetch kernel fills with the pages QSA selects (LRU over
cycles). The GPU page pool of a layer is laid out as [S*C cache | S*R ring | max_pages staging | scratch]; staging
pages hold a prompt during its prefill, after which complete pages go to the host pool and the partial one to the
ring.

The reference keeps session history in a host pool with GPU hot blocks and swap-in on demand (paper section 8.2;
``agi2/work/qwen38fn_l4/kaggle/frozen_arc2/hisparse_bridge.py``).
"""
from __future__ import annotations

import torch

from ._ext import C


def gpu_pages(S: int, max_pages: int, cache_slots: int, ring: int) -> int:
    return S * (cache_slots + ring) + max_pages + 1


class HiSparseState:
    def __init__(self, kv, qsa_cache, S: int, max_pages: int, cache_slots: int, ring: int = 4, fp8: bool = False):
        kc0 = kv[0][0]
        dev = kc0.device
        _, Hkv, page, D = kc0.shape
        self.S, self.max_pages, self.C, self.R, self.fp8 = S, max_pages, cache_slots, ring, fp8
        self.staging_base = S * (cache_slots + ring)
        page_bytes = Hkv * page * D * (1 if fp8 else 2)
        ext = C()
        self.pools, self.tables, ptrs = [], [], []
        for (kc, vc), (raw, _key) in zip(kv, qsa_cache):
            hk = ext.HostPool(S * max_pages * page_bytes)
            hv = ext.HostPool(S * max_pages * page_bytes)
            sk = torch.ones(S * max_pages, Hkv, dtype=torch.float32, device=dev) if fp8 else None
            sv = torch.ones(S * max_pages, Hkv, dtype=torch.float32, device=dev) if fp8 else None
            res = torch.full((S, max_pages), -1, dtype=torch.int32, device=dev)
            slot_page = torch.full((S, cache_slots), -1, dtype=torch.int32, device=dev)
            stamp = torch.full((S, cache_slots), -1, dtype=torch.int32, device=dev)
            self.pools.append((hk, hv))
            self.tables.append((res, slot_page, stamp, sk, sv))
            ptrs.append([kc.data_ptr(), vc.data_ptr(), hk.device_ptr(), hv.device_ptr(),
                         sk.data_ptr() if fp8 else 0, sv.data_ptr() if fp8 else 0, res.data_ptr(),
                         slot_page.data_ptr(), stamp.data_ptr(), raw.data_ptr()])
        self.cycle = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ctx = ext.HsCtx(S, max_pages, cache_slots, ring, Hkv, D, fp8, self.cycle, ptrs)

    def ring_page(self, s: int, p: int) -> int:
        return self.S * self.C + s * self.R + p % self.R

    def reset_session(self, s: int):
        for res, slot_page, stamp, _, _ in self.tables:
            res[s].fill_(-1)
            slot_page[s].fill_(-1)
            stamp[s].fill_(-1)

    def host_tensors(self):
        """CPU uint8 views of the host pools [(K, V) per layer] (to fill synthetic contexts)."""
        return [(hk.tensor(), hv.tensor()) for hk, hv in self.pools]

    def close(self):
        for hk, hv in self.pools:
            hk.close()
            hv.close()
        self.pools = []
