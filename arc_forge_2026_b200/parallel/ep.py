"""Expert parallelism for serving: attention / GDN layers stay data-parallel (each rank keeps its own sessions),
the routed experts are split in contiguous blocks of ``E / world`` per rank, and every MoE layer exchanges tokens
through a symmetric device heap with the native kernels of ``csrc/ep.cu``:

    router (local; also lists each expert's entries) -> ep_dispatch (per-row e4m3 quantisation fused with the
    all-gather to every rank's receive region; the lists go to each expert's owner) -> shared expert (local, overlaps
    the exchange) -> w13 GEMM (waits in its prologue for every rank's dispatch, gathers the listed rows itself) ->
    per-row requantisation of the listed h rows -> w2 GEMM whose epilogue stores each routed row into its token
    owner's combine region and publishes the exchange -> combine (waits in its prologue; k rows in slot order +
    shared + residual). No sort, gather or wait launches: 9 kernels per layer besides the router GEMM.

The reference splits experts the same way (``--ep 4`` in its B200 server configs, ``training/run_records/A1/
config/p30241.server.json:32``) and, on its L4 stack, dispatches by all-gather and combines by a reduce to the
owner rows (``hostcomm.cu:525-700``); here both ends are stores into peer HBM over NVSwitch from inside the
kernels that produce the data.

Every rank must run the same MoE layers in the same order (the exchanges are barriers): the engine steps all
ranks together, a rank with no tokens still joins each exchange with ``T = 0``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import C
from ..ops.moe import Int3ExpertBank

EP_DISPATCH, EP_COMBINE = 0, 1
MAX_RANKS = 8


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def expert_range(E: int, world: int, rank: int) -> tuple[int, int]:
    """[e0, e1) of the experts rank ``rank`` owns."""
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    return rank * n, (rank + 1) * n


def local_bank(bank: Int3ExpertBank, world: int, rank: int) -> Int3ExpertBank:
    e0, e1 = expert_range(bank.num_experts, world, rank)
    return Int3ExpertBank(bank.w13_codes[e0:e1].contiguous(), bank.w13_scales[e0:e1].contiguous(),
                          bank.w2_codes[e0:e1].contiguous(), bank.w2_scales[e0:e1].contiguous())


class ExpertParallel:
    """The exchange state of one EP group: symmetric heap, region views, counters and the native context.

    ``T_cap`` is the most tokens one rank sends per MoE layer (its workspace capacity); the heap holds
    ``world * T_cap`` receive slots and this rank's ``T_cap * k`` combine rows."""

    def __init__(self, world: int, rank: int, T_cap: int, H: int, k: int, E: int, device, group=None):
        if not 1 <= world <= MAX_RANKS:
            raise ValueError(f"expert parallelism supports 1..{MAX_RANKS} ranks, got {world}")
        if world > 1:  # the region layout (slot = rank * T_cap + t, entry owner = entry // (T_cap * k)) must agree
            shapes = [None] * world
            dist.all_gather_object(shapes, (T_cap, H, k, E), group=group)
            if any(sh != shapes[0] for sh in shapes):
                raise ValueError(f"expert-parallel shapes differ across ranks (T_cap, H, k, E): {shapes}; every rank "
                                 f"must use the same capacity (the largest per-rank token count)")
        self.world, self.rank, self.T_cap, self.H, self.k, self.E = world, rank, T_cap, H, k, E
        self.e0, self.e1 = expert_range(E, world, rank)
        self.E_local = self.e1 - self.e0
        dev = torch.device(device)
        rows = world * T_cap
        self.ld_s = (rows + 32 + 3) // 4 * 4
        off_x = 0
        off_s = _align(off_x + rows * H)
        off_ids = _align(off_s + self.ld_s * 4)  # one activation scale per received row
        off_w = _align(off_ids + rows * k * 4)
        off_comb = _align(off_w + rows * k * 4)
        off_flags = _align(off_comb + T_cap * k * H * 2)
        off_rcnt = _align(off_flags + 2 * MAX_RANKS * 8)     # [world sources][E_local] entries per local expert
        off_rlist = _align(off_rcnt + world * self.E_local * 4)  # [world][E_local][T_cap] those entries
        total = _align(off_rlist + world * self.E_local * T_cap * 4)
        self.offsets = [off_x, off_s, off_ids, off_w, off_comb, off_flags, off_rcnt, off_rlist]
        ext = C()
        self.heap = ext.SymmHeap(total, rank, world, dev.index if dev.index is not None else 0)
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, self.heap.handle(), group=group)
            self.heap.open(handles)
            dist.barrier(group=group)  # every heap is zeroed and mapped before any rank stores a flag
        buf = self.heap.tensor()
        self.recv_x = buf[off_x:off_x + rows * H].view(torch.float8_e4m3fn).view(rows, H)
        self.recv_s = buf[off_s:off_s + rows * 4].view(torch.float32)
        self.rcnt = buf[off_rcnt:off_rcnt + world * self.E_local * 4].view(torch.int32).view(world, self.E_local)
        self.rlist = buf[off_rlist:off_rlist + world * self.E_local * T_cap * 4].view(torch.int32).view(
            world, self.E_local, T_cap)
        self.recv_ids = buf[off_ids:off_ids + rows * k * 4].view(torch.int32).view(rows, k)
        self.recv_w = buf[off_w:off_w + rows * k * 4].view(torch.float32)
        self.comb = buf[off_comb:off_comb + T_cap * k * H * 2].view(torch.bfloat16).view(T_cap * k, H)
        self.done = torch.zeros(2, dtype=torch.int32, device=dev)
        self.sent = torch.zeros(2, dtype=torch.int64, device=dev)
        self.expected = torch.zeros(2, dtype=torch.int64, device=dev)
        self.wait_done = torch.zeros(2, dtype=torch.int32, device=dev)
        self.ctx = ext.EpCtx(world, rank, T_cap, H, k, self.E_local, list(self.heap.peers()), self.offsets, self.ld_s,
                             self.done, self.sent, self.expected, self.wait_done)
        self.wait_log = None

    def track_waits(self, layers: int):
        """Accumulate, per MoE layer, the nanoseconds this rank's w13 GEMM waited for the dispatch exchange and its
        combine waited for the combine exchange (block 0 of each kernel; ``wait_log`` int64 [layers, 2]). The
        model's forward restarts the layer count (``ctx.begin_step``); zero the log to start a measurement."""
        self.wait_log = torch.zeros(layers, 2, dtype=torch.int64, device=self.done.device)
        self.ctx.set_wait_log(self.wait_log)
        return self.wait_log

    def close(self):
        if self.heap is not None:
            self.heap.close()
            self.heap = None


class EPMoEWorkspace:
    """Per-layer buffers of the expert-parallel MoE (fixed addresses: CUDA-graph safe). Entries are numbered over
    all ranks (source * T_cap * k + t * k + slot)."""

    def __init__(self, ep: ExpertParallel, I: int, Is: int, device):
        dev = torch.device(device)
        T, k, H, E = ep.T_cap, ep.k, ep.H, ep.E
        n = ep.world * T * k
        i32 = dict(dtype=torch.int32, device=dev)
        self.n = n
        self.logits = torch.empty(T, E + 8, dtype=torch.float32, device=dev)
        self.ids = torch.empty(T, k, **i32)
        self.weights = torch.empty(T, k, dtype=torch.float32, device=dev)
        self.lcnt = torch.zeros(E, **i32)       # this rank's entries per expert (router)
        self.llist = torch.zeros(E, T, **i32)   # and the entries themselves
        self.h = torch.empty(n, I, dtype=torch.bfloat16, device=dev)
        self.hq = torch.empty(n, I, dtype=torch.float8_e4m3fn, device=dev)
        self.hs = torch.zeros(n, dtype=torch.float32, device=dev)
        self.sh_gu = torch.empty(T, 2 * Is, dtype=torch.bfloat16, device=dev)
        self.sh_h = torch.empty(T, Is, dtype=torch.bfloat16, device=dev)
        self.sh_out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)


def moe_forward_ep(x: torch.Tensor, resid: torch.Tensor, router_ext: torch.Tensor, bank: Int3ExpertBank,
                   shared_w13: torch.Tensor, shared_w2: torch.Tensor, ep: ExpertParallel, ws: EPMoEWorkspace,
                   out: torch.Tensor, renorm: bool = True) -> torch.Tensor:
    """out = resid + MoE(x) for this rank's T tokens, with the routed experts spread over the EP group."""
    c = C()
    T, H = x.shape
    k, E = ep.k, ep.E
    if T > ep.T_cap:
        raise ValueError(f"{T} tokens exceed the expert-parallel capacity {ep.T_cap}")
    logits = ws.logits[:T]
    ids, w = ws.ids[:T], ws.weights[:T]
    if T > 0:
        c.gemm(x, router_ext, out=logits, out_fp32=True)
    c.router_topk(logits, E, k, renorm, ids, w, ws.lcnt, ws.llist)  # T == 0: the lists are only cleared
    ep.ctx.dispatch(x, T, ws.ids, ws.weights, ws.lcnt, ws.llist)
    if T > 0:  # the shared expert runs while the peers' dispatch stores land
        c.gemm(x, shared_w13, out=ws.sh_gu[:T])
        c.swiglu(ws.sh_gu[:T], ws.sh_h[:T])
        c.gemm(ws.sh_h[:T], shared_w2, out=ws.sh_out[:T])
    # w13 waits for every rank's dispatch in its prologue; rows and scales come from the receive region
    c.moe_int3_gemm(bank.w13_codes, bank.w13_scales, ep.rcnt, ep.rlist, k, ep.recv_x, ep.recv_s, True, None, None,
                    ws.h, None, None, ep.ctx, True)
    ep.ctx.quant_routed(ws.h, ws.hq, ws.hs)
    c.moe_int3_gemm(bank.w2_codes, bank.w2_scales, ep.rcnt, ep.rlist, 1, ws.hq, ws.hs, False, None, None, ep.comb,
                    ep.recv_w, None, ep.ctx)
    ep.ctx.combine(ep.comb, ws.sh_out[:T] if T > 0 else None, logits if T > 0 else None, E,
                   resid if T > 0 else None, out, T)
    return out
