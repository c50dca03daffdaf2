"""The allocation-free attention entry point, called the way a caller without an allocator would: through its
exported C symbol, with inputs and outputs it owns, and no scratch of its own. Its results must match the regular
entry point (same kernels, scratch from the framework) on two calls in a row -- the second call reuses the fixed
device array the first one left behind, with different inputs and a different split count.

Kept in a file that pytest collects last, so a run that stops at the first failure has run everything else."""
import ctypes
import math

import pytest
import torch

import arc_forge_2026_b200._C as ext
from arc_forge_2026_b200.ops import C
from arc_forge_2026_b200.ops.attention import paged_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


class Params(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("kcache", ctypes.c_void_p), ("vcache", ctypes.c_void_p),
                ("num_pages", ctypes.c_int), ("block_table", ctypes.c_void_p), ("max_pages", ctypes.c_int),
                ("seq_lens", ctypes.c_void_p), ("num_seqs", ctypes.c_int), ("q_per_seq", ctypes.c_int),
                ("Hq", ctypes.c_int), ("Hkv", ctypes.c_int), ("D", ctypes.c_int), ("scale", ctypes.c_float),
                ("splits", ctypes.c_int), ("window", ctypes.c_int), ("gate", ctypes.c_void_p),
                ("gate_ld", ctypes.c_int), ("gate_head_stride", ctypes.c_int), ("out", ctypes.c_void_p)]


def _lib():
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.afb_paged_attention_noalloc
    fn.argtypes = [ctypes.POINTER(Params), ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _status(reset=True):
    """The entry point's kernel status word on the current device (0 = every wait finished)."""
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.afb_paged_attention_noalloc_status
    fn.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]
    fn.restype = ctypes.c_int
    v = ctypes.c_uint(0xFFFFFFFF)
    assert fn(ctypes.byref(v), int(reset)) == 0
    return v.value


def _case(seed, lens, qp, D=256, Hq=16, Hkv=2):
    g = torch.Generator().manual_seed(seed)
    S = len(lens)
    maxp = max((L + 63) // 64 for L in lens)
    P = S * maxp + 2
    kc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    bt = torch.randperm(P, generator=g)[: S * maxp].view(S, maxp).int().to(dev)
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(S * qp, Hq, D, generator=g).bfloat16().to(dev)
    qkv = torch.randn(S * qp, Hq, 2 * D, generator=g).bfloat16().to(dev)  # gate = qkv[..., D:]
    return kc, vc, bt, seq_lens, q, qkv, maxp


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _poison_scratch(fn):
    """Leave NaN partials in the shared array: one call over NaN queries with more splits than the calls after it,
    so a later call that read a partial it did not write itself would return NaN."""
    kc, vc, bt, seq_lens, q, qkv, maxp = _case(7, [4000, 4000], 5)
    q.fill_(float("nan"))
    out = torch.empty_like(q)
    p = Params(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), maxp, seq_lens.data_ptr(),
               2, 5, 16, 2, 256, 1 / 16.0, 8, 0, None, 0, 0, out.data_ptr())
    assert fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()


@torch.no_grad()
def test_noalloc_attention_matches_regular_entry_point_twice():
    fn = _lib()
    _status(reset=True)
    _poison_scratch(fn)
    for seed, lens, qp, splits in ((0, [5, 700, 3000, 130], 5, 4), (1, [2000, 9, 4100], 1, 3)):
        kc, vc, bt, seq_lens, q, qkv, maxp = _case(seed, lens, qp)
        S, Hq, D = len(lens), q.shape[1], q.shape[2]
        gate = qkv[..., D:]
        scale = 1.0 / math.sqrt(D)
        pps = math.ceil(maxp / splits)
        expected = torch.empty_like(q)
        C().paged_attention(q, kc, vc, bt, seq_lens, qp, scale, expected, gate, Hq * 2 * D, 2 * D, splits, pps, 0,
                            None)
        got = torch.full_like(q, float("nan"))
        p = Params(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), maxp, seq_lens.data_ptr(),
                   S, qp, Hq, kc.shape[1], D, scale, splits, 0, gate.data_ptr(), Hq * 2 * D, 2 * D, got.data_ptr())
        rc = fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0, rc
        # same kernels, same split count and pages per split: the results are identical bit for bit
        assert torch.equal(got, expected)
        ref = paged_attention_reference(q, kc, vc, bt, seq_lens, qp, gate=gate)
        assert _rel(got, ref) < 1e-2
    assert _status(reset=True) == 0


def test_noalloc_attention_rejects_oversized_split_scratch():
    fn = _lib()
    kc, vc, bt, seq_lens, q, qkv, maxp = _case(2, [64] * 40, 5)
    out = torch.empty_like(q)
    # 64 splits x 200 tokens x 16 heads x 257 floats is far beyond the fixed 4 MiB
    p = Params(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), maxp, seq_lens.data_ptr(),
               40, 5, 16, 2, 256, 1 / 16.0, 64, 0, None, 0, 0, out.data_ptr())
    assert fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == -2


def test_noalloc_attention_rejects_bad_shapes_before_launching():
    fn = _lib()
    kc, vc, bt, seq_lens, q, qkv, maxp = _case(3, [100, 200], 5)
    out = torch.empty_like(q)
    base = dict(num_seqs=2, q_per_seq=5, Hq=16, Hkv=2, D=256)

    def call(**kw):
        a = dict(base, **kw)
        p = Params(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), maxp,
                   seq_lens.data_ptr(), a["num_seqs"], a["q_per_seq"], a["Hq"], a["Hkv"], a["D"], 1 / 16.0, 1, 0,
                   None, 0, 0, out.data_ptr())
        return fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)

    assert call(D=64) == -1            # only head dims 128 and 256 are built
    assert call(q_per_seq=9) == -1     # 9 rows x 8 query heads per KV head = 72 > 64 rows of one tile
    assert call(Hq=15) == -1           # Hq must be a multiple of Hkv


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@torch.no_grad()
def test_noalloc_attention_on_a_second_device():
    """The first call on another GPU resolves that GPU's own copy of the array and raises that GPU's shared-memory
    limit for the kernel; its result must match the regular entry point there too."""
    fn = _lib()
    with torch.cuda.device(1):
        global dev
        old, dev = dev, "cuda:1"
        try:
            kc, vc, bt, seq_lens, q, qkv, maxp = _case(4, [300, 2500], 5)
        finally:
            dev = old
        D, Hq = 256, 16
        gate = qkv[..., D:]
        expected = torch.empty_like(q)
        pps = math.ceil(maxp / 2)
        C().paged_attention(q, kc, vc, bt, seq_lens, 5, 1 / 16.0, expected, gate, Hq * 2 * D, 2 * D, 2, pps, 0, None)
        got = torch.empty_like(q)
        p = Params(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], bt.data_ptr(), maxp, seq_lens.data_ptr(),
                   2, 5, Hq, 2, D, 1 / 16.0, 2, 0, gate.data_ptr(), Hq * 2 * D, 2 * D, got.data_ptr())
        assert fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, expected)
        assert _status(reset=True) == 0
