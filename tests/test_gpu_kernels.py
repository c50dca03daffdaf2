"""GPU numerics of the dense GEMM and the elementwise/routing kernels against fp32 PyTorch references."""
import pytest
import torch

from arc_forge_2026_b200.models import reference as R
from arc_forge_2026_b200.ops import C, check_status
from arc_forge_2026_b200.quant import fp8

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(1, 64, 128), (100, 2048, 2048), (640, 12352, 2048), (1024, 4096, 4096),
                                   (130, 320, 2048), (640, 2048, 4096)])
def test_gemm_bf16(M, N, K):
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randn(M, K, device=dev, generator=g).bfloat16()
    b = torch.randn(N, K, device=dev, generator=g).bfloat16()
    ref = a.float() @ b.float().t()
    out = C().gemm(a, b)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out, ref) < 1e-2
    out32 = C().gemm(a, b, out_fp32=True)
    assert _rel(out32, ref) < 1e-5


@pytest.mark.parametrize("bn,splits", [(64, 1), (128, 1), (256, 1), (64, 4), (128, 3), (256, 2), (64, 8), (128, 6)])
def test_gemm_tiles_splitk_residual(bn, splits):
    """Split-K runs as one cluster per tile, the partials summed over distributed shared memory in split order:
    accurate, bitwise reproducible, and the fp32 output form agrees with the fp32 product to 1e-5."""
    g = torch.Generator(device=dev).manual_seed(7)
    M, N, K = 300, 1024, 3072
    a = torch.randn(M, K, device=dev, generator=g).bfloat16()
    b = torch.randn(N, K, device=dev, generator=g).bfloat16()
    r = torch.randn(M, N, device=dev, generator=g).bfloat16()
    ref = 0.5 * (a.float() @ b.float().t()) + r.float()
    out = C().gemm(a, b, residual=r, alpha=0.5, bn=bn, splits=splits)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out, ref) < 1e-2
    assert torch.equal(out, C().gemm(a, b, residual=r, alpha=0.5, bn=bn, splits=splits))
    out32 = C().gemm(a, b, out_fp32=True, bn=bn, splits=splits)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out32, a.float() @ b.float().t()) < 1e-5


@pytest.mark.parametrize("act,splits", [(0, 1), (1, 1), (2, 1), (1, 3), (2, 4)])
def test_gemm_bias_gelu_residual_epilogue(act, splits):
    """out = act(alpha * a @ b.T + bias) + residual, in the GEMM's epilogue and in the split-K reduce."""
    import torch.nn.functional as F
    g = torch.Generator(device=dev).manual_seed(11 + act)
    M, N, K = 200, 1024, 2048
    a = torch.randn(M, K, device=dev, generator=g).bfloat16()
    b = (torch.randn(N, K, device=dev, generator=g) * 0.03).bfloat16()
    bias = torch.randn(N, device=dev, generator=g).bfloat16()
    r = torch.randn(M, N, device=dev, generator=g).bfloat16()
    x = 0.5 * (a.float() @ b.float().t()) + bias.float()
    x = {0: x, 1: F.gelu(x, approximate="tanh"), 2: F.gelu(x)}[act]
    out = C().gemm(a, b, residual=r, alpha=0.5, bias=bias, act=act, splits=splits)
    torch.cuda.synchronize()
    check_status()
    assert _rel(out, x + r.float()) < 1e-2
    out32 = C().gemm(a, b, alpha=0.5, bias=bias, act=act, splits=splits, out_fp32=True)
    assert _rel(out32, x) < 1e-4


def test_gemm_strided_a():
    g = torch.Generator(device=dev).manual_seed(8)
    big = torch.randn(64, 4096, device=dev, generator=g).bfloat16()
    a = big[:, 1024:3072]  # row stride 4096
    b = torch.randn(256, 2048, device=dev, generator=g).bfloat16()
    out = C().gemm(a, b)
    assert _rel(out, a.float() @ b.float().t()) < 1e-2


def test_rmsnorm_residual():
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(77, 2048, device=dev, generator=g).bfloat16()
    res = torch.randn(77, 2048, device=dev, generator=g).bfloat16()
    w = (torch.randn(2048, device=dev, generator=g) * 0.1).bfloat16()
    y = torch.empty_like(x)
    res2 = res.clone()
    C().rmsnorm(x, res2, w, y, 1e-6, True)
    h = (x.float() + res.float()).bfloat16()
    assert torch.equal(res2, h)
    ref = R.rms_norm(h.float(), w.float(), 1e-6)
    assert _rel(y, ref) < 5e-3


def test_qk_norm_rope_store():
    g = torch.Generator(device=dev).manual_seed(2)
    T, Hq, Hkv, D, rot, ps = 5, 16, 2, 256, 64, 64
    qkv = torch.randn(T, Hq * 2 * D + 2 * Hkv * D, device=dev, generator=g).bfloat16()
    qw = (torch.randn(D, device=dev, generator=g) * 0.1).bfloat16()
    kw = (torch.randn(D, device=dev, generator=g) * 0.1).bfloat16()
    pos = torch.tensor([0, 1, 700, 5000, 26000], device=dev, dtype=torch.int32)
    slots = torch.tensor([3, 64, 65, 130, 200], device=dev, dtype=torch.int32)
    cos, sin = R.rope_cos_sin(torch.arange(32768, device=dev), rot, 1e7)
    q_out = torch.empty(T, Hq, D, device=dev, dtype=torch.bfloat16)
    kc = torch.zeros(4, Hkv, ps, D, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    C().qk_norm_rope_store(qkv, Hq, Hkv, D, rot, qw, kw, pos, slots, cos, sin, 1e-6, q_out, kc, vc)
    q = qkv[:, : Hq * 2 * D].view(T, Hq, 2 * D)[..., :D].float()
    k = qkv[:, Hq * 2 * D: Hq * 2 * D + Hkv * D].view(T, Hkv, D).float()
    v = qkv[:, Hq * 2 * D + Hkv * D:].view(T, Hkv, D)
    c, s = R.rope_cos_sin(pos.long(), rot, 1e7)
    qr = R.apply_rope(R.rms_norm(q, qw.float(), 1e-6), c, s)
    kr = R.apply_rope(R.rms_norm(k, kw.float(), 1e-6), c, s)
    assert _rel(q_out, qr) < 5e-3
    for t in range(T):
        p, o = divmod(int(slots[t]), ps)
        assert _rel(kc[p, :, o], kr[t]) < 5e-3
        assert torch.equal(vc[p, :, o], v[t])


def test_router_sort_quant_combine():
    g = torch.Generator(device=dev).manual_seed(3)
    T, E, k, H = 640, 320, 10, 2048
    logits = torch.randn(T, E + 8, device=dev, generator=g)
    ids = torch.empty(T, k, device=dev, dtype=torch.int32)
    w = torch.empty(T, k, device=dev)
    C().router_topk(logits, E, k, True, ids, w)
    rw, rid = R.route(logits[:, :E], k, True)
    assert torch.equal(ids.long(), rid)
    torch.testing.assert_close(w, rw, rtol=1e-5, atol=1e-6)
    off = torch.empty(E + 1, device=dev, dtype=torch.int32)
    row_token = torch.empty(T * k, device=dev, dtype=torch.int32)
    row_entry = torch.empty_like(row_token)
    entry_row = torch.empty_like(row_token)
    C().expert_sort(ids, E, None, off, row_token, row_entry, entry_row, 1)
    flat = ids.flatten().long()
    order = torch.sort(flat, stable=True).indices
    assert torch.equal(row_entry.long(), order)
    assert torch.equal(entry_row.long()[order], torch.arange(T * k, device=dev))
    counts = torch.bincount(flat, minlength=E)
    assert torch.equal(off[1:].long(), counts.cumsum(0))
    # padded segments: starts are multiples of 8, rows keep the stable order inside each segment
    rows = T * k + 7 * E
    off8 = torch.empty(E + 1, device=dev, dtype=torch.int32)
    rt8, re8 = torch.empty(rows, device=dev, dtype=torch.int32), torch.empty(rows, device=dev, dtype=torch.int32)
    er8 = torch.empty(T * k, device=dev, dtype=torch.int32)
    C().expert_sort(ids, E, None, off8, rt8, re8, er8, 8)
    assert torch.all(off8 % 8 == 0)
    for e in (0, 5, E - 1):
        a, c_ = int(off8[e]), int(counts[e])
        assert torch.equal(re8[a:a + c_].long(), order[int(off[e]):int(off[e]) + c_])
        assert torch.all(re8[a + c_:int(off8[e + 1])] == -1)
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    q = torch.empty(T * k, H, device=dev, dtype=torch.float8_e4m3fn)
    sc = torch.empty(T * k, H // 128, device=dev)
    C().quant_rows_e4m3(x, row_token, None, T * k, q, sc, False)
    sc_gm = torch.empty(H // 128, T * k + 32, device=dev)
    C().quant_rows_e4m3(x, row_token, None, T * k, q, sc_gm, True)
    assert torch.equal(sc_gm[:, :T * k].t(), sc)
    rq, rs = fp8.quantize_act_groups(x[row_token.long()].float())
    torch.testing.assert_close(sc, rs, rtol=1e-6, atol=0)
    assert _rel(q.float(), rq.float()) < 1e-2
    y = torch.randn(T * k, H, device=dev, generator=g).bfloat16()
    shared = torch.randn(T, H, device=dev, generator=g).bfloat16()
    out = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
    C().moe_combine(y, entry_row, k, shared, logits, E, x, out)
    ref = x.float() + torch.sigmoid(logits[:, E:E + 1]) * shared.float() + y.float()[entry_row.long()].view(T, k, H).sum(1)
    assert _rel(out, ref) < 5e-3
    check_status()


def test_peer_wait_gives_up_with_status_and_the_context_survives():
    """A peer flag that nothing raises: the bounded wait returns after ~2 s with the timeout bit set; the device
    keeps working. A dispatch followed by its own wait (one rank) does not time out."""
    from arc_forge_2026_b200.parallel.ep import EP_COMBINE, EP_DISPATCH, ExpertParallel
    check_status()
    ep = ExpertParallel(1, 0, 8, 256, 2, 4, "cuda")
    x = torch.randn(8, 256, device="cuda").bfloat16()
    ids = torch.tensor([[0, 1]] * 8, dtype=torch.int32, device="cuda")  # every token: experts 0 and 1
    w = torch.ones(8, 2, device="cuda")
    cnt = torch.tensor([8, 8, 0, 0], dtype=torch.int32, device="cuda")
    lst = torch.zeros(4, 8, dtype=torch.int32, device="cuda")
    lst[0] = torch.arange(0, 16, 2, dtype=torch.int32, device="cuda")
    lst[1] = torch.arange(1, 16, 2, dtype=torch.int32, device="cuda")
    ep.ctx.dispatch(x, 8, ids, w, cnt, lst)
    ep.ctx.wait(EP_DISPATCH)
    torch.cuda.synchronize()
    assert check_status() == 0
    ep.ctx.wait(EP_COMBINE)  # nothing publishes a combine: gives up
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer wait timed out"):
        check_status()
    y = torch.ones(4, device="cuda")
    assert float((y * 2).sum()) == 8.0
    ep.close()
