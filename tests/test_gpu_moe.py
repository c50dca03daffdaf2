"""GPU numerics of the INT3 W3A8 expert GEMMs and the whole routed-MoE block against the fp32 oracle."""
import pytest
import torch

from arc_forge_2026_b200.ops import C, check_status
from arc_forge_2026_b200.ops.moe import (Int3ExpertBank, MoEWorkspace, moe_forward, moe_reference,
                                         router_weight_with_shared_gate)

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("E,H,I,Is,k,T", [(8, 256, 128, 128, 2, 1), (8, 256, 256, 128, 2, 100),
                                          (32, 512, 256, 256, 4, 37), (320, 2048, 512, 512, 10, 640)])
def test_moe_block_matches_oracle(E, H, I, Is, k, T):
    g = torch.Generator(device="cpu").manual_seed(E + T)
    bank = Int3ExpertBank.random(E, H, I, dev, seed=E + H)
    router = (torch.randn(E, H, generator=g) * 0.02).bfloat16().to(dev)
    sgate = (torch.randn(1, H, generator=g) * 0.02).bfloat16().to(dev)
    rext = router_weight_with_shared_gate(router, sgate)
    sw13 = (torch.randn(2 * Is, H, generator=g) * 0.02).bfloat16().to(dev)
    sw2 = (torch.randn(H, Is, generator=g) * 0.02).bfloat16().to(dev)
    x = torch.randn(T, H, generator=g).bfloat16().to(dev)
    resid = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)  # compare the MoE output itself
    ws = MoEWorkspace(T, E, k, H, I, Is, dev)
    out = moe_forward(x, resid, rext, bank, sw13, sw2, k, ws)
    torch.cuda.synchronize()
    check_status()
    ref = moe_reference(x, resid, rext, bank, sw13, sw2, k)
    assert _rel(out, ref) < 2e-2


def test_int3_gemm_single_expert_exact_inputs():
    """One expert, inputs whose per-row fp8 quantisation is exact: the kernel must match the fp32 product tightly.
    The expert's list names the rows in a shuffled order; outputs land on the rows of their entries."""
    E, H, I, T = 1, 256, 256, 40
    bank = Int3ExpertBank.random(E, H, I, dev, seed=3)
    g = torch.Generator(device="cpu").manual_seed(1)
    # values in e4m3's integer range with a row amax of exactly 448 -> scale 1, exact
    x = torch.randint(-8, 8, (T, H), generator=g).float()
    x[:, 0] = 448.0
    x = x.bfloat16().to(dev)
    cnt = torch.tensor([T], dtype=torch.int32, device=dev)
    lst = torch.randperm(T, generator=g).int().view(1, T).to(dev)
    xq = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
    xs = torch.zeros(T, device=dev)
    C().quant_rows_e4m3_row(x, None, None, T, xq, xs)
    assert torch.all(xs == 1.0)
    h = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
    C().moe_int3_gemm(bank.w13_codes, bank.w13_scales, cnt, lst, 1, xq, xs, True, None, None, h, None)
    torch.cuda.synchronize()
    check_status()
    w13, w2 = bank.dequant()
    hr = x.float() @ w13[0].t()
    hh = torch.nn.functional.silu(hr[:, :I]) * hr[:, I:]
    assert _rel(h, hh) < 1e-2  # bf16 output rounding only
    # w2 on the same rows (scale 1 again), a routing weight per entry
    hq = torch.empty(T, I, dtype=torch.float8_e4m3fn, device=dev)
    hs = torch.zeros(T, device=dev)
    C().quant_rows_e4m3_row(h, None, None, T, hq, hs)
    rw = torch.rand(T, device=dev)
    y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    C().moe_int3_gemm(bank.w2_codes, bank.w2_scales, cnt, lst, 1, hq, hs, False, None, None, y, rw)
    torch.cuda.synchronize()
    check_status()
    yr = (hq.float() * hs[:, None]) @ w2[0].t() * rw[:, None]
    assert _rel(y, yr) < 1e-2


def test_router_lists_name_every_entry_once():
    T, E, k = 300, 64, 6
    g = torch.Generator(device="cpu").manual_seed(2)
    logits = torch.randn(T, E + 8, generator=g).to(dev)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    w = torch.empty(T, k, device=dev)
    cnt = torch.full((E,), 7, dtype=torch.int32, device=dev)  # stale counts are cleared by the launcher
    lst = torch.full((E, T), -1, dtype=torch.int32, device=dev)
    C().router_topk(logits, E, k, True, ids, w, cnt, lst)
    torch.cuda.synchronize()
    cnt, lst, ids = cnt.cpu(), lst.cpu(), ids.cpu()
    assert int(cnt.sum()) == T * k
    seen = torch.cat([lst[e, : int(cnt[e])] for e in range(E)])
    assert torch.equal(seen.sort().values, torch.arange(T * k, dtype=torch.int32))
    for e in range(E):
        entries = lst[e, : int(cnt[e])].long()
        assert torch.all(ids.view(-1)[entries] == e)


def test_per_row_quantisation_matches_oracle():
    from arc_forge_2026_b200.quant import fp8
    g = torch.Generator(device="cpu").manual_seed(4)
    x = (torch.randn(300, 2048, generator=g) * torch.rand(300, 1, generator=g) * 5).bfloat16()
    x[7] = 0  # an all-zero row: scale 1e-30 / 448, codes zero
    rt = torch.randint(0, 300, (500,), generator=g).int()
    q = torch.empty(520, 2048, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.zeros(520, device=dev)
    n = torch.tensor([500], dtype=torch.int32, device=dev)
    C().quant_rows_e4m3_row(x.to(dev), rt.to(dev), n, 520, q, s)
    torch.cuda.synchronize()
    rq, rs = fp8.quantize_rows(x[rt.long()].float())
    assert torch.equal(s[:500].cpu(), rs)
    assert torch.equal(q[:500].cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("E,H,I,k,T", [(8, 256, 256, 2, 37), (64, 1024, 512, 8, 300)])
def test_fp8_block_experts_match_oracle(E, H, I, k, T):
    """Block-FP8 experts (the teacher's format) through the same expert kernels: W8A8 with 128x128 weight scales."""
    from arc_forge_2026_b200.ops.moe import Fp8ExpertBank
    g = torch.Generator(device="cpu").manual_seed(E + T + 1)
    bank = Fp8ExpertBank.from_weights(torch.randn(E, 2 * I, H, generator=g) * 0.02,
                                      torch.randn(E, H, I, generator=g) * 0.02, dev)
    rext = router_weight_with_shared_gate((torch.randn(E, H, generator=g) * 0.02).bfloat16().to(dev),
                                          (torch.randn(1, H, generator=g) * 0.02).bfloat16().to(dev))
    sw13 = (torch.randn(2 * 128, H, generator=g) * 0.02).bfloat16().to(dev)
    sw2 = (torch.randn(H, 128, generator=g) * 0.02).bfloat16().to(dev)
    x = torch.randn(T, H, generator=g).bfloat16().to(dev)
    resid = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    ws = MoEWorkspace(T, E, k, H, I, 128, dev)
    out = moe_forward(x, resid, rext, bank, sw13, sw2, k, ws)
    torch.cuda.synchronize()
    check_status()
    ref = moe_reference(x, resid, rext, bank, sw13, sw2, k)
    assert _rel(out, ref) < 2e-2
