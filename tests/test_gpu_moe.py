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
    """One expert, inputs whose fp8 quantisation is exact: the kernel must match the fp32 product tightly."""
    E, H, I, T = 1, 256, 128, 40
    bank = Int3ExpertBank.random(E, H, I, dev, seed=3)
    g = torch.Generator(device="cpu").manual_seed(1)
    # values in e4m3's integer range with an amax of exactly 448 per group -> scale 1, exact
    x = torch.randint(-8, 8, (T, H), generator=g).float()
    x[:, ::128] = 448.0
    x = x.bfloat16().to(dev)
    off = torch.tensor([0, T], dtype=torch.int32, device=dev)
    xq = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=dev)
    xs = torch.zeros(H // 128, 128, device=dev)  # group-major, row stride % 4 == 0, >= T + 32
    C().quant_rows_e4m3(x, None, None, T, xq, xs, True)
    assert torch.all(xs[:, :T] == 1.0)
    hq = torch.empty(T, I, dtype=torch.float8_e4m3fn, device=dev)
    hs = torch.zeros(I // 128, 128, device=dev)
    C().moe_int3_gemm(bank.w13_codes, bank.w13_scales, off, xq, xs, True, hq, hs, None, None, None)
    torch.cuda.synchronize()
    check_status()
    w13, _ = bank.dequant()
    h = x.float() @ w13[0].t()
    hh = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
    got = hq.float() * hs[:, :T].t().repeat_interleave(128, -1)
    assert _rel(got, hh) < 4e-2  # e4m3 output quantisation (3 mantissa bits)


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
