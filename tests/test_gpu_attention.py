"""GPU numerics of the paged decode/verify attention against the fp32 oracle."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.ops.attention import paged_attention, paged_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("D,Hq,Hkv,qp,lens,splits", [
    (256, 16, 2, 5, [5, 64, 70, 1000], None),
    (256, 16, 2, 1, [1, 300, 4097], 4),
    (128, 16, 2, 5, [7, 129, 2000], 3),
    (256, 16, 2, 5, [24000, 4100], None),
])
def test_paged_attention(D, Hq, Hkv, qp, lens, splits):
    g = torch.Generator(device="cpu").manual_seed(D + qp + len(lens))
    S = len(lens)
    maxp = max((L + 63) // 64 for L in lens)
    P = S * maxp + 3
    kc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(P, Hkv, 64, D, generator=g).bfloat16().to(dev)
    perm = torch.randperm(P, generator=g)[: S * maxp].view(S, maxp).int().to(dev)  # scattered pages
    seq_lens = torch.tensor(lens, dtype=torch.int32, device=dev)
    q = torch.randn(S * qp, Hq, D, generator=g).bfloat16().to(dev)
    qkv_like = torch.randn(S * qp, Hq, 2 * D, generator=g).bfloat16().to(dev)  # gate at [..., D:]
    gate_view = qkv_like[..., D:]
    out = torch.empty_like(q)
    paged_attention(q, kc, vc, perm, seq_lens, qp, out, gate=qkv_like[..., D:], gate_ld=Hq * 2 * D,
                    gate_head_stride=2 * D, splits=splits)
    torch.cuda.synchronize()
    check_status()
    ref = paged_attention_reference(q, kc, vc, perm, seq_lens, qp, gate=gate_view)
    assert _rel(out, ref) < 1e-2
