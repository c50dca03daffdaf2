"""Chunked gated delta rule (training): the batched-chunk form with the hand-derived inter-chunk backward against
the token-by-token recurrence and against autograd through an unrolled chunk loop (CPU oracles; the native
state-scan kernel is compared with the CPU scan in the GPU tests)."""
import torch

from arc_forge_2026_b200.models.reference import gated_delta_rule
from arc_forge_2026_b200.train.gdn_chunk import chunk_gated_delta_rule, chunk_gated_delta_rule_loop


def _inputs(B=2, T=150, H=3, Dk=16, Dv=8, seed=0, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g, dtype=dtype), dim=-1) * Dk ** -0.5
    k = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g, dtype=dtype), dim=-1)
    v = torch.randn(B, T, H, Dv, generator=g, dtype=dtype)
    gate = -torch.rand(B, T, H, generator=g, dtype=dtype) * 0.5
    beta = torch.rand(B, T, H, generator=g, dtype=dtype)
    s0 = torch.randn(B, H, Dk, Dv, generator=g, dtype=dtype) * 0.1
    return q, k, v, gate, beta, s0


def test_chunked_forward_matches_recurrence():
    q, k, v, gate, beta, s0 = _inputs(dtype=torch.float32)
    o, S = chunk_gated_delta_rule(q, k, v, gate, beta, chunk=32, state=s0)
    o_ref, S_ref = gated_delta_rule(q, k, v, gate, beta, state=s0)
    assert torch.allclose(o, o_ref.float(), atol=2e-5, rtol=1e-4)
    assert torch.allclose(S, S_ref.float(), atol=2e-5, rtol=1e-4)


def test_inter_chunk_backward_matches_unrolled_autograd():
    q, k, v, gate, beta, s0 = _inputs()
    ins = [t.clone().requires_grad_(True) for t in (q, k, v, gate, beta, s0)]
    ref = [t.clone().requires_grad_(True) for t in (q, k, v, gate, beta, s0)]
    dout = torch.randn(2, 150, 3, 8, dtype=torch.float64, generator=torch.Generator().manual_seed(5))
    dS = torch.randn(2, 3, 16, 8, dtype=torch.float64, generator=torch.Generator().manual_seed(6))
    o, S = chunk_gated_delta_rule(*ins[:5], chunk=32, state=ins[5])
    (o.double() * dout).sum().backward(retain_graph=True)
    (S.double() * dS).sum().backward()
    o2, S2 = chunk_gated_delta_rule_loop(*ref[:5], chunk=32, state=ref[5])
    (o2.double() * dout).sum().backward(retain_graph=True)
    (S2.double() * dS).sum().backward()
    assert torch.allclose(o.double(), o2.double(), atol=1e-6)
    for a, b in zip(ins, ref):
        err = ((a.grad - b.grad).norm() / b.grad.norm()).item()
        assert err < 1e-5, err
