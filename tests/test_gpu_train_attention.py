"""Native training attention (csrc/attention_train.cu) against the fp32 varlen causal oracle: forward output and
the q / k / v gradients, GQA, D 128 and 256, ragged packed segments; bitwise reproducible across runs."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.train.attention import varlen_attention, varlen_attention_reference

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("Hq,Hkv,D,lens", [
    (4, 1, 128, [300, 129, 64, 1000]),
    (16, 2, 256, [77, 513, 200]),
    (24, 2, 256, [130, 640]),     # the reference model's heads (GQA 12)
    (8, 8, 128, [1, 63, 65, 128]),
])
def test_forward_and_gradients_match_oracle(Hq, Hkv, D, lens):
    g = torch.Generator().manual_seed(Hq + D)
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    q = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev).requires_grad_()
    k = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    v = torch.randn(T, Hkv, D, generator=g).bfloat16().to(dev).requires_grad_()
    do = torch.randn(T, Hq, D, generator=g).bfloat16().to(dev)
    out = varlen_attention(q, k, v, cu)
    out.backward(do)
    torch.cuda.synchronize()
    check_status()
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    ref = varlen_attention_reference(qf, kf, vf, cu)
    ref.backward(do.float())
    assert _rel(out, ref) < 1e-2
    assert _rel(q.grad, qf.grad) < 2e-2
    assert _rel(k.grad, kf.grad) < 2e-2
    assert _rel(v.grad, vf.grad) < 2e-2
    # bitwise reproducible: one owner per output element, fixed order
    grads = [t.grad.clone() for t in (q, k, v)]
    for t in (q, k, v):
        t.grad = None
    out2 = varlen_attention(q, k, v, cu)
    out2.backward(do)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    for a, t in zip(grads, (q, k, v)):
        assert torch.equal(a, t.grad)
