"""GPU numerics of the GDN decode/verify kernels: prefill, plain decode and speculative cycles with a deferred
commit of the accepted prefix, against the sequential fp32 recurrence."""
import pytest
import torch

from arc_forge_2026_b200.ops import check_status
from arc_forge_2026_b200.ops.gdn import GdnScratch, GdnShape, GdnState, gdn_decode, gdn_reference_from_mixed

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _params(shape, g):
    conv_w = (torch.randn(shape.conv_dim, 4, generator=g) * 0.3).to(dev)
    A_log = torch.log(torch.empty(shape.Hv).uniform_(1, 16, generator=g)).to(dev)
    dt_bias = (torch.randn(shape.Hv, generator=g) * 0.5).to(dev)
    norm_w = (1 + 0.1 * torch.randn(shape.Dv, generator=g)).bfloat16().to(dev)
    return conv_w, A_log, dt_bias, norm_w


@pytest.mark.parametrize("dims", [(2, 64, 4, 64), (16, 128, 32, 128)])
def test_gdn_spec_cycles_match_sequential(dims):
    shape = GdnShape(*dims)
    g = torch.Generator().manual_seed(sum(dims))
    conv_w, A_log, dt_bias, norm_w = _params(shape, g)
    S, P, K1, cycles = 3, 9, 5, 6
    L = P + cycles * K1
    true = (torch.randn(S, L, shape.mixed_dim, generator=g)).bfloat16().to(dev)
    refs = [gdn_reference_from_mixed(true[s], shape, conv_w, A_log, dt_bias, norm_w) for s in range(S)]
    slots = torch.tensor([2, 0, 1], dtype=torch.int32, device=dev)  # sequences live in permuted slots
    state = GdnState(shape, 4, K1, dev)
    n_commit = torch.zeros(4, dtype=torch.int32, device=dev)
    # prefill P tokens per sequence (commit everything)
    scratch = GdnScratch(shape, S, P, dev)
    out = torch.empty(S * P, shape.Hv * shape.Dv, dtype=torch.bfloat16, device=dev)
    gdn_decode(true[:, :P].reshape(S * P, -1).contiguous(), shape, state, conv_w, A_log, dt_bias, norm_w,
               n_commit, slots, out, P, commit_current=True, scratch=scratch)
    for s in range(S):
        assert _rel(out[s * P:(s + 1) * P], refs[s][:P]) < 2e-2
    # speculative cycles: row 0 is the committed-but-unprocessed token, rows 1..4 drafts; a random prefix is right
    pos = [P] * S
    acc_prev = [0] * S
    for c in range(cycles):
        rows = torch.randn(S, K1, shape.mixed_dim, generator=g).bfloat16().to(dev)  # wrong drafts by default
        n_acc = [int(torch.randint(0, K1, (1,), generator=g)) for _ in range(S)]
        for s in range(S):
            m = n_acc[s] + 1
            rows[s, :m] = true[s, pos[s]:pos[s] + m]
        nc = torch.zeros(4, dtype=torch.int32)
        for s in range(S):
            nc[int(slots[s])] = acc_prev[s]
        n_commit.copy_(nc)
        out = torch.empty(S * K1, shape.Hv * shape.Dv, dtype=torch.bfloat16, device=dev)
        gdn_decode(rows.reshape(S * K1, -1).contiguous(), shape, state, conv_w, A_log, dt_bias, norm_w, n_commit,
                   slots, out, K1, parity=c & 1)
        torch.cuda.synchronize()
        for s in range(S):
            m = n_acc[s] + 1
            assert _rel(out[s * K1:s * K1 + m], refs[s][pos[s]:pos[s] + m]) < 2e-2, (c, s)
            pos[s] += m
            acc_prev[s] = m
    check_status()
