"""Packed training bins (train/packing.py): best-fit-decreasing placement, labels / positions / resets, and the
student's packed forward equal to running every sequence on its own (conv history, GDN state and attention all
stop at sequence starts)."""
import pytest
import torch

from arc_forge_2026_b200.config import preset
from arc_forge_2026_b200.train.packing import best_fit_decreasing, pack
from arc_forge_2026_b200.train.student import random_student


def test_best_fit_decreasing_and_bin_layout():
    assert best_fit_decreasing([128, 64, 128, 192], 256) == [[3, 1], [0, 2]]
    with pytest.raises(ValueError):
        best_fit_decreasing([300], 256)
    seqs = [list(range(1, 71)), list(range(100, 140))]
    masks = [[1] * 70, [0] * 10 + [1] * 30]
    (b,) = pack(seqs, 256, loss_masks=masks)
    assert b.seq_index == [0, 1] and b.cu_seqlens.tolist() == [0, 128, 192]
    assert b.chunk_reset.tolist() == [1, 0, 1]
    assert b.labels[:3].tolist() == [2, 3, 4] and b.labels[69].item() == -1 and (b.labels[70:128] == -1).all()
    assert (b.labels[128:137] == -1).all() and b.labels[137].item() == 110  # prompt part of the second one masked
    assert b.pos[128].item() == 0 and b.pos[127].item() == 127
    assert b.tokens == 69 + 30  # position 9 predicts the first unmasked token


def test_packed_forward_equals_separate_sequences():
    torch.manual_seed(0)
    cfg = preset("tiny_cpu")
    st = random_student(cfg, "cpu", seed=3, checkpoint_layers=False)
    g = torch.Generator().manual_seed(1)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (70, 40, 100)]
    bins = pack(seqs, 256)
    with torch.no_grad():
        for b in bins:
            h = st.hidden(b.ids[None], pack=b.forward_args())[0]
            for s0, i in zip(b.cu_seqlens.tolist(), b.seq_index):
                n = len(seqs[i])
                ref = st.hidden(torch.tensor([seqs[i]]))[0].float()
                # bf16 activations: shapes differ (pads, bin length), so allow rounding-level differences only
                err = (h[s0:s0 + n].float() - ref).norm() / ref.norm()
                assert err < 1e-2, (i, float(err))


def test_no_gradient_crosses_a_sequence_start():
    cfg = preset("tiny_cpu")
    st = random_student(cfg, "cpu", seed=4, checkpoint_layers=False)
    g = torch.Generator().manual_seed(2)
    seqs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (90, 60)]
    (b,) = pack(seqs, 256)
    x = torch.nn.functional.embedding(b.ids[None], st.embed).detach().requires_grad_(True)
    h = x
    for L in st.layers:
        h = L(h, b.forward_args())
    s1 = b.cu_seqlens[1].item()
    h[0, s1:s1 + len(seqs[b.seq_index[1]])].float().pow(2).sum().backward()
    assert x.grad[0, :s1].abs().max().item() == 0.0          # nothing flows back into the earlier sequence
    assert x.grad[0, s1:].abs().max().item() > 0.0
