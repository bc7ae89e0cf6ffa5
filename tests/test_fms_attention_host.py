"""Host-side checks of the fms-shaped layer (no GPU): parameters, their
shapes and initialisation, and the arguments it rejects."""

import pytest
import torch

from telescope_cache_b200.fms_attention import DEFAULT_CACHE_SIZE, DEFAULT_FMAP, MultiHeadAttention, ShortConv1d


def test_parameters_follow_fms_names_and_shapes():
    m = MultiHeadAttention(64, 16, 32, 8, 2, weight_mode="linear", use_kv_short_conv=True, use_sinks=True,
                           use_gate=True, position_mode="relative", relative_dim=4)
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes == {
        "in_proj.weight": (8 * 16 + 2 * 16 + 2 * 32, 64),
        "dense.weight": (64, 8 * 32),
        "w.weight": (2, 64),
        "k_sconv.weight": (2 * 16, 4),
        "v_sconv.weight": (2 * 32, 4),
        "sinks": (8,),
        "gate_proj.weight": (8 * 32, 64),
        "relative_weight": (8 * 4, 64),
        "relative_proj": (4, DEFAULT_CACHE_SIZE),
    }
    assert m.fmap == DEFAULT_FMAP and m.num_summary_levels == 3
    # fms's initialisation: zero conv (identity) and sinks, small projections
    assert torch.count_nonzero(m.k_sconv.weight) == 0 and torch.count_nonzero(m.sinks) == 0
    assert 0 < m.in_proj.weight.std() < 0.05
    u = MultiHeadAttention(64, 16, 16, 4, 4, fused=False)
    assert {n for n, _ in u.named_parameters()} == {"query.weight", "key.weight", "value.weight",
                                                    "dense.weight"}


def test_rejected_arguments():
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, p_dropout=0.1)
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, weight_mode=None)
    with pytest.raises(NotImplementedError):
        MultiHeadAttention(32, 16, 16, 4, 2, position_encoder=object())
    with pytest.raises(ValueError):
        MultiHeadAttention(32, 16, 16, 4, 3)
    with pytest.raises(ValueError):
        MultiHeadAttention(32, 16, 16, 4, 2, position_mode="alibi")
    with pytest.raises(ValueError):
        ShortConv1d(8, 0)


def test_rope_tables_are_kept_and_grown_by_doubling():
    """Decode steps reuse one table (the rotated ring stays current); a longer
    sequence doubles it, and the rows already there do not change."""
    m = MultiHeadAttention(32, 16, 16, 4, 2, position_mode="rope")
    cpu = torch.device("cpu")
    c1, s1 = m._rope_tables(100, cpu)
    c2, _ = m._rope_tables(60, cpu)
    assert c2 is c1 and c1.shape == (100, 8)
    c3, s3 = m._rope_tables(101, cpu)
    assert c3.shape == (200, 8) and torch.equal(c3[:100], c1) and torch.equal(s3[:100], s1)
    c4, _ = m._rope_tables(450, cpu)
    assert c4.shape == (450, 8)
