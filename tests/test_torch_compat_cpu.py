"""replace_linear_modules / FusedQKVProjection surface on CPU (reference
tests/test_replace_threshold.py and test_fused_qkv.py): host-resident
weights build BPositLinear without touching the GPU."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
nn = torch.nn

from mosyne_bposit.torch_compat import (BPositLinear, FusedQKVProjection,  # noqa: E402
                                        replace_linear_modules)


class _ToyAttention(nn.Module):
    def __init__(self, hidden=256, kv_dim=64):
        super().__init__()
        self.q_proj = nn.Linear(hidden, hidden, bias=False)
        self.k_proj = nn.Linear(hidden, kv_dim, bias=False)
        self.v_proj = nn.Linear(hidden, kv_dim, bias=False)
        self.o_proj = nn.Linear(hidden, hidden, bias=False)


class _ToyFFN(nn.Module):
    def __init__(self, hidden=256, ffn_dim=896):
        super().__init__()
        self.gate_proj = nn.Linear(hidden, ffn_dim, bias=False)
        self.up_proj = nn.Linear(hidden, ffn_dim, bias=False)
        self.down_proj = nn.Linear(ffn_dim, hidden, bias=False)


class _ToyBlock(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = _ToyAttention()
        self.mlp = _ToyFFN()


def _count(model, cls):
    return sum(1 for m in model.modules() if isinstance(m, cls) and not (
        cls is nn.Linear and isinstance(m, BPositLinear)))


def test_threshold_none_replaces_everything():
    b = _ToyBlock()
    n = _count(b, nn.Linear)
    replace_linear_modules(b)
    assert _count(b, BPositLinear) == n and _count(b, nn.Linear) == 0


def test_threshold_skips_narrow_n():
    b = _ToyBlock()
    replace_linear_modules(b, narrow_n_threshold=128)
    assert not isinstance(b.attn.k_proj, BPositLinear)
    assert not isinstance(b.attn.v_proj, BPositLinear)
    for m in (b.attn.q_proj, b.attn.o_proj, b.mlp.gate_proj, b.mlp.up_proj, b.mlp.down_proj):
        assert isinstance(m, BPositLinear)


def test_predicate_threshold_and_kv_compose():
    b = _ToyBlock()
    replace_linear_modules(b, predicate=lambda n, m: n.startswith("attn."), skip_kv_proj=True)
    assert isinstance(b.attn.q_proj, BPositLinear) and isinstance(b.attn.o_proj, BPositLinear)
    assert not isinstance(b.attn.k_proj, BPositLinear) and not isinstance(b.attn.v_proj, BPositLinear)
    assert not isinstance(b.mlp.gate_proj, BPositLinear)
    b = _ToyBlock()
    replace_linear_modules(b, narrow_n_threshold=10, skip_kv_proj=True)
    assert not isinstance(b.attn.k_proj, BPositLinear)
    assert isinstance(b.mlp.down_proj, BPositLinear)
    b = _ToyBlock()
    replace_linear_modules(b, narrow_n_threshold=100_000)
    assert _count(b, BPositLinear) == 0


def test_kv_suffix_match_only():
    class Trap(nn.Module):
        def __init__(self):
            super().__init__()
            self.k_proj_norm = nn.Linear(32, 32, bias=False)
            self.k_proj = nn.Linear(32, 32, bias=False)
    m = Trap()
    replace_linear_modules(m, skip_kv_proj=True)
    assert isinstance(m.k_proj_norm, BPositLinear)
    assert not isinstance(m.k_proj, BPositLinear)


def test_bposit_linear_validation_and_repr():
    with pytest.raises(ValueError, match="2-D"):
        BPositLinear(torch.zeros(4))
    m = BPositLinear(torch.zeros(8, 4), bias=torch.zeros(8))
    assert "path=host-fallback" in repr(m) and "has_bias=True" in repr(m)
    with pytest.raises(ValueError, match="in_features"):
        m(torch.zeros(2, 5))


def test_fused_qkv_construction():
    q, k, v = nn.Linear(64, 64), nn.Linear(64, 16), nn.Linear(64, 16)
    f = FusedQKVProjection.from_separate(q_proj=q, k_proj=k, v_proj=v)
    assert f.out_features == 96 and f._fused.out_features == 96
    with pytest.raises(ValueError, match="bias"):
        FusedQKVProjection.from_separate(q_proj=q, k_proj=nn.Linear(64, 16, bias=False), v_proj=v)
    with pytest.raises(ValueError, match="in_features mismatch"):
        FusedQKVProjection.from_separate(q_proj=q, k_proj=nn.Linear(32, 16), v_proj=v)
    with pytest.raises(ValueError):
        FusedQKVProjection(0, 1, 1, 1)
    with pytest.raises(RuntimeError, match="from_separate"):
        FusedQKVProjection(4, 4, 4, 4)(torch.zeros(1, 4))
