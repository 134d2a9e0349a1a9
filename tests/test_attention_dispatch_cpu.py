"""Attention kernel selection (host logic only; runs on the CPU).

The persistent attention schedules give each CTA a fixed list of work and
launch one CTA per SM. Inside a multi-rank process group collective kernels
run on the same GPU at the same time, so the wrappers fall back to the
per-tile grids there; on one rank the kernels choose by size.
"""
import torch.distributed as dist

from scirs_b200.ops import kernels as K


def test_backward_codes(monkeypatch):
    monkeypatch.setattr(K, "ATTN_BWD_IMPL", "tcgen05_auto")
    monkeypatch.setattr(dist, "is_initialized", lambda: False)
    assert K._bwd_code() == 4 and K._fwd_persist() == -1
    assert K._bwd_code(sparse=True) == 4  # the C++ side keeps sparse patterns on the per-tile grid
    monkeypatch.setattr(K, "ATTN_BWD_IMPL", "mma")
    assert K._bwd_code() == 0 and K._bwd_code(sparse=True) == 1
    monkeypatch.setattr(K, "ATTN_BWD_IMPL", "nope")
    try:
        K._bwd_code()
        raise AssertionError("unknown implementation accepted")
    except ValueError:
        pass


def test_multi_rank_uses_per_tile_grids(monkeypatch):
    monkeypatch.setattr(K, "ATTN_BWD_IMPL", "tcgen05_auto")
    monkeypatch.setattr(dist, "is_initialized", lambda: True)
    monkeypatch.setattr(dist, "get_world_size", lambda *a, **k: 2)
    assert K._bwd_code() == 2 and K._fwd_persist() == 0
    monkeypatch.setattr(dist, "get_world_size", lambda *a, **k: 1)
    assert K._bwd_code() == 4 and K._fwd_persist() == -1
