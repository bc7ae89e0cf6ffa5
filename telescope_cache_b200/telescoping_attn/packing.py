"""Packed level-major K/V (reference ``telescoping_attn/packing.py`` /
``reference.py:587-668``): ``[L0 | L1 | ... | LL]`` along the sequence axis,
``level_offsets[l] = sum_{j<l} N_j``, BSHD layout [B, sumN, Hkv, D]."""

from typing import List, NamedTuple, Tuple

import torch


class PackedKV(NamedTuple):
    k: torch.Tensor                 # [B, sumN, Hkv, Dk]
    v: torch.Tensor                 # [B, sumN, Hkv, Dv]
    level_offsets: Tuple[int, ...]  # len num_levels + 1, from the tensors


def _packed_parent(levels):
    """The packed buffer the levels are consecutive views of (as written by
    build_dyadic_summaries), or None."""
    tag = getattr(levels[0], "_tc_packed", None)
    if tag is None or tag[1] != 0 or len(tag[2]) != len(levels) + 1:
        return None
    parent = tag[0]
    for lv, t in enumerate(levels):
        tg = getattr(t, "_tc_packed", None)
        if tg is None or tg[0] is not parent or tg[1] != lv:
            return None
        if t.data_ptr() != parent[:, tg[2][lv]:].data_ptr() or t.shape[1] != tg[2][lv + 1] - tg[2][lv]:
            return None
    return parent


def pack_levels(k_levels: List[torch.Tensor], v_levels: List[torch.Tensor]) -> PackedKV:
    """One level-major buffer per tensor with offsets taken from the tensors
    (reference.py:604-640).  Levels produced by build_dyadic_summaries
    already live in one buffer and are returned without a copy; anything
    else is concatenated on its device."""
    if len(k_levels) != len(v_levels) or not k_levels:
        raise ValueError("k_levels and v_levels must be nonempty, same length")
    B, _, Hkv, Dk = k_levels[0].shape
    Dv = v_levels[0].shape[-1]
    device = k_levels[0].device
    k_dtype, v_dtype = k_levels[0].dtype, v_levels[0].dtype
    offsets = [0]
    for level, (k_l, v_l) in enumerate(zip(k_levels, v_levels)):
        if k_l.shape[1] != v_l.shape[1]:
            raise ValueError(f"level {level}: K length {k_l.shape[1]} != V length {v_l.shape[1]}")
        if k_l.shape[0] != B or v_l.shape[0] != B:
            raise ValueError(f"level {level}: batch mismatch")
        if k_l.shape[2] != Hkv or v_l.shape[2] != Hkv:
            raise ValueError(f"level {level}: Hkv mismatch")
        if k_l.shape[-1] != Dk or v_l.shape[-1] != Dv:
            raise ValueError(f"level {level}: head-dim mismatch")
        if k_l.device != device or v_l.device != device:
            raise ValueError(f"level {level}: device mismatch")
        if k_l.dtype != k_dtype or v_l.dtype != v_dtype:
            raise ValueError(f"level {level}: dtype mismatch")
        offsets.append(offsets[-1] + k_l.shape[1])
    kp, vp = _packed_parent(k_levels), _packed_parent(v_levels)
    if kp is None or vp is None:
        kp, vp = torch.cat(k_levels, dim=1), torch.cat(v_levels, dim=1)
    return PackedKV(k=kp, v=vp, level_offsets=tuple(offsets))


def _packed_slice(packed: PackedKV, level: int, k_start: int, k_end: int) -> Tuple[int, int]:
    """Level-local [k_start, k_end) -> physical rows of the packed buffer
    (reference.py:643-660)."""
    lo = packed.level_offsets[level]
    hi = packed.level_offsets[level + 1]
    assert 0 <= k_start <= k_end <= hi - lo, (level, k_start, k_end, hi - lo)
    return lo + k_start, lo + k_end


__all__ = ["PackedKV", "pack_levels"]
