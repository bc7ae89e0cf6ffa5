"""The device closed forms (the ones every kernel evaluates) are bit-exact
with the reference's range tables on every golden schedule."""

import ctypes

import numpy as np
import pytest
import torch

import cases as C
from oracle_runner import load_golden
from telescope_cache_b200 import _lib
from telescope_cache_b200 import range_spec as R

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sched", [s[0] for s in C.SCHEDULES])
def test_device_bounds_match_reference(sched):
    name, N, cache, fmap = next(s for s in C.SCHEDULES if s[0] == sched)
    g = load_golden("sched_" + name)
    ns = R.native_schedule(R.RangeSpec.from_fmap(fmap, cache, N))
    qs = torch.from_numpy(g["qs"].astype(np.int32)).cuda()
    out = torch.full((len(qs), ns.num_levels, 2), -7, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().tc_range_bounds_device(ctypes.byref(ns), _lib.ptr(qs), len(qs),
                                                 _lib.ptr(out), _lib.stream_of(qs)),
               "tc_range_bounds_device")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), g["bounds"]), name
