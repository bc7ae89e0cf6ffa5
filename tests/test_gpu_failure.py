"""Failure detection without a GPU fault: a pipeline wait that can never
complete gives up by itself, the device status word reports it, and the
context keeps running the product path afterwards."""

import numpy as np
import pytest
import torch

import telescope_cache_b200 as T
from telescope_cache_b200 import _lib
from telescope_cache_b200.telescoping_attn.attention import device_status, read_device_status

pytestmark = pytest.mark.gpu

TC_DEV_WAIT_TIMEOUT = 1


def test_bounded_wait_gives_up_and_context_survives():
    dev = torch.device("cuda")
    read_device_status(dev)  # clear
    st = device_status(dev)
    rc = _lib.lib().tc_selftest_wait_timeout(st.data_ptr(), _lib.stream_of(st))
    assert rc == 0
    assert read_device_status(dev) & TC_DEV_WAIT_TIMEOUT
    assert read_device_status(dev) == 0  # cleared by the read
    # the same context still runs the tensor-core forward correctly
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    B, N, H, D = 1, 256, 2, 128
    q, k, v = (torch.randn(B, N, H, D, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(3))
    fmap, cache = {1: 32, 2: 64}, 96
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, 2)
    out, lse = T.multilevel_attention_forward(q, T.pack_levels(kl, vl), fmap, cache, softcap=20.0)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    assert read_device_status(dev) == 0
    # and the same call again agrees bit for bit
    out2, lse2 = T.multilevel_attention_forward(q, T.pack_levels(kl, vl), fmap, cache, softcap=20.0)
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
