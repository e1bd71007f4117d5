"""smoe_moe_group_noalloc: the grouping entry point for callers that cannot allocate device memory.

Callers recording into a CUDA graph, or running under a memory planner that forbids allocation on the token
path, cannot hand smoe_moe_group a scratch buffer; this variant keeps its tables in a static device array.
It must give exactly what smoe_moe_group gives, call after call, although every call reuses the same array.
This file is collected last so that a failure here cannot hide any other test's result.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from stratametal_b200 import api
from stratametal_b200._lib import lib

pytestmark = pytest.mark.gpu


def routing(rng, T, E, k):
    return np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)


def group_with_scratch(ids, T, E, k, dev):
    scratch = torch.empty(api.moe_group_scratch_bytes(T, k, E), dtype=torch.uint8, device=dev)
    slot = torch.empty(T * k, dtype=torch.int32, device=dev)
    src = torch.empty(T * k, dtype=torch.int32, device=dev)
    api.moe_group(ids, T, k, E, scratch, slot, src)
    return slot, src


def group_noalloc(ids, T, E, k, dev):
    slot = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    src = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
    st = lib().smoe_moe_group_noalloc(ids.data_ptr(), T, k, E, slot.data_ptr(), src.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert st == 0, lib().smoe_last_error()
    return slot, src


@pytest.mark.parametrize("T,E,k", [(64, 512, 10), (300, 512, 10), (5, 7, 3), (2, 1024, 64)])
def test_noalloc_matches_scratch_entry_point_twice(cuda, T, E, k):
    rng = np.random.default_rng(T * 1000 + E)
    first = torch.from_numpy(routing(rng, T, E, k)).to(cuda)
    second = torch.from_numpy(routing(rng, T, E, k)).to(cuda)
    for ids in (first, second):            # two calls in a row on the shared static array
        want_slot, want_src = group_with_scratch(ids, T, E, k, cuda)
        got_slot, got_src = group_noalloc(ids, T, E, k, cuda)
        torch.cuda.synchronize()
        assert torch.equal(got_slot, want_slot)
        assert torch.equal(got_src, want_src)
    assert api.device_status() == 0


def test_noalloc_refuses_more_experts_than_its_table(cuda):
    ids = torch.zeros(10, dtype=torch.int32, device=cuda)
    st = lib().smoe_moe_group_noalloc(ids.data_ptr(), 1, 10, 1025, ids.data_ptr(), None,
                                      torch.cuda.current_stream().cuda_stream)
    assert st == 1
    assert b"1024" in lib().smoe_last_error()
