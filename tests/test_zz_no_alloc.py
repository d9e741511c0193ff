"""The allocation-free routing entry point, bokt_moe_route_noalloc.

It serves callers that cannot allocate device memory (everything is owned by
another allocator, a foreign runtime has no device allocator, or allocation
is forbidden in the calling loop), so it keeps its scratch in a fixed device
array inside the library.  This file is collected last on purpose: it runs
after every other test, and must also pass alone in a fresh process.

Both calls go straight through the C ABI (ctypes), with the caller's own
pre-allocated output tensors, and are compared with bokt_moe_route (the
workspace entry point) on the same ids: integer outputs, so the tolerance is
exact equality, as in every routing test.
"""

import ctypes

import numpy as np
import pytest
import torch

from flashattentionanycard_b200 import _native
from flashattentionanycard_b200.workloads import zipf_routing

pytestmark = pytest.mark.gpu


def _outputs(a, e, device):
    i32 = dict(device=device, dtype=torch.int32)
    return (torch.full((e,), -1, **i32), torch.full((e + 1,), -1, **i32),
            torch.full((e + 1,), -1, device=device, dtype=torch.int64),
            torch.full((a,), -1, **i32), torch.full((a,), -1, **i32))


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _route_with_workspace(lib, ids, e, device):
    a = ids.numel()
    counts, offsets, offsets64, perm, inv = _outputs(a, e, device)
    nbytes = max(int(lib.bokt_moe_route_workspace_bytes(a, e)), 4)
    workspace = torch.empty(nbytes // 4, device=device, dtype=torch.int32)
    _native.check(lib.bokt_moe_route(ids.data_ptr(), a, e, counts.data_ptr(), offsets.data_ptr(),
                                     offsets64.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                     workspace.data_ptr(), workspace.numel() * 4, _stream(device)),
                  "bokt_moe_route")
    return counts, offsets, offsets64, perm, inv


def _route_noalloc(lib, ids, e, device):
    a = ids.numel()
    counts, offsets, offsets64, perm, inv = _outputs(a, e, device)
    _native.check(lib.bokt_moe_route_noalloc(ids.data_ptr(), a, e, counts.data_ptr(),
                                             offsets.data_ptr(), offsets64.data_ptr(),
                                             perm.data_ptr(), inv.data_ptr(), _stream(device)),
                  "bokt_moe_route_noalloc")
    return counts, offsets, offsets64, perm, inv


def test_noalloc_route_matches_workspace_route_twice_in_a_row(cuda_device):
    lib = _native.load()
    _native.device_status(reset=True)
    # Two calls in a row on different inputs: the second call runs on scratch
    # that still holds the first call's contents.
    cases = [(zipf_routing(16384, 64, 2, 1.1, 11).reshape(-1), 64),
             (zipf_routing(5000, 200, 2, 1.1, 12).reshape(-1), 200)]
    for ids_cpu, experts in cases:
        ids = ids_cpu.to(cuda_device)
        got = _route_noalloc(lib, ids, experts, cuda_device)
        want = _route_with_workspace(lib, ids, experts, cuda_device)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert torch.equal(g, w)
        counts = np.bincount(ids_cpu.numpy(), minlength=experts)
        assert np.array_equal(got[0].cpu().numpy(), counts)
        assert np.array_equal(got[3].cpu().numpy(), np.argsort(ids_cpu.numpy(), kind="stable"))
    assert _native.device_status(reset=True)[0] == 0


def test_noalloc_route_rejects_requests_beyond_its_array(cuda_device):
    lib = _native.load()
    limit = int(lib.bokt_moe_route_noalloc_max_words())
    assert limit == 65536
    e = 1024
    a = (limit // e + 1) * 4096  # one chunk too many
    rc = lib.bokt_moe_route_noalloc(None, a, e, None, None, None, None, None, None)
    assert rc == 1  # null outputs are rejected before the size check
    ids = torch.zeros(a, device=cuda_device, dtype=torch.int32)
    counts, offsets, offsets64, perm, inv = _outputs(a, e, cuda_device)
    rc = lib.bokt_moe_route_noalloc(ids.data_ptr(), a, e, counts.data_ptr(), offsets.data_ptr(),
                                    None, perm.data_ptr(), inv.data_ptr(), _stream(cuda_device))
    assert rc == 2
    assert b"exceeds the fixed" in lib.bokt_last_error()
