"""The scratch-free sender-CSR entry point (atom_sender_csr_noalloc).

Some callers cannot allocate device memory -- typically a host MD engine or framework whose own
pool allocator owns the GPU's memory -- so they cannot hand atom_sender_csr its N-int scratch.
The scratch-free variant keeps that scratch in a static device array inside the library. This
test calls it through the C ABI twice in a row on different graphs and checks that each result
equals the allocating entry point's exactly (integer output), which also shows that the shared
array's leftover contents from the first call do not leak into the second.

The file name sorts last so that a run stopping at the first failure has run every other test.
"""

import pytest
import torch

from tt_atom import _lib as L
from tt_atom._lib import call, ptr

pytestmark = pytest.mark.gpu


def _edges(seed, N, E):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, N, (E,), generator=g, dtype=torch.int32).cuda()


def _reference(src, N):
    E = src.numel()
    send_ptr = torch.empty(N + 1, dtype=torch.int32, device="cuda")
    send_eid = torch.empty(max(E, 1), dtype=torch.int32, device="cuda")
    scratch = torch.empty(N, dtype=torch.int32, device="cuda")
    call("atom_sender_csr", ptr(src), E, N, ptr(scratch), ptr(send_ptr), ptr(send_eid),
         L.stream_ptr())
    return send_ptr, send_eid[:E]


def _noalloc(src, N):
    E = src.numel()
    send_ptr = torch.full((N + 1,), -7, dtype=torch.int32, device="cuda")
    send_eid = torch.full((max(E, 1),), -7, dtype=torch.int32, device="cuda")
    call("atom_sender_csr_noalloc", ptr(src), E, N, ptr(send_ptr), ptr(send_eid), L.stream_ptr())
    return send_ptr, send_eid[:E]


def test_noalloc_sender_csr_matches_allocating_entry_point_twice():
    # first call: many nodes; second call: fewer nodes, different edges
    for seed, N, E in [(11, 5000, 150000), (12, 700, 9000)]:
        src = _edges(seed, N, E)
        p_ref, e_ref = _reference(src, N)
        p_new, e_new = _noalloc(src, N)
        torch.cuda.synchronize()
        assert torch.equal(p_new, p_ref)
        assert torch.equal(e_new, e_ref)


def _free_bytes():
    return torch.cuda.mem_get_info()[0]      # cudaMemGetInfo: device-wide free bytes


def test_noalloc_sender_csr_allocates_nothing():
    """The point of the entry point: a call after the first on this device changes the
    device's free memory by not a byte (the first call only looks up the static array)."""
    src = _edges(13, 3000, 60000)
    p, e = _noalloc(src, 3000)          # warm-up: the one-time set-up
    torch.cuda.synchronize()
    before = _free_bytes()
    call("atom_sender_csr_noalloc", ptr(src), src.numel(), 3000, ptr(p), ptr(e), L.stream_ptr())
    torch.cuda.synchronize()
    assert _free_bytes() == before


def test_noalloc_sender_csr_empty_inputs():
    # E = 0: every node's range is empty, send_ptr all zeros
    N = 257
    src = torch.zeros(1, dtype=torch.int32, device="cuda")
    send_ptr = torch.full((N + 1,), -7, dtype=torch.int32, device="cuda")
    send_eid = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    call("atom_sender_csr_noalloc", ptr(src), 0, N, ptr(send_ptr), ptr(send_eid), L.stream_ptr())
    torch.cuda.synchronize()
    assert int(send_ptr.abs().sum()) == 0
    assert int(send_eid[0]) == -7
    # N = 0: nothing to do, nothing written
    call("atom_sender_csr_noalloc", ptr(src), 0, 0, ptr(send_ptr), ptr(send_eid), L.stream_ptr())
    torch.cuda.synchronize()
    assert int(send_ptr.abs().sum()) == 0


def test_noalloc_sender_csr_rejects_oversize():
    src = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(4, dtype=torch.int32, device="cuda")
    rc = L.lib().atom_sender_csr_noalloc(ptr(src), 1, (1 << 20) + 1, ptr(out), ptr(out),
                                         L.stream_ptr())
    assert rc == L.ATOM_ERR_CAPACITY
    assert "exceeds the built-in scratch" in L.last_error()
