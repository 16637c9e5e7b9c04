"""The allocation-free top-k entry point (fathom_sink_local_topk_static).

Some callers cannot allocate device memory where they call this library: a host that has handed
all device memory to its own pool, or a decode loop that cannot take the implicit device
synchronisation of cudaMalloc.  For them the library keeps its own scratch array for top-k.  These
tests call that entry point through the C ABI, with only the caller's inputs and outputs, twice in
a row on different inputs (the scratch keeps the previous call's contents), and require the same
indices as fathom_sink_local_topk with a caller workspace.  Indices are compared exactly, as in
the other top-k tests: the selection order is deterministic.

This file sorts last so that a stop-at-first-failure run has already run every other test.
"""
import ctypes

import pytest
import torch

from fathom_b200 import _lib

pytestmark = pytest.mark.gpu


def _with_workspace(L, s, k, sink, local):
    rows, n = s.shape
    idx = torch.empty(rows, k, dtype=torch.int64, device=s.device)
    nbytes = L.fathom_select_workspace_bytes(rows, n, k - sink - local)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=s.device)
    st = torch.cuda.current_stream().cuda_stream
    assert L.fathom_sink_local_topk(s.data_ptr(), rows, n, k, sink, local, idx.data_ptr(), ws.data_ptr(), nbytes,
                                    st) == 0
    return idx


def _static(L, s, k, sink, local):
    rows, n = s.shape
    idx = torch.empty(rows, k, dtype=torch.int64, device=s.device)
    st = torch.cuda.current_stream().cuda_stream
    rc = L.fathom_sink_local_topk_static(s.data_ptr(), rows, n, k, sink, local, idx.data_ptr(), st)
    assert rc == 0, L.fathom_last_error()
    return idx


def test_static_scratch_topk_matches_workspace_variant_twice():
    L = _lib.lib()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(2024)
    first = torch.randn(32, 131072, generator=g, device="cuda")          # Qwen3-8B batch 1: 8 KV heads x G=4
    second = torch.randint(0, 40, (64, 50000), generator=g, device="cuda").float()   # heavy ties, the row limit
    for s, k, sink, local in ((first, 580, 4, 64), (second, 600, 4, 64)):
        got = _static(L, s, k, sink, local)
        torch.cuda.synchronize()
        ref = _with_workspace(L, s, k, sink, local)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


def test_static_scratch_histogram_path_after_group_path():
    """The histogram path, whose counters must start at zero in the shared scratch, right after calls
    that left the scratch dirty: a dense k (too few 32-token groups for the group-key path), and rows
    whose group keys do not fit the scratch (64 x 1M), each compared with the workspace variant."""
    L = _lib.lib()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(77)
    warm = torch.randn(32, 131072, generator=g, device="cuda")
    dense = torch.randn(64, 4096, generator=g, device="cuda")
    big = torch.randn(64, 1 << 20, generator=g, device="cuda")
    for s, k, sink, local in ((warm, 580, 4, 64), (dense, 1500, 4, 64), (warm, 580, 4, 64), (big, 580, 4, 64),
                              (dense, 1500, 4, 64)):
        got = _static(L, s, k, sink, local)
        torch.cuda.synchronize()
        ref = _with_workspace(L, s, k, sink, local)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


def test_static_scratch_call_takes_no_device_memory():
    """Once the library's selection module is loaded on the device (any earlier call), a call takes no
    device memory: the free memory the driver reports is the same before and after it."""
    L = _lib.lib()
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(3)
    s = torch.randn(64, 1 << 20, generator=g, device="cuda")
    idx = torch.empty(64, 580, dtype=torch.int64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.fathom_sink_local_topk_static(s.data_ptr(), 64, 1 << 20, 580, 4, 64, idx.data_ptr(), st) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        assert L.fathom_sink_local_topk_static(s.data_ptr(), 64, 1 << 20, 580, 4, 64, idx.data_ptr(), st) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free0 == free1


def test_static_scratch_rejects_rows_beyond_its_limit():
    L = _lib.lib()
    p = ctypes.c_void_p(256)        # never dereferenced: the row check fails first
    rc = L.fathom_sink_local_topk_static(p, 65, 1000, 100, 4, 32, p, None)
    assert rc == _lib.FATHOM_ERR_SHAPE
    assert b"64" in L.fathom_last_error()
