"""The C-ABI library: loads, exports every declared symbol, and rejects bad arguments with
status codes before touching the GPU.  CPU only (no kernel is launched)."""
import ctypes
import os
import re

import pytest

from fathom_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "fathom_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fathom_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 15
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert L.fathom_abi_version() == 2


def test_null_and_shape_errors_are_status_codes():
    L = _lib.lib()
    assert L.fathom_scan(None, 1, 4, 100, 16, None, None, 4, None, None, 0, 2, None, None) == _lib.FATHOM_ERR_NULL
    assert b"NULL" in L.fathom_last_error()
    p = ctypes.c_void_p(16)          # never dereferenced: validation fails first
    assert L.fathom_scan(p, 1, 9, 100, 16, p, p, 4, p, p, 0, 2, p, None) == _lib.FATHOM_ERR_UNSUPPORTED
    assert L.fathom_scan(p, 1, 4, 100, 16, p, p, 4, p, p, 0, 3, p, None) == _lib.FATHOM_ERR_SHAPE
    assert L.fathom_make_plan(p, p, 4, 5, 30, p, p, p, p, p, p, p, None) == _lib.FATHOM_ERR_SHAPE
    assert L.fathom_sink_local_topk(p, 1, 100, 10, 4, 6, p, p, 1 << 20, None) == _lib.FATHOM_ERR_SHAPE
    need = L.fathom_select_workspace_bytes(4, 1000, 10)
    assert need >= 512
    # 256 bytes hold neither the group keys (4 rows x 32 groups) nor the histogram path's buffers
    assert L.fathom_select_topk(p, 4, 1000, 1000, 10, 0, 1000, 0, p, 10, None, ctypes.c_void_p(256), 256,
                                None) == _lib.FATHOM_ERR_WORKSPACE
    assert L.fathom_merge_topk(p, p, 1, 9000, 10, p, None, None) == _lib.FATHOM_ERR_SHAPE
    assert L.fathom_decode_attention(p, 2, 4, p, 20000, p, p, 10, 0, 10, None, None, 0, p, None, p, 1 << 30,
                                     None) == _lib.FATHOM_ERR_UNSUPPORTED
    assert L.fathom_quantise_pack(p, 7, 1, 64, 64 * 128, 16, 1, None, None, 0, None, None, None) == \
        _lib.FATHOM_ERR_UNSUPPORTED
    assert L.fathom_klt_quantise_pack(p, 1, 1, 64, 64 * 128, None, p, 16, 0, None, None, 0, p, p, None,
                                      None) == _lib.FATHOM_ERR_NULL
    assert L.fathom_klt_quantise_pack(p, 1, 1, 64, 64 * 128, p, ctypes.c_void_p(20), 16, 0, None, None, 0, p, p, None,
                                      None) == _lib.FATHOM_ERR_SHAPE
    assert L.fathom_klt_query(p, 2, 9, p, p, p, p, None) == _lib.FATHOM_ERR_UNSUPPORTED
    assert L.fathom_klt_query(p, 2, 4, p, None, p, p, None) == _lib.FATHOM_ERR_NULL
    assert L.fathom_gather_runs(p, None, p, p, p, 4, 100, 64, None) == _lib.FATHOM_ERR_NULL
    assert L.fathom_gather_runs(p, ctypes.c_void_p(20), p, p, p, 4, 100, 64, None) == _lib.FATHOM_ERR_SHAPE
    assert L.fathom_gather_runs(p, p, p, p, p, 4, 1 << 30, 1, None) == _lib.FATHOM_ERR_SHAPE   # > 65535 chunks
    assert L.fathom_stage_planes(p, p, p, 2, 100, 64, 101, p, p, None) == _lib.FATHOM_ERR_SHAPE  # b1 > nblk
    assert L.fathom_stage_planes(p, p, None, 2, 100, 0, 64, p, p, None) == _lib.FATHOM_ERR_NULL


def test_chunk_bounds_cover_the_blocks_with_aligned_inner_edges():
    from fathom_b200.offload import chunk_bounds
    assert chunk_bounds(16384, 4) == [(0, 4096), (4096, 8192), (8192, 12288), (12288, 16384)]
    assert chunk_bounds(1094, 3) == [(0, 320), (320, 704), (704, 1094)]
    assert chunk_bounds(100, 8) == [(0, 64), (64, 100)]      # empty chunks dropped
    assert chunk_bounds(79, 1) == [(0, 79)]
    for nblk, parts in ((5000, 7), (64, 3), (16384, 8)):
        b = chunk_bounds(nblk, parts)
        assert b[0][0] == 0 and b[-1][1] == nblk
        assert all(x[1] == y[0] and x[1] % 64 == 0 for x, y in zip(b, b[1:]))


def test_python_layer_rejects_cpu_tensors():
    import torch
    from fathom_b200 import bitplane as bp
    with pytest.raises(ValueError, match="CUDA"):
        bp.quantise_u4(torch.zeros(2, 64, 128))
    with pytest.raises(ValueError, match="CUDA"):
        bp.make_plan(torch.zeros(2, 128), 48.0)
    with pytest.raises(ValueError, match="CUDA"):
        bp.sink_local_topk(torch.zeros(2, 4, 500), 100, 4, 32)
    from fathom_b200 import klt
    basis = klt.KLTBasis(torch.zeros(2, 128), torch.zeros(2, 128, 128), torch.zeros(2, 128))
    with pytest.raises(ValueError, match="CUDA"):
        klt.klt_query(torch.zeros(2, 4, 128), basis)
    with pytest.raises(ValueError, match="CUDA"):
        klt.KLTPlaneStore(torch.zeros(2, 64, 128), basis)


def test_build_entry_compiles_for_sm100a():
    from fathom_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert os.path.exists(_lib.LIB_PATH)
