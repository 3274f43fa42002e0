"""Host-side checks of the C ABI that need no GPU: the library loads, exports
every entry point include/mrt_b200.h declares, validates arguments before
touching the device, and its tensor-parallel shard map is right."""
import ctypes as C

import numpy as np
import pytest

from mruntime_b200 import capi


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    declared = capi.header_functions()
    assert len(declared) >= 25
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    assert lib.mrt_version() == 100


def test_ctypes_signatures_cover_header():
    assert set(capi.header_functions()) == set(capi._SIGS)


def test_argument_errors_before_device_work():
    lib = capi.lib()
    h = C.c_void_p()
    rc = lib.mrt_weight_upload(None, 0, 0, 4, 4, None, 0, 0, 4, None, C.byref(h))
    assert rc == 1 and b"NULL" in lib.mrt_last_error_string()
    buf = np.zeros(16, np.uint16)
    rc = lib.mrt_weight_upload(buf.ctypes.data, 7, 0, 4, 4, None, 0, 0, 4, None, C.byref(h))
    assert rc == 3  # bad dtype
    rc = lib.mrt_weight_upload(buf.ctypes.data, 0, 0, 4, 4, None, 0, 2, 9, None, C.byref(h))
    assert rc == 2  # bad column range
    rr = (C.c_int64 * 2)(3, 9)
    rc = lib.mrt_weight_upload(buf.ctypes.data, 0, 0, 4, 4, rr, 1, 0, 4, None, C.byref(h))
    assert rc == 2  # row range outside [0, N)
    assert lib.mrt_gemm(None, None, 0, None, 0, 1, 0, None) == 1
    assert lib.mrt_gemm_general(None, 9, 1, 1, None, 0, 1, 1, None, 0, 1.0, 0.0, 0, 0, None) == 3
    assert lib.mrt_gemm_general(None, 0, 2, 3, None, 0, 4, 5, None, 0, 1.0, 0.0, 0, 1, None) == 2
    assert lib.mrt_argmax_f16(None, 1, 10, 5, 0, None, None, None) == 2
    assert lib.mrt_convert(None, 0, None, 5, 1, None) == 3


def test_no_gpu_reports_cuda_error_not_crash():
    import torch

    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    with pytest.raises(capi.MrtError) as ei:
        capi.init(0)
    assert ei.value.code == 4


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_rows_partitions_every_part(world):
    parts = [3584, 512, 512]  # fused q,k,v of the 7B shape
    seen = [np.zeros(p, bool) for p in parts]
    for rank in range(world):
        ranges = capi.shard_rows(parts, world, rank)
        off = 0
        for p, (b, e) in enumerate(ranges):
            assert off <= b < e <= off + parts[p]
            assert e - b == parts[p] // world  # these sizes divide evenly
            seen[p][b - off:e - off] = True
            off += parts[p]
    assert all(s.all() for s in seen)


@pytest.mark.parametrize("K,world", [(3584, 8), (18944, 8), (896, 2), (4864, 4), (100, 3)])
def test_shard_cols_partitions_k(K, world):
    spans = [capi.shard_cols(K, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == K
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 < a1
    if K % (8 * world) == 0:
        assert all((b - a) % 8 == 0 for a, b in spans)


def test_shard_rejects_bad_rank():
    with pytest.raises(capi.MrtError):
        capi.shard_rows([16], 2, 2)
    with pytest.raises(capi.MrtError):
        capi.shard_cols(4, 8, 0)
