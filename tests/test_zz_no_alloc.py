"""GPU: the allocation-free split-K product (ne_gemm_splitk_noalloc).

Callers that cannot allocate device memory (allocator hooks, plug-ins whose
host process owns every device allocation, start-up code) call this entry
point; it keeps its split-K partial slabs in a static device array of the
library instead of allocating them.  This test calls it through the C ABI
twice in a row, with different shapes and data so that the second call runs
over the array the first one left behind, and compares each result with the
existing entry point ne_gemm_device (epilogue 1) on the same inputs, within
the GEMM tests' tolerance.  The file sorts last so that a run stopping at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _tol(a, b, K):
    # same bound as tests/test_gpu_gemm.py
    return 4 * 2e-5 * np.sqrt(K) * float(a.float().abs().max()) * float(b.float().abs().max())


def _noalloc_fn():
    import neural_engine_b200 as ne
    lib = ne.load_library()
    fn = lib.ne_gemm_splitk_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                   ctypes.c_longlong, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_matches_existing_entry_point_twice():
    import neural_engine_b200 as ne
    fn = _noalloc_fn()
    eng = ne.Engine(ne.ModelConfig(1, 128, 256, 2, 2, 64, 256))
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for (M, N, K, splits, seed) in [(512, 48, 1024, 4, 1), (256, 96, 512, 2, 7)]:
            a, b = _bf16((M, K), seed, 0.05), _bf16((N, K), seed + 1)
            da, db = a.cuda(), b.cuda()
            got = torch.full((M, N), float("nan"), device="cuda")
            st = fn(da.data_ptr(), K, M, db.data_ptr(), K, N, K, splits, got.data_ptr(), N, stream)
            assert st == 0, f"ne_gemm_splitk_noalloc returned {st}"
            want = torch.full((M, N), float("nan"), device="cuda")
            eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 1, want.data_ptr(), N)
            eng.sync()
            torch.cuda.synchronize()
            err = (got.double() - want.double()).abs().max().item()
            assert err <= _tol(a, b, K), (M, N, K, splits, err)
    finally:
        eng.close()


def test_noalloc_rejects_requests_beyond_the_scratch_array():
    fn = _noalloc_fn()
    a = torch.zeros((4096, 64), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((4096, 1024), device="cuda")
    # 4096 * 1024 floats > the 2 Mi-float array: refused before any GPU work
    st = fn(a.data_ptr(), 64, 4096, a.data_ptr(), 64, 1024, 64, 1, out.data_ptr(), 1024, None)
    assert st == 1  # NE_ERR_INVALID
