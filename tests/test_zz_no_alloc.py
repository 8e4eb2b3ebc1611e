"""GPU: the allocation-free split-K product (ne_gemm_splitk_noalloc).

Callers that cannot allocate device memory (allocator hooks, plug-ins whose
host process owns every device allocation, start-up code) call this entry
point; it keeps its split-K partial slabs in a static device array of the
library instead of allocating them.  This test calls it through the C ABI
several times in a row, with different shapes and data so that each call runs
over the array the previous one left behind, and compares each result with the
existing entry point ne_gemm_device (epilogue 1) and with a float64 product of
the same bf16 inputs, within the GEMM tests' tolerance.  One case fills the
array exactly and runs on CTA-pair tiles; a request one float larger is
refused; free device memory is the same before and after a repeated call.
The file sorts last so that a run stopping at the first failure has already
run every other test.
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


LIMIT = 2 * 1024 * 1024   # NE_NOALLOC_SCRATCH_FLOATS

# (M, N, K, splits, seed): 128-wide single-CTA tiles, 64-wide tiles, and
# 256 x 256 CTA-pair tiles whose 16 slabs fill the array exactly
CASES = [(512, 48, 1024, 4, 1), (256, 96, 512, 2, 7), (512, 256, 1024, 16, 11)]


def test_noalloc_matches_existing_entry_point_and_float64():
    import neural_engine_b200 as ne
    fn = _noalloc_fn()
    assert CASES[-1][0] * CASES[-1][1] * CASES[-1][3] == LIMIT
    eng = ne.Engine(ne.ModelConfig(1, 128, 256, 2, 2, 64, 256))
    stream = torch.cuda.current_stream().cuda_stream
    try:
        for (M, N, K, splits, seed) in CASES:
            a, b = _bf16((M, K), seed, 0.05), _bf16((N, K), seed + 1)
            da, db = a.cuda(), b.cuda()
            got = torch.full((M, N), float("nan"), device="cuda")
            st = fn(da.data_ptr(), K, M, db.data_ptr(), K, N, K, splits, got.data_ptr(), N, stream)
            assert st == 0, f"ne_gemm_splitk_noalloc returned {st}"
            want = torch.full((M, N), float("nan"), device="cuda")
            eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 1, want.data_ptr(), N)
            eng.sync()
            torch.cuda.synchronize()
            tol = _tol(a, b, K)
            err = (got.double() - want.double()).abs().max().item()
            assert err <= tol, (M, N, K, splits, err)
            ref = a.double() @ b.double().T          # independent of the tcgen05 kernel
            err64 = (got.double().cpu() - ref).abs().max().item()
            assert err64 <= tol, (M, N, K, splits, err64)
    finally:
        eng.close()


def test_noalloc_allocates_nothing_on_a_repeated_call():
    fn = _noalloc_fn()
    M, N, K, splits, seed = CASES[0]
    a, b = _bf16((M, K), seed, 0.05).cuda(), _bf16((N, K), seed + 1).cuda()
    out = torch.empty((M, N), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # the first call may load the library's kernels (lazy module loading)
    assert fn(a.data_ptr(), K, M, b.data_ptr(), K, N, K, splits, out.data_ptr(), N, stream) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert fn(a.data_ptr(), K, M, b.data_ptr(), K, N, K, splits, out.data_ptr(), N,
                  stream) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_requests_beyond_the_scratch_array():
    fn = _noalloc_fn()
    a = torch.zeros((4096, 64), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((4096, 1024), device="cuda")
    # 4096 * 1024 floats > the 2 Mi-float array: refused before any GPU work
    st = fn(a.data_ptr(), 64, 4096, a.data_ptr(), 64, 1024, 64, 1, out.data_ptr(), 1024, None)
    assert st == 1  # NE_ERR_INVALID
    # one float beyond the array: a single-row product of LIMIT + 1 columns
    st = fn(a.data_ptr(), 64, 1, a.data_ptr(), 64, LIMIT + 1, 64, 1, out.data_ptr(), LIMIT + 1,
            None)
    assert st == 1
    # exactly at the limit the size check passes (here a bad row pitch is what
    # is refused, still before any GPU work)
    st = fn(a.data_ptr(), 60, 1, a.data_ptr(), 64, LIMIT, 64, 1, out.data_ptr(), LIMIT, None)
    assert st == 1
