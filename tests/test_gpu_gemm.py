"""GPU: the tcgen05 GEMM (ne_gemm_device) against a float64 reference.

Operands are bf16 (exactly representable inputs), accumulation fp32 on the
tensor cores; the reference is float64 on the CPU of the same bf16 values.
Tolerance: max |err| <= 2e-5 * sqrt(K) * max|A| * max|B| * 4 (fp32 summation
error bound scale), well below one bf16 ulp of the result.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    import neural_engine_b200 as ne
    cfg = ne.ModelConfig(1, 128, 256, 2, 2, 64, 256)
    e = ne.Engine(cfg)
    yield e
    e.close()


def _bf16(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


def _ref(a, b):
    return (a.double() @ b.double().T)


def _tol(a, b, K):
    return 4 * 2e-5 * np.sqrt(K) * float(a.float().abs().max()) * float(b.float().abs().max())


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (300, 200, 192),
                                   (1000, 16, 128), (64, 40, 256), (513, 300, 320)])
def test_gemm_f32_rowmajor(eng, M, N, K):
    a, b = _bf16((M, K), 1), _bf16((N, K), 2)
    da, db = a.cuda(), b.cuda()
    out = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 1, out.data_ptr(), N)
    eng.sync()
    ref = _ref(a, b)
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= _tol(a, b, K), err


@pytest.mark.parametrize("M,N,K", [(4096, 1, 1024), (1024, 5, 2048), (512, 32, 1024),
                                   (384, 256, 256), (640, 100, 64)])
def test_gemm_f32_transposed_decode(eng, M, N, K):
    """swap-AB: A = weight [M, K], B = activations [N, K]; out[n*ld + m]."""
    w, x = _bf16((M, K), 3, 0.05), _bf16((N, K), 4)
    dw, dx = w.cuda(), x.cuda()          # keep the device tensors alive during the call
    out = torch.full((N, M), float("nan"), device="cuda")
    eng.gemm_device(dw.data_ptr(), K, M, dx.data_ptr(), K, N, K, 0, out.data_ptr(), M)
    eng.sync()
    ref = _ref(w, x).T
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= _tol(w, x, K), err


def test_gemm_bf16_out(eng):
    M, N, K = 384, 512, 512
    a, b = _bf16((M, K), 5), _bf16((N, K), 6, 0.1)
    da, db = a.cuda(), b.cuda()
    out = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 2, out.data_ptr(), N)
    eng.sync()
    ref = _ref(a, b)
    # bf16 rounding of the result: half an ulp (2^-8 relative) plus accumulation
    rel = ((out.cpu().double() - ref).abs() / (ref.abs() + 1e-3)).max().item()
    assert rel <= 2 ** -8 + 1e-3, rel


def test_gemm_residual_epilogue(eng):
    M, N, K = 257, 384, 256
    a, b = _bf16((M, K), 7), _bf16((N, K), 8, 0.1)
    x0 = torch.randn(M, N)
    x = x0.clone().cuda()
    alpha = 0.25
    da, db = a.cuda(), b.cuda()
    eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 3, x.data_ptr(), N, alpha)
    eng.sync()
    ref = x0.double() + alpha * _ref(a, b)
    err = (x.cpu().double() - ref).abs().max().item()
    assert err <= _tol(a, b, K), err


def test_gemm_swiglu_epilogue(eng):
    """B = [W1/W3 interleaved in 16-row blocks]; out[m, j] = silu(h1_j) * h3_j."""
    M, F, K = 200, 256, 128
    a = _bf16((M, K), 9)
    w1, w3 = _bf16((F, K), 10, 0.1), _bf16((F, K), 11, 0.1)
    w13 = torch.empty((2 * F, K), dtype=torch.bfloat16)
    for c in range(F // 16):
        w13[32 * c:32 * c + 16] = w1[16 * c:16 * c + 16]
        w13[32 * c + 16:32 * c + 32] = w3[16 * c:16 * c + 16]
    out = torch.zeros((M, F), dtype=torch.bfloat16, device="cuda")
    da, dw = a.cuda(), w13.cuda()
    eng.gemm_device(da.data_ptr(), K, M, dw.data_ptr(), K, 2 * F, K, 4, out.data_ptr(), F)
    eng.sync()
    h1, h3 = _ref(a, w1), _ref(a, w3)
    ref = h1 * (1.0 / (1.0 + torch.exp(-h1))) * h3
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= 2 ** -8 * ref.abs().max().item() + 1e-3, err


def test_gemm_rejects_bad_k(eng):
    import neural_engine_b200 as ne
    a = torch.zeros((128, 100), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((128, 128), device="cuda")
    with pytest.raises(ne.NeError):
        eng.gemm_device(a.data_ptr(), 100, 128, a.data_ptr(), 100, 128, 100, 1, out.data_ptr(), 128)


@pytest.mark.parametrize("bn", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("epi", [0, 1])
def test_gemm_every_tile_width(eng, bn, epi):
    M, N, K = 320, 72, 512
    a, b = _bf16((M, K), 12, 0.05), _bf16((N, K), 13)
    da, db = a.cuda(), b.cuda()
    shape, ld = ((N, M), M) if epi == 0 else ((M, N), N)
    out = torch.full(shape, float("nan"), device="cuda")
    eng.gemm_device_ex(da.data_ptr(), K, M, db.data_ptr(), K, N, K, epi, out.data_ptr(), ld, 1.0,
                       bn, 1, 0)
    eng.sync()
    o = out.cpu().double()
    if epi == 0:
        o = o.T
    err = (o - _ref(a, b)).abs().max().item()
    assert err <= _tol(a, b, K), err


@pytest.mark.parametrize("splits", [2, 4, 8])
def test_gemm_split_k_slabs(eng, splits):
    """Split-K partial slabs sum to the product (the decode path reduces them
    in its consumer kernels in a fixed order)."""
    M, N, K = 1024, 24, 2048
    a, b = _bf16((M, K), 14, 0.05), _bf16((N, K), 15)
    da, db = a.cuda(), b.cuda()
    out = torch.zeros((splits, N, M), device="cuda")
    used = eng.gemm_device_ex(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 0, out.data_ptr(), M,
                              1.0, 0, splits, N * M)
    eng.sync()
    assert used == splits
    o = out.sum(0).cpu().double().T
    err = (o - _ref(a, b)).abs().max().item()
    assert err <= _tol(a, b, K), err
