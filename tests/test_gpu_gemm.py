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


@pytest.mark.parametrize("M,N,K,mn", [(600, 300, 320, 0), (1300, 520, 256, 0), (4096, 1024, 1024, 0),
                                      (600, 296, 320, 1), (1024, 768, 512, 2)])
@pytest.mark.parametrize("epi", [1, 2, 3])
def test_gemm_cta_pair_tiles(eng, M, N, K, mn, epi):
    """M >= 512 with 256-wide tiles runs on CTA pairs (cta_group::2: one MMA
    over two SMs, each CTA holding half of A's and half of B's rows): ragged M
    and N (the odd CTA's rows or B-half past the end), K-major and MN-major
    operands (mn 1: B MN-major, 2: both), fp32 / bf16 / residual outputs."""
    if mn == 2:
        at, bt = _bf16((K, M), 41, 0.1), _bf16((K, N), 42, 0.1)
        a, b = at.T, bt.T
        da, db = at.cuda(), bt.cuda()
        lda, ldb, a_mn, b_mn = M, N, 1, 1
    elif mn == 1:
        a, bt = _bf16((M, K), 41), _bf16((K, N), 42, 0.1)
        b = bt.T
        da, db = a.cuda(), bt.cuda()
        lda, ldb, a_mn, b_mn = K, N, 0, 1
    else:
        a, b = _bf16((M, K), 41), _bf16((N, K), 42, 0.1)
        da, db = a.cuda(), b.cuda()
        lda, ldb, a_mn, b_mn = K, K, 0, 0
    if mn == 2 and epi != 3:
        pytest.skip("MN/MN products accumulate (dW)")
    x0 = torch.randn(M, N)
    if epi == 2:
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    elif epi == 3:
        out = x0.clone().cuda()
    else:
        out = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm(da.data_ptr(), lda, M, db.data_ptr(), ldb, N, K, epi, out.data_ptr(), N,
             alpha=0.5 if epi == 3 else 1.0, a_mn=a_mn, b_mn=b_mn, bn=256)
    eng.sync()
    ref = a.double() @ b.double().T
    if epi == 3:
        ref = x0.double() + 0.5 * ref
    got = out.cpu().double()
    tol = _tol(a, b, K) + (float(ref.abs().max()) * 2 ** -8 if epi == 2 else 0.0)
    err = (got - ref).abs().max().item()
    assert err <= tol, (err, tol)


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
    # with a second output the raw projection is saved too (bf16, same interleaved columns)
    h13 = torch.zeros((M, 2 * F), dtype=torch.bfloat16, device="cuda")
    out2 = torch.zeros_like(out)
    eng.gemm(da.data_ptr(), K, M, dw.data_ptr(), K, 2 * F, K, 4, out2.data_ptr(), F,
             aux0=h13.data_ptr())
    eng.sync()
    assert torch.equal(out2, out)
    raw = _ref(a, w13)
    assert (h13.cpu().double() - raw).abs().max().item() <= 2 ** -8 * raw.abs().max().item()


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


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("M,N,K", [(256, 384, 256), (320, 200, 128), (1024, 64, 512)])
def test_gemm_mn_major_b(eng, bn, M, N, K):
    """dX-style product: B read MN-major from a [K, N] row-major matrix."""
    a, bt = _bf16((M, K), 21), _bf16((K, N), 22, 0.1)      # bt = B^T stored [K, N]
    da, db = a.cuda(), bt.cuda()
    out = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm(da.data_ptr(), K, M, db.data_ptr(), N, N, K, 1, out.data_ptr(), N, b_mn=1, bn=bn)
    eng.sync()
    ref = a.double() @ bt.double()
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= _tol(a, bt, K), err


@pytest.mark.parametrize("bn", [64, 256])
@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (384, 192, 320), (1024, 128, 2048)])
def test_gemm_mn_major_both(eng, bn, M, N, K):
    """dW-style product: A [K, M] and B [K, N] both read MN-major (token-major
    activations), accumulated into fp32 (epi 3)."""
    at, bt = _bf16((K, M), 23, 0.1), _bf16((K, N), 24, 0.1)
    da, db = at.cuda(), bt.cuda()
    x0 = torch.randn(M, N)
    out = x0.clone().cuda()
    eng.gemm(da.data_ptr(), M, M, db.data_ptr(), N, N, K, 3, out.data_ptr(), N, alpha=0.5,
             a_mn=1, b_mn=1, bn=bn)
    eng.sync()
    ref = x0.double() + 0.5 * (at.double().T @ bt.double())
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= _tol(at, bt, K), err


def test_gemm_swiglu_backward_epilogue(eng):
    """d_gate = dY . W2 (W2 read MN-major) with the SwiGLU-backward epilogue."""
    M, F, D = 192, 256, 128
    dy = _bf16((M, D), 25)
    w2 = _bf16((D, F), 26, 0.1)          # W2 [D, F]: MN-major B for d_gate = dY W2
    h1, h3 = _bf16((M, F), 27), _bf16((M, F), 28)
    # the forward saves h1 / h3 interleaved in 16-feature blocks: (h1 x16 | h3 x16) ...
    h13 = torch.stack([h1.reshape(M, F // 16, 16), h3.reshape(M, F // 16, 16)], 2).reshape(M, 2 * F)
    ddy, dw2, dh13 = dy.cuda(), w2.cuda(), h13.cuda()
    out = torch.zeros((M, 2 * F), dtype=torch.bfloat16, device="cuda")
    eng.gemm(ddy.data_ptr(), D, M, dw2.data_ptr(), F, F, D, 6, out.data_ptr(), 2 * F, alpha=0.7,
             b_mn=1, aux0=dh13.data_ptr(), aux_ld=F)
    eng.sync()
    dg = 0.7 * (dy.double() @ w2.double())
    x1, x3 = h1.double(), h3.double()
    s = torch.sigmoid(x1)
    r1 = dg * x3 * s * (1 + x1 * (1 - s))
    r3 = dg * x1 * s
    o = out.cpu().double()
    idx = torch.arange(F)
    c1 = (idx // 16) * 32 + idx % 16
    got1, got3 = o[:, c1], o[:, c1 + 16]
    tol = 2 ** -7 * max(r1.abs().max().item(), r3.abs().max().item()) + 1e-3
    assert (got1 - r1).abs().max().item() <= tol
    assert (got3 - r3).abs().max().item() <= tol


@pytest.mark.parametrize("M,N", [(256, 1024), (200, 1000), (128, 151936 // 64)])
def test_gemm_softmax_statistics_epilogue(eng, M, N):
    """epi 7 (classifier logits): fp32 logits plus per-(row, 32-column chunk)
    (max, sum exp(x - max)) over the columns < N; combining a row's chunks
    gives its log-sum-exp."""
    K = 128
    a, b = _bf16((M, K), 31), _bf16((N, K), 32, 0.3)
    da, db = a.cuda(), b.cuda()
    nck = (N + 31) // 32
    out = torch.full((M, N), float("nan"), device="cuda")
    stats = torch.full((M, nck, 2), float("nan"), device="cuda")
    eng.gemm(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 7, out.data_ptr(), N,
             aux0=stats.data_ptr(), aux_ld=nck)
    eng.sync()
    ref = _ref(a, b)
    assert (out.cpu().double() - ref).abs().max().item() <= _tol(a, b, K)
    st = stats.cpu().double()
    pad = torch.full((M, nck * 32 - N), float("-inf"), dtype=torch.float64)
    chunks = torch.cat([ref, pad], 1).reshape(M, nck, 32)
    cmax = chunks.max(-1).values
    csum = torch.exp(chunks - cmax[..., None]).sum(-1)
    assert (st[..., 0] - cmax).abs().max().item() <= _tol(a, b, K)
    assert ((st[..., 1] - csum).abs() / csum).max().item() <= 1e-4
    lse = (st[..., 0] + torch.log(st[..., 1])).logsumexp(-1)
    assert (lse - torch.logsumexp(ref, -1)).abs().max().item() <= 1e-4


@pytest.mark.parametrize("M,N,K", [(4096, 256, 1024), (1024, 256, 3072), (6144, 5, 1024),
                                   (1000, 1, 512)])
def test_gemm_transposed_accumulate(eng, M, N, K):
    """epi 8 (decode projections): out[n, m] += alpha * (A B^T)[m, n], split-K
    partials added in L2; the existing contents are kept."""
    a, b = _bf16((M, K), 41), _bf16((N, K), 42)
    da, db = a.cuda(), b.cuda()
    base = torch.randn(N, M, generator=torch.Generator().manual_seed(43))
    out = base.clone().cuda()
    eng.gemm(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 8, out.data_ptr(), M, alpha=0.5)
    eng.sync()
    ref = base.double() + 0.5 * _ref(a, b).T
    assert (out.cpu().double() - ref).abs().max().item() <= 0.5 * _tol(a, b, K) + 1e-5


@pytest.mark.parametrize("F,N,K", [(3072, 256, 1024), (256, 200, 128), (512, 77, 192)])
def test_gemm_swiglu_transposed_epilogue(eng, F, N, K):
    """epi 10 (the decode step's fused W1/W3 projection): A = W1/W3 interleaved
    in 16-row blocks, B = the batch; gate[n, f] = silu(h1) * h3 written
    transposed (bf16), one unsplit pass."""
    w1, w3 = _bf16((F, K), 51, 0.1), _bf16((F, K), 52, 0.1)
    w13 = torch.empty((2 * F, K), dtype=torch.bfloat16)
    for c in range(F // 16):
        w13[32 * c:32 * c + 16] = w1[16 * c:16 * c + 16]
        w13[32 * c + 16:32 * c + 32] = w3[16 * c:16 * c + 16]
    x = _bf16((N, K), 53)
    gate = torch.full((N, F), float("nan"), dtype=torch.bfloat16, device="cuda")
    dw, dx = w13.cuda(), x.cuda()
    eng.gemm(dw.data_ptr(), K, 2 * F, dx.data_ptr(), K, N, K, 10, gate.data_ptr(), F)
    eng.sync()
    h1, h3 = _ref(x, w1), _ref(x, w3)
    ref = h1 * (1.0 / (1.0 + torch.exp(-h1))) * h3
    got = gate.cpu().double()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err <= 2 ** -8 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("M,N,K", [(4000, 600, 8192), (1800, 1100, 16384), (520, 300, 65536)])
def test_gemm_grouped_raster(eng, M, N, K):
    """A panels beyond ~48 MB: the units run in raster groups of m-tiles
    (ragged last group, ragged edge tiles; the first two shapes run on CTA
    pairs, the third on single CTAs with its 128-row A panels of 16 MB)."""
    a, b = _bf16((M, K), 21, 0.05), _bf16((N, K), 22, 0.05)
    da, db = a.cuda(), b.cuda()
    out = torch.full((M, N), float("nan"), device="cuda")
    eng.gemm_device(da.data_ptr(), K, M, db.data_ptr(), K, N, K, 1, out.data_ptr(), N)
    eng.sync()
    ref = _ref(a, b)
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= _tol(a, b, K), err


@pytest.mark.parametrize("M,N,K,ld,cuts", [(200, 208, 512, 256, (64 * 100, 64 * 401)),
                                           (768, 512, 1024, 512, (0, 64 * 3000)),
                                           (1024, 768, 2048, 768, (64 * 4000, 64 * 8000))])
def test_gemm_dw_owned_parts(eng, M, N, K, ld, cuts):
    """The fused dW exchange's epilogue on one GPU: three "ranks'" copies are
    three local buffers (rank 1's is local, the others take the system-scope
    reductions); each copy gains alpha * A^T B exactly on its own flat range
    [bounds[q], bounds[q+1]) and keeps its other elements bit for bit.  Rows
    beyond M and columns beyond N within ld are never touched."""
    a, b = _bf16((K, M), 31), _bf16((K, N), 32, 0.1)      # MN-major operands
    da, db = a.cuda(), b.cuda()
    world, rank, alpha = 3, 1, 0.5
    bounds = [0, cuts[0], cuts[1], M * ld]
    init = [torch.randn(M, ld, generator=torch.Generator().manual_seed(40 + q)) for q in range(world)]
    dst = [x.clone().cuda() for x in init]
    eng.gemm_dw_owned(da.data_ptr(), M, M, db.data_ptr(), N, N, K, alpha,
                      [x.data_ptr() for x in dst], bounds, rank, ld)
    eng.sync()
    ref = torch.zeros(M, ld, dtype=torch.float64)
    ref[:, :N] = alpha * (a.double().T @ b.double())
    tol = _tol(a, b, K) * alpha
    for q in range(world):
        got = dst[q].cpu().reshape(-1)
        x0 = init[q].reshape(-1)
        lo, hi = bounds[q], bounds[q + 1]
        want = x0.double().clone()
        want[lo:hi] += ref.reshape(-1)[lo:hi]
        assert torch.equal(got[:lo], x0[:lo]) and torch.equal(got[hi:], x0[hi:]), q
        if hi > lo:
            err = (got[lo:hi].double() - want[lo:hi]).abs().max().item()
            assert err <= tol + 1e-6, (q, err)
