"""Scaled-bf16 epilogue (BASELINE config 2 variant) and the bf16 x bf16 -> fp32 GEMM.

The scaled epilogue is bit-exact against the oracle: (float)acc and both multiplies are
round-to-nearest-even in a fixed order with no FMA, then bf16 round-to-nearest-even.
The bf16 GEMM is checked within 1e-2 relative Frobenius error (north_star tolerance) against an
f64 CPU reference over sampled full rows, and exactly on small-integer inputs where fp32
accumulation is exact (the reference's own bf16 trick, src/bench.zig:542-548).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FROB_TOL = 1e-2


def _scaled_case(zxo, M, N, K, layout, seed):
    r = zxo.Rng.from_seed(seed)
    A = r.s8((M, K))
    B = r.s8((N, K) if layout == 0 else (K, N))
    rs = r.uniform_f32(M, 0.5, 2.0)
    cs = r.uniform_f32(N, 1e-3, 1e-2)
    return A, B, rs, cs


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (1024, 1024, 1024), (200, 336, 176)])
def test_scaled_bf16_exact(zx, zxo, policy, M, N, K, layout):
    A, B, rs, cs = _scaled_case(zxo, M, N, K, layout, M + N + K)
    dC = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    zx.gemm_s8_scaled_bf16(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(),
                           torch.from_numpy(rs).cuda(), torch.from_numpy(cs).cuda(), dC, layout=layout)
    torch.cuda.synchronize()
    got = dC.view(torch.int16).cpu().numpy().view(np.uint16)
    want = zxo.gemm_s8_scaled_bf16(A, B, rs, cs, N, K, layout, 0, M)
    if not np.array_equal(got, want):
        bad = np.argwhere(got != want)
        r, c = bad[0]
        pytest.fail(f"{len(bad)} mismatches; first ({r},{c}) want {want[r, c]:#06x} got {got[r, c]:#06x}")


@pytest.mark.slow
def test_scaled_bf16_full_size(zx, zxo):
    M = N = K = 8192
    A, B, rs, cs = _scaled_case(zxo, M, N, K, 0, 0)
    dC = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    zx.gemm_s8_scaled_bf16(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(),
                           torch.from_numpy(rs).cuda(), torch.from_numpy(cs).cuda(), dC)
    torch.cuda.synchronize()
    got = dC.view(torch.int16).cpu().numpy().view(np.uint16)
    for r0 in (0, 1, 127, 128, 4095, 8191):
        want = zxo.gemm_s8_scaled_bf16(A, B, rs, cs, N, K, 0, r0, r0 + 1)
        assert np.array_equal(got[r0], want[0]), f"row {r0}"


def _bf16_case(zxo, M, N, K, layout, seed):
    r = zxo.Rng.from_seed(seed)
    A = r.normal_bf16((M, K), 1.0 / np.sqrt(K))
    B = r.normal_bf16((N, K) if layout == 0 else (K, N), 1.0 / np.sqrt(K))
    return A, B


def _to_dev_bf16(a):
    return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (512, 512, 1024), (300, 264, 136)])
def test_bf16_frobenius(zx, zxo, policy, M, N, K, layout):
    A, B = _bf16_case(zxo, M, N, K, layout, 5 + M + layout)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    zx.gemm_bf16(_to_dev_bf16(A), _to_dev_bf16(B), dC, layout=layout)
    torch.cuda.synchronize()
    got = dC.cpu().numpy().astype(np.float64)
    want = zxo.gemm_bf16_f64(A, B, N, K, layout, 0, M)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= FROB_TOL, err
    # fp32 accumulation of bf16 products is far tighter than the contract; flag regressions
    assert err <= 1e-5, err


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (512, 512, 1024), (300, 264, 136), (2560, 4096, 512)])
def test_f16_frobenius(zx, policy, M, N, K, layout):
    """f16 operands on the same kernels (A/B format f16 in the instruction descriptor): within the
    1e-2 relative Frobenius contract of the 16-bit float path against a float64 product (measured
    far tighter), on every tile path."""
    g = torch.Generator().manual_seed(M + N + K + layout)
    A = (torch.randn((M, K), generator=g) / K ** 0.5).to(torch.float16)
    B = (torch.randn((N, K) if layout == 0 else (K, N), generator=g) / K ** 0.5).to(torch.float16)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    zx.gemm_f16(A.cuda(), B.cuda(), dC, layout=layout)
    torch.cuda.synchronize()
    assert zx.device_status() == 0
    want = A.double() @ (B.double().t() if layout == 0 else B.double())
    got = dC.cpu().double()
    err = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
    assert err <= FROB_TOL, err
    assert err <= 1e-5, err
    # the same bits read as bf16 give a different product: the f16 format really is in use
    if M == 128 and layout == 0:
        dX = torch.empty((M, N), dtype=torch.float32, device="cuda")
        zx.gemm_bf16(A.cuda().view(torch.bfloat16), B.cuda().view(torch.bfloat16), dX, layout=layout)
        torch.cuda.synchronize()
        assert not torch.allclose(dX.cpu(), dC.cpu())


def test_bf16_small_int_exact(zx, zxo):
    """Reference bf16 harness data (values -2..2, src/bench.zig:559-571): exact in fp32."""
    n = 512
    r = zxo.Rng(zxo.REF_STATE_BF16)
    vals = np.array([r.next() % 5 for _ in range(2 * n * n)], dtype=np.int64) - 2
    a = vals[: n * n].astype(np.float32).reshape(n, n)
    b = vals[n * n:].astype(np.float32).reshape(n, n)  # K x N (reference layout)
    tb = lambda x: torch.from_numpy(x).cuda().to(torch.bfloat16).contiguous()
    dC = torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda")
    zx.hgemm_bf16(tb(a), tb(b), dC, n)
    torch.cuda.synchronize()
    want = a.astype(np.float64) @ b.astype(np.float64)
    assert np.array_equal(dC.cpu().numpy().astype(np.float64), want)


def _sample_rows(M, count, state=0xDEADBEEF):
    """Row indices drawn with the reference's generator and verify state (src/bench.zig:384-413)."""
    from zoxide_b200.verify import xorshift32

    rows = []
    for _ in range(count):
        v, state = xorshift32(state)
        rows.append(v % M)
    return rows


@pytest.mark.slow
def test_bf16_config5_full_shape(zx, zxo):
    """BASELINE config 5 at its own shape: M=65536, N=K=8192, A row-major, B column-major, on the
    automatic tile choice (many 256 x 512 tiles per CTA pair). 256 full rows drawn with the
    reference's generator are compared with the oracle's f64 GEMM: relative Frobenius error
    <= 1e-2 (north_star), and the reference's per-sample rule (rel err <= 1e-2, denominator
    max(|want|, 1)) on every element of those rows."""
    M, N, K = 65536, 8192, 8192
    r = zxo.Rng.from_seed(55)
    B = r.normal_bf16((N, K), 1.0 / np.sqrt(K))
    g = torch.Generator(device="cuda")
    g.manual_seed(55)
    dA = (torch.randn((M, K), device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    zx.gemm_bf16(dA, _to_dev_bf16(B), dC)
    torch.cuda.synchronize()
    rows = _sample_rows(M, 256)
    idx = torch.tensor(rows, device="cuda")
    A_rows = dA[idx].cpu().view(torch.int16).numpy().view(np.uint16)
    got = dC[idx].cpu().numpy().astype(np.float64)
    want = zxo.gemm_bf16_f64(np.ascontiguousarray(A_rows), B, N, K, 0, 0, len(rows))
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= FROB_TOL, err
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
    assert rel.max() <= FROB_TOL, rel.max()
    assert err <= 1e-5, err  # fp32 accumulation: far inside the contract
    # no element left unwritten anywhere (the NaN fill), checked on the device
    assert not torch.isnan(dC).any().item()


@pytest.mark.parametrize("pol", [0, 4], ids=["auto", "2sm512"])
def test_bf16_many_tiles_per_pair(zx, zxo, pol):
    """bf16 on the 256 x 512 pair kernel with several tiles per CTA pair (2560 x 4096: 80 tiles
    over 74 pairs, and a ragged last row block), every element against the oracle."""
    M, N, K = 2560, 4096, 1024
    A, B = _bf16_case(zxo, M, N, K, 0, 77)
    zx.set_kernel_policy(pol)
    try:
        dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        zx.gemm_bf16(_to_dev_bf16(A), _to_dev_bf16(B), dC)
        torch.cuda.synchronize()
        kernel = zx.last_kernel()
    finally:
        zx.set_kernel_policy(0)
    got = dC.cpu().numpy().astype(np.float64)
    want = zxo.gemm_bf16_f64(A, B, N, K, 0, 0, M)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err <= 1e-5, (err, kernel)
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
    assert rel.max() <= FROB_TOL, (rel.max(), kernel)
    if pol == 4:
        assert "tc2w" in kernel, kernel
