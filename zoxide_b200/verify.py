"""Result checks for a benchmark run, on the host: the reference bench's "time, then check" step.

The reference bench verifies every run it times: C is poisoned with 0xff bytes before the run,
downloaded afterwards, and 256 elements drawn with xorshift32 from state 0xdeadbeef are compared
with an i64 dot product, exactly for the integer kernels (src/bench.zig:712-740) and within a
relative error of 1e-2 (denominator max(|want|, 1)) for the float ones (src/bench.zig:384-413).
This module restates that check for the layouts and operand formats of this library and adds two
whole-matrix checks that stay affordable at full size:

- Freivalds' identity C x == A (op(B) x) for the integer GEMMs, with x a random integer vector
  in [-8, 8). Every partial sum is an integer below 2^53, so float64 arithmetic is exact and the
  comparison is exact equality; a wrong element is missed with probability <= 1/16 per random vector.
- For bf16 -> fp32, the relative Frobenius error over sampled full rows against a float64 GEMM
  (the 1e-2 tolerance of the bf16 path).

Only torch CPU tensors are used: the check is independent of the kernels it checks.
"""
from __future__ import annotations

VERIFY_STATE = 0xDEADBEEF  # src/bench.zig:717
BF16_TOL = 1e-2            # src/bench.zig:405 (relative, per sample) and the bf16 Frobenius bound


def xorshift32(state: int) -> tuple[int, int]:
    """One step of the reference's generator (src/bench.zig:26-33): (value, new state)."""
    x = state & 0xFFFFFFFF
    x ^= (x << 13) & 0xFFFFFFFF
    x ^= x >> 17
    x ^= (x << 5) & 0xFFFFFFFF
    return x, x


def sample_positions(M: int, N: int, samples: int = 256, state: int = VERIFY_STATE) -> list[tuple[int, int]]:
    """The reference's sample draw: idx = xorshift % (M*N), row = idx / N, col = idx % N."""
    out = []
    elems = M * N
    for _ in range(samples):
        v, state = xorshift32(state)
        idx = v % elems
        out.append((idx // N, idx % N))
    return out


# ---------------------------------------------------------------- operand expansion (host)
def unpack_s4_rows(W, rows):
    """Signed int4 rows of W (N x K/2 bytes, low nibble = even k) as int16 rows x K."""
    import torch

    w = W[rows].to(torch.int16)
    lo = w & 0xF
    hi = (w >> 4) & 0xF
    out = torch.stack([lo, hi], dim=-1).reshape(w.shape[0], -1)
    return torch.where(out >= 8, out - 16, out)


def decompress24_rows(A_c, meta, rows, K: int):
    """Dense int16 rows of a 2:4-sparse A from its kept values (M x K/2) and the reference's
    metadata (M x K/32 u32; nibble j of word w = idx0 | idx1 << 2 of k group 32w + 4j)."""
    import torch

    rows = torch.as_tensor(rows, dtype=torch.long)
    vals = A_c[rows].to(torch.int16).reshape(len(rows), K // 4, 2)
    words = meta[rows].to(torch.int64) & 0xFFFFFFFF
    shifts = 4 * torch.arange(8, dtype=torch.int64)
    nib = ((words.unsqueeze(-1) >> shifts) & 0xF).reshape(len(rows), K // 4)
    dense = torch.zeros((len(rows), K // 4, 4), dtype=torch.int16)
    dense.scatter_(2, (nib & 3).unsqueeze(-1), vals[..., 0:1])
    dense.scatter_(2, (nib >> 2).unsqueeze(-1), vals[..., 1:2])
    return dense.reshape(len(rows), K)


def decompress48_rows(A_c, meta, rows, K: int):
    """Dense int16 rows of imma_sp_s4's 4:8 pair-clustered s4 A (src/examples_abi.zig:83-96) from
    its kept bytes (M x K/4: per 8-wide k chunk, the two kept 2-wide sub-chunks p0 < p1, one packed
    byte each, low nibble = element 0) and metadata (M x K/64 u32; nibble j of word w =
    p0 | p1 << 2 of chunk 8w + j)."""
    import torch

    rows = torch.as_tensor(rows, dtype=torch.long)
    n = len(rows)
    b = A_c[rows].to(torch.int16)
    vals = torch.stack([b & 0xF, (b >> 4) & 0xF], dim=-1)
    vals = torch.where(vals >= 8, vals - 16, vals).reshape(n, K // 8, 2, 2)  # [chunk][kept][element]
    words = meta[rows].to(torch.int64) & 0xFFFFFFFF
    shifts = 4 * torch.arange(8, dtype=torch.int64)
    nib = ((words.unsqueeze(-1) >> shifts) & 0xF).reshape(n, K // 8)
    dense = torch.zeros((n, K // 8, 4, 2), dtype=torch.int16)
    dense.scatter_(2, (nib & 3).view(n, K // 8, 1, 1).expand(n, K // 8, 1, 2), vals[:, :, 0:1, :])
    dense.scatter_(2, (nib >> 2).view(n, K // 8, 1, 1).expand(n, K // 8, 1, 2), vals[:, :, 1:2, :])
    return dense.reshape(n, K)


def _kdim(kind, A):
    return A.shape[1] * {"sp_s8": 2, "s4s4": 2, "sp_s4": 4}.get(kind, 1)


def _a_rows(kind, A, rows, K, meta=None):
    import torch

    if kind == "sp_s4":
        return decompress48_rows(A, meta, rows, K).to(torch.int64)
    if kind == "sp_s8":
        return decompress24_rows(A, meta, rows, K).to(torch.int64)
    if kind == "s4s4":  # A packed two s4 per byte along K
        return unpack_s4_rows(A, rows).to(torch.int64)
    return A[rows].to(torch.int64)


def _b_cols(kind, B, cols, layout):
    """Columns of op(B) as int64 rows (len(cols) x K)."""
    import torch

    cols = torch.as_tensor(cols, dtype=torch.long)
    if kind in ("s4s4", "sp_s4"):  # B K x N packed two s4 per byte along N (src/examples/imma_s4.zig:89-101)
        return unpack_s4_rows(B, slice(None))[:, cols].t().to(torch.int64)
    if kind == "w4a8":
        return unpack_s4_rows(B, cols).to(torch.int64)
    if layout == 1:  # NN: B is K x N
        return B[:, cols].t().to(torch.int64)
    return B[cols].to(torch.int64)


# ---------------------------------------------------------------- sampled exact check
def check_samples(kind, A, B, C, layout=0, meta=None, rs=None, cs=None, samples=256):
    """The reference's 256-sample check on host tensors. Integer kinds and the scaled-bf16
    epilogue are compared bit for bit; bf16 -> fp32 within a relative error of 1e-2.
    Returns {"samples", "bad", "first_bad"} (+ "max_rel" for bf16)."""
    import torch

    M, N = C.shape
    K = _kdim(kind, A)
    pos = sample_positions(M, N, samples)
    rows = [r for r, _ in pos]
    cols = [c for _, c in pos]
    if kind == "bf16":
        a = A[rows].float().double()
        b = (B[:, cols].t() if layout == 1 else B[cols]).float().double()
        want = (a * b).sum(1)
        got = C[rows, cols].double()
        rel = (got - want).abs() / want.abs().clamp_min(1.0)
        rel = torch.where(torch.isnan(rel), torch.full_like(rel, float("inf")), rel)
        badm = rel > BF16_TOL
        out = {"samples": samples, "bad": int(badm.sum()), "max_rel": float(rel.max())}
    else:
        a = _a_rows(kind, A, rows, K, meta)
        b = _b_cols(kind, B, cols, layout)
        acc = (a * b).sum(1)  # exact i64 dot products
        if kind == "s8_scaled":
            want = ((acc.to(torch.float32) * rs[rows].float()) * cs[cols].float()).to(torch.bfloat16)
            got = C[rows, cols]
            badm = want.view(torch.int16) != got.view(torch.int16)
        else:
            got = C[rows, cols].to(torch.int64)
            badm = acc != got
        out = {"samples": samples, "bad": int(badm.sum())}
    if out["bad"]:
        i = int(torch.nonzero(badm)[0])
        out["first_bad"] = {"row": rows[i], "col": cols[i]}
    return out


# ---------------------------------------------------------------- Freivalds (integer kinds)
def _opb_times(kind, B, x, layout, K, chunk=2048):
    """y = op(B) x in float64 (x: N rows, y: K rows): y[k] = sum_n op(B)[k, n] x[n]."""
    import torch

    y = torch.zeros((K,) + tuple(x.shape[1:]), dtype=torch.float64)
    if kind in ("s4s4", "sp_s4"):  # B stored K x N: y = B x by blocks of k rows
        for k0 in range(0, K, chunk):
            k1 = min(K, k0 + chunk)
            y[k0:k1] = unpack_s4_rows(B, slice(k0, k1)).double() @ x
        return y
    nrows = B.shape[0] if layout == 0 or kind == "w4a8" else B.shape[1]
    for n0 in range(0, nrows, chunk):
        n1 = min(nrows, n0 + chunk)
        if kind == "w4a8":
            blk = unpack_s4_rows(B, slice(n0, n1)).double()    # (n1-n0) x K
        elif layout == 1:
            blk = B[:, n0:n1].t().double()                      # (n1-n0) x K
        else:
            blk = B[n0:n1].double()
        y += blk.t() @ x[n0:n1]
    return y


def freivalds(kind, A, B, C, layout=0, meta=None, rounds=2, seed=1234, chunk=2048):
    """Exact Freivalds' check of C == A op(B) for the integer kinds (float64, all sums exact).
    The `rounds` random vectors are the columns of one N x rounds matrix: one pass over the data."""
    import torch

    M, N = C.shape
    K = _kdim(kind, A)
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-8, 8, (N, rounds), generator=g, dtype=torch.int64).double()
    y = _opb_times(kind, B, x, layout, K, chunk)  # K x rounds
    for m0 in range(0, M, chunk):
        m1 = min(M, m0 + chunk)
        if kind == "sp_s8":
            a = decompress24_rows(A, meta, list(range(m0, m1)), K).double()
        elif kind == "sp_s4":
            a = decompress48_rows(A, meta, list(range(m0, m1)), K).double()
        elif kind == "s4s4":
            a = unpack_s4_rows(A, slice(m0, m1)).double()
        else:
            a = A[m0:m1].double()
        if not torch.equal(C[m0:m1].double() @ x, a @ y):
            return False
    return True


# ---------------------------------------------------------------- bf16 Frobenius over rows
def frobenius_rows(A, B, C, layout=0, rows=256, state=VERIFY_STATE):
    """Relative Frobenius error ||C - C_ref||_F / ||C_ref||_F over `rows` full rows of C drawn
    with the reference's generator, C_ref in float64 from the bf16 operands."""
    import torch

    M, N = C.shape
    picked = []
    for _ in range(min(rows, M)):
        v, state = xorshift32(state)
        picked.append(v % M)
    a = A[picked].double()
    bt = (B.double() if layout == 1 else B.double().t())  # K x N
    ref = a @ bt
    got = C[picked].double()
    den = float(torch.linalg.vector_norm(ref))
    err = float(torch.linalg.vector_norm(got - ref))
    if err != err:  # NaN (e.g. a poisoned element left unwritten)
        err = float("inf")
    return {"rows": len(picked), "rel_frobenius": err / max(den, 1e-300), "tol": BF16_TOL}


def check_result(kind, A, B, C, layout=0, meta=None, rs=None, cs=None, freivalds_rounds=2):
    """Every check that applies to `kind`, on host tensors; "ok" is the verdict."""
    res = check_samples(kind, A, B, C, layout, meta, rs, cs)
    ok = res["bad"] == 0
    if kind in ("s8", "w4a8", "sp_s8", "s4s4", "sp_s4"):
        res["freivalds"] = freivalds(kind, A, B, C, layout, meta, rounds=freivalds_rounds)
        ok = ok and res["freivalds"]
    elif kind == "bf16":
        fr = frobenius_rows(A, B, C, layout)
        res["rel_frobenius_256_rows"] = fr["rel_frobenius"]
        ok = ok and fr["rel_frobenius"] <= BF16_TOL
    elif kind == "s8_scaled":
        # the epilogue is not linear: add four full rows compared bit for bit
        import torch

        M, N = C.shape
        rows = [0, M // 3, (2 * M) // 3, M - 1]
        # float64 products and sums of these integers are exact (|acc| < 2^31 < 2^53)
        acc = A[rows].double() @ (B.double() if layout == 1 else B.double().t())
        want = ((acc.to(torch.float32) * rs[rows].float().unsqueeze(1)) * cs.float().unsqueeze(0)).to(torch.bfloat16)
        res["full_rows_exact"] = bool(torch.equal(want.view(torch.int16), C[rows].view(torch.int16)))
        ok = ok and res["full_rows_exact"]
    res["ok"] = bool(ok)
    return res
