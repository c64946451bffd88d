"""GEMMs on host (pinned) buffers with the PCIe copies overlapped with the kernels.

A caller whose operands live in host memory pays for moving A and B to the device and C back.
`pipelined_host_gemm` cuts A and C into row chunks and runs three streams: one copies B and
then A's chunks to the device, the caller's stream runs each chunk's GEMM as soon as its rows
have arrived, and a third copies each chunk of C back as soon as it is computed. The two copy
directions and the kernels then overlap instead of running back to back; the result is the
same as one call on the whole problem (each row of C depends only on its row of A).
"""
from __future__ import annotations

_streams: dict = {}


def _copy_streams(device):
    import torch

    key = str(device)
    if key not in _streams:
        _streams[key] = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device))
    return _streams[key]


def pipelined_host_gemm(gemm_rows, a_host, b_host, c_host, a_dev, b_dev, c_dev, chunks: int = 8, stream=None):
    """C_host = gemm(A_host, B_host) through device buffers, overlapping copies and kernels.

    gemm_rows(a_rows, b, c_rows) launches the GEMM of a block of A's rows into the same rows of C
    on the current stream. a_host / b_host / c_host are pinned host tensors, a_dev / b_dev / c_dev
    device tensors of the same shapes. Work is only enqueued: `stream` (default: the current
    stream) waits for the last copy back, so synchronising it (or recording an event on it)
    covers everything."""
    import torch

    s = stream or torch.cuda.current_stream()
    h2d, d2h = _copy_streams(s.device)
    rows = a_host.shape[0]
    chunks = max(1, min(chunks, rows))
    bounds = [rows * i // chunks for i in range(chunks + 1)]
    start = torch.cuda.Event()
    start.record(s)
    h2d.wait_event(start)
    d2h.wait_event(start)
    arrived = []
    with torch.cuda.stream(h2d):
        b_dev.copy_(b_host, non_blocking=True)
        for i in range(chunks):
            r0, r1 = bounds[i], bounds[i + 1]
            a_dev[r0:r1].copy_(a_host[r0:r1], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(h2d)
            arrived.append(ev)
    with torch.cuda.stream(s):
        for i in range(chunks):
            r0, r1 = bounds[i], bounds[i + 1]
            s.wait_event(arrived[i])
            gemm_rows(a_dev[r0:r1], b_dev, c_dev[r0:r1])
            computed = torch.cuda.Event()
            computed.record(s)
            d2h.wait_event(computed)
            with torch.cuda.stream(d2h):
                c_host[r0:r1].copy_(c_dev[r0:r1], non_blocking=True)
    done = torch.cuda.Event()
    done.record(d2h)
    s.wait_event(done)
    return c_host
