"""zx_gemm_s8_mgpu: one host thread driving several GPUs over the C ABI (M-row shards, no
collective). Every shard is compared with the oracle element for element. With one GPU the
shards run on the same device (the entry point allows repeats); with two, one per device."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(zxo, M, N, K, layout, state):
    r = zxo.Rng(state)
    A = r.s8((M, K))
    B = r.s8((N, K) if layout == 0 else (K, N))
    return A, B, zxo.gemm_s8(A, B, M, N, K, layout)


def _run(zx, A, B, M, N, devices, layout):
    n = len(devices)
    bounds = [M * i // n for i in range(n + 1)]
    As = [torch.from_numpy(np.ascontiguousarray(A[bounds[i]:bounds[i + 1]])).to(f"cuda:{d}") for i, d in enumerate(devices)]
    Bs = [torch.from_numpy(B).to(f"cuda:{d}") for d in devices]
    Cs = [torch.full((bounds[i + 1] - bounds[i], N), -1, dtype=torch.int32, device=f"cuda:{d}")
          for i, d in enumerate(devices)]
    zx.gemm_s8_mgpu(As, Bs, Cs, M, layout=layout)
    for d in set(devices):
        torch.cuda.synchronize(d)
    return np.concatenate([c.cpu().numpy() for c in Cs])


@pytest.mark.parametrize("layout", [0, 1], ids=["NT", "NN"])
@pytest.mark.parametrize("nshards", [1, 3])
def test_mgpu_shards_one_device(zx, zxo, layout, nshards):
    M, N, K = 777, 512, 384
    A, B, want = _case(zxo, M, N, K, layout, 0x600D + nshards + layout)
    got = _run(zx, A, B, M, N, [0] * nshards, layout)
    assert np.array_equal(got, want)
    assert torch.cuda.current_device() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_mgpu_two_devices(zx, zxo):
    M, N, K = 2048, 1024, 512
    A, B, want = _case(zxo, M, N, K, 0, 0x7007)
    torch.cuda.set_device(1)
    got = _run(zx, A, B, M, N, [0, 1], 0)
    assert torch.cuda.current_device() == 1  # the caller's device is restored
    torch.cuda.set_device(0)
    assert np.array_equal(got, want)
