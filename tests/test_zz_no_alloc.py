"""The allocation-free row-norm entry point (arcqml_rt_v2_norms_noalloc), checked on a B200.

It exists for callers that cannot allocate device memory while they run (their memory is all
in their own pool, or an allocation would synchronise the device at a bad moment), so it keeps
its scratch in a static device array instead of a cudaMalloc'd workspace. These tests compare it
with the regular arcqml_rt_v2_norms through the C ABI on two calls in a row (different batch
sizes, so the second call must not see the first call's scratch contents), and check that a
batch over its row limit is rejected. The file is named to be collected last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _states(seed, batch, n):
    g = np.random.Generator(np.random.PCG64(seed))
    a = g.normal(size=(batch, 1 << n)) + 1j * g.normal(size=(batch, 1 << n))
    a *= g.uniform(0.5, 2.0, size=(batch, 1))  # rows of different norms
    return np.ascontiguousarray(a)


def test_noalloc_norms_match_the_allocating_entry_point_twice(runtime):
    import torch

    for seed, batch, n in [(1, 37, 12), (2, 5, 20)]:
        a = torch.from_numpy(_states(seed, batch, n)).cuda()
        want = runtime.norms_device(a, n)
        got = runtime.norms_device_noalloc(a, n)
        assert got.shape == (batch,)
        np.testing.assert_allclose(got, want, rtol=1e-12, atol=0)
        exact = np.einsum("ij,ij->i", a.cpu().numpy().conj(), a.cpu().numpy()).real
        np.testing.assert_allclose(got, exact, rtol=1e-12, atol=0)


def test_noalloc_norms_reject_batches_over_the_limit(runtime):
    import torch

    a = torch.zeros((8193, 2), dtype=torch.complex128, device="cuda")
    with pytest.raises(runtime.RuntimeError, match="8192-row limit"):
        runtime.norms_device_noalloc(a, 1)


def test_noalloc_norms_leave_device_memory_unchanged(runtime):
    """Its one promise: a call allocates no device memory. The first call on the device (symbol
    lookup, module load) is made beforehand; the measured call then runs on a new host thread,
    whose per-thread workspace is empty, so any use of that workspace would cudaMalloc and show
    up in the device's free memory."""
    import threading

    import torch

    a = torch.from_numpy(_states(3, 64, 14)).cuda()
    runtime.norms_device_noalloc(a, 14)
    torch.cuda.synchronize()
    out = {}

    def worker():
        torch.cuda.set_device(a.device)
        free0, _ = torch.cuda.mem_get_info()
        out["norms"] = runtime.norms_device_noalloc(a, 14, stream=0)
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        out["delta"] = free0 - free1

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert out["delta"] == 0
    np.testing.assert_allclose(out["norms"], runtime.norms_device(a, 14), rtol=1e-12, atol=0)
