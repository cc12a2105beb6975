"""The chunked scan entry point that allocates nothing.

Some callers cannot call cudaMalloc while they work -- a host whose own pool
allocator already owns the device memory, or a latency-critical loop that
cannot absorb the device-wide synchronisation an allocation may cause.  For
them nk_scan_chunked_noalloc_device runs the time-chunked scan on a fixed
scratch array inside the library instead of allocating one per call.  This
test calls it through the C ABI and checks it against the allocating entry
point nk_scan_device(chunked=1) on two calls in a row with different shapes
and data (the second call reuses the scratch the first one left behind), and
checks that a scan too large for the fixed scratch is refused with a message.
It lives in its own file so that pytest collects it last."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the scan tolerance of the reference's own test (scan.rs:286)


def _scan_pair(nb, torch, a, b, batch, t, d, stream):
    """(no-alloc result, allocating-entry-point result) for the same inputs."""
    da = torch.from_numpy(a).cuda()
    db = torch.from_numpy(b).cuda()
    h_new = torch.full_like(da, float("nan"))
    h_ref = torch.full_like(da, float("nan"))
    L = nb.lib()
    nb._check(L.nk_scan_chunked_noalloc_device(C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()),
                                               C.c_void_p(h_new.data_ptr()), batch, t, d, C.c_void_p(stream)))
    nb._check(L.nk_scan_device(C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()), C.c_void_p(h_ref.data_ptr()),
                               batch, t, d, 1, C.c_void_p(stream)))
    torch.cuda.synchronize()
    return h_new.cpu().numpy(), h_ref.cpu().numpy()


def test_noalloc_scan_matches_the_allocating_scan_on_two_calls(gpu, orc):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    rs = np.random.default_rng(123)
    for batch, t, d in [(3, 1000, 17), (2, 700, 33)]:
        n = batch * t * d
        a = rs.uniform(0.01, 0.99, n).astype(np.float32)
        b = rs.standard_normal(n).astype(np.float32)
        new, ref = _scan_pair(gpu, torch, a, b, batch, t, d, stream)
        assert np.isfinite(new).all()
        assert np.abs(new - ref).max() <= TOL
        assert np.abs(new - orc.scan_sequential(a, b, batch, t, d, 1)).max() <= TOL


def test_noalloc_scan_refuses_sizes_beyond_its_fixed_scratch(gpu):
    import torch

    # 8 streams x 512 time blocks x 257 channels > 1048576 block states.
    batch, t, d = 8, 512 * 256, 257
    L = gpu.lib()
    dummy = torch.zeros(4, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    status = L.nk_scan_chunked_noalloc_device(p, p, p, batch, t, d, None)
    assert status == gpu.NK_ERR_INVALID
    assert "exceeds the fixed scratch limit" in L.nk_last_error().decode()


def test_noalloc_scan_at_the_exact_scratch_boundary(gpu):
    """batch * ceil(t / 256) * d == 1048576 fills the fixed scratch exactly
    (every one of its floats is written and read) and is accepted, equal to
    the allocating scan; one more stream, or one more time step (a second
    time block per channel), is refused before anything runs."""
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    batch, t, d = 512, 1, 2048
    rs = np.random.default_rng(7)
    n = batch * t * d
    a = rs.uniform(0.01, 0.99, n).astype(np.float32)
    b = rs.standard_normal(n).astype(np.float32)
    new, ref = _scan_pair(gpu, torch, a, b, batch, t, d, stream)
    assert np.isfinite(new).all()
    assert np.abs(new - ref).max() <= TOL
    L = gpu.lib()
    dummy = torch.zeros(4, device="cuda")
    p = C.c_void_p(dummy.data_ptr())
    for shape in [(513, 1, 2048), (512, 257, 2048)]:
        status = L.nk_scan_chunked_noalloc_device(p, p, p, *shape, None)
        assert status == gpu.NK_ERR_INVALID, shape
        assert "exceeds the fixed scratch limit" in L.nk_last_error().decode()
