"""fk_assign_static_scratch: the assignment entry point that allocates nothing.

It serves callers that cannot allocate device memory: a host that hands a
plugin only its inputs and outputs (no workspace hook), a memory pool that
forbids side allocations, or a latency-bound loop where cudaMalloc's possible
device synchronisation is unacceptable.  Its scratch is a 16 MiB file-scope
device array instead of a caller workspace.  This file is named to be
collected last so that a run stopping at the first failure has run every
other test first; it must also pass on its own in a fresh process.
"""
import pytest
import torch

from _parity import assert_labels
from oracle import kmeans_oracle as ko

pytestmark = pytest.mark.gpu


def _call_static(lib, x, c, xsq, out, status, c_sq=None):
    from flash_kmeans import _native as nat
    B, N, D = x.shape
    K = c.shape[1]
    return lib.fk_assign_static_scratch(
        nat.ptr(x), nat.ptr(c), nat.ptr(xsq), nat.ptr(c_sq), nat.ptr(out), None,
        nat.dtype_code(x.dtype), nat.dtype_code(xsq.dtype),
        nat.dtype_code(c_sq.dtype) if c_sq is not None else 0, B, N, K, D,
        nat.strides(x, 3), nat.strides(c, 3), nat.strides(xsq, 2),
        nat.strides(c_sq, 2) if c_sq is not None else None, nat.strides(out, 2),
        nat.ptr(status), nat.stream_handle(x.device))


NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}


@pytest.mark.parametrize("dt,B,N,K,D,given_csq", [
    (torch.float16, 4, 6000, 1000, 128, False),   # 256-column tiles
    (torch.float16, 3, 5000, 100, 64, False),     # K <= 128: narrow tiles, resident centroids
    (torch.bfloat16, 2, 3000, 300, 128, True),    # caller-provided c_sq
    (torch.float32, 2, 3000, 300, 96, False),     # 3xTF32 split-D path
])
def test_static_scratch_matches_workspace_entry_point(dt, B, N, K, D, given_csq):
    """Two calls in a row (the shared scratch is rewritten each time): labels
    equal fk_assign's with a caller workspace, and agree with the CPU oracle at
    the parity bar."""
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    lib = nat.load()
    g = torch.Generator(device="cuda").manual_seed(11)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    name = NAMES[dt]
    for call in range(2):
        x = torch.randn(B, N, D, device="cuda", generator=g).to(dt)
        c = torch.randn(B, K, D, device="cuda", generator=g).to(dt)
        xsq = _ops.row_sqnorm(x)
        c_sq = _ops.row_sqnorm(c) if given_csq else None
        ref = _ops.assign(x, c, xsq, c_sq=c_sq)          # existing entry point, caller workspace
        got = torch.full((B, N), -1, dtype=torch.int32, device="cuda")
        nat.check(_call_static(lib, x, c, xsq, got, status, c_sq=c_sq), "fk_assign_static_scratch")
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        assert torch.equal(got, ref), f"call {call}: labels differ from fk_assign"
        xn, cn = x.float().cpu().numpy(), c.float().cpu().numpy()
        o = ko.assign(xn, cn, xsq.float().cpu().numpy(), name)
        assert_labels(xn, cn, got.cpu().numpy(), o, name, f"static scratch call {call} vs oracle")


def test_static_scratch_allocates_nothing():
    """After the first call (which loads the library's device module, static
    array included), further calls leave the device's free memory unchanged."""
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    lib = nat.load()
    B, N, K, D = 8, 4000, 512, 128
    x = torch.randn(B, N, D, device="cuda").half()
    c = torch.randn(B, K, D, device="cuda").half()
    xsq = _ops.row_sqnorm(x)
    out = torch.empty((B, N), dtype=torch.int32, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    nat.check(_call_static(lib, x, c, xsq, out, status), "fk_assign_static_scratch")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        nat.check(_call_static(lib, x, c, xsq, out, status), "fk_assign_static_scratch")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert int(status[0]) == 0


def test_static_scratch_rejects_oversize_without_launch():
    from flash_kmeans import _native as nat
    lib = nat.load()
    B, K, D = 32, 2048, 128   # c_sq 256 KiB + -2c 16 MiB > 16 MiB
    assert lib.fk_assign_workspace_size(B, K, D, nat.FK_F16) > (16 << 20)
    x = torch.zeros(B, 8, D, dtype=torch.float16, device="cuda")
    c = torch.zeros(B, K, D, dtype=torch.float16, device="cuda")
    xsq = torch.zeros(B, 8, dtype=torch.float16, device="cuda")
    out = torch.full((B, 8), -7, dtype=torch.int32, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    rc = _call_static(lib, x, c, xsq, out, status)
    assert rc == 3  # FK_ERR_WORKSPACE
    assert b"static" in lib.fk_last_error()
    torch.cuda.synchronize()
    assert int(out.min()) == -7 and int(out.max()) == -7  # nothing ran
