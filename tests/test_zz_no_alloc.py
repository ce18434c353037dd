"""fk_assign_static_scratch: the assignment entry point that allocates nothing.

It serves callers that cannot allocate device memory (a host that only hands
over inputs and outputs, a pool that forbids side allocations, a loop where
cudaMalloc's possible device synchronisation is unacceptable).  Its scratch is
a 1 MiB file-scope device array instead of a caller workspace.  This file is
named to be collected last so that a run stopping at the first failure has run
every other test first; it must also pass on its own in a fresh process.
"""
import ctypes

import numpy as np
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


@pytest.mark.parametrize("dt,B,N,K,D", [(torch.float16, 4, 6000, 1000, 128),
                                         (torch.float32, 2, 3000, 300, 96)])
def test_static_scratch_matches_workspace_entry_point(dt, B, N, K, D):
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    lib = nat.load()
    g = torch.Generator(device="cuda").manual_seed(11)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    for call in range(2):  # two calls in a row: the shared scratch is rewritten each time
        x = torch.randn(B, N, D, device="cuda", generator=g).to(dt)
        c = torch.randn(B, K, D, device="cuda", generator=g).to(dt)
        xsq = _ops.row_sqnorm(x)
        ref = _ops.assign(x, c, xsq)                      # existing entry point, caller workspace
        got = torch.full((B, N), -1, dtype=torch.int32, device="cuda")
        rc = _call_static(lib, x, c, xsq, got, status)
        nat.check(rc, "fk_assign_static_scratch")
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        name = "float16" if dt == torch.float16 else "float32"
        assert_labels(x.float().cpu().numpy(), c.float().cpu().numpy(), got.cpu().numpy(),
                      ref.cpu().numpy(), name, f"static scratch call {call}")
        assert torch.equal(got, ref), f"call {call}: labels differ from fk_assign"


def test_static_scratch_rejects_oversize_without_launch():
    from flash_kmeans import _native as nat
    lib = nat.load()
    x = torch.zeros(2, 8, 128, dtype=torch.float16, device="cuda")
    c = torch.zeros(2, 131_072, 128, dtype=torch.float16, device="cuda")  # B*Kpad = 262144 > 262080
    xsq = torch.zeros(2, 8, dtype=torch.float16, device="cuda")
    out = torch.full((2, 8), -7, dtype=torch.int32, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    rc = _call_static(lib, x, c, xsq, out, status)
    assert rc == 3  # FK_ERR_WORKSPACE
    assert b"static" in lib.fk_last_error()
    torch.cuda.synchronize()
    assert int(out.min()) == -7 and int(out.max()) == -7  # nothing ran
