"""gsdlq_hex2d_matvec_noalloc: the packed matvec for callers that cannot allocate device memory.

The allocating drop-in gsdlq_hex2d_matvec keeps the reference signature, which has no workspace
argument, so it cudaMallocs its scratch on first use.  Hosts that own all device memory through
their own allocator or budget, and latency-critical loops that must not risk the device-wide
synchronisation of cudaMalloc/cudaFree, call this variant instead.  Its scratch is a fixed
4 MiB device array inside the library.

These tests call both entry points through the C ABI on the same inputs and require the same
result within the matvec tolerance, on two calls in a row.  The file is named so that pytest
collects it last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from test_gpu_kernels import rand_hex, oracle_rec, matvec_err, dev, MATVEC_TOL  # noqa: E402


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _matvec(fn, xd, h, xy, tk, y, stream=None):
    return fn(_vp(xd), _vp(h.codes), _vp(h.scales), _vp(xy), _vp(h.U), _vp(tk), _vp(h.row_ptr),
              _vp(h.kink_cols), _vp(h.kink_deltas), _vp(y), h.rows, h.cols, h.k_dim, h.n_pts, stream)


@pytest.mark.parametrize("rows,cols,k,nnz", [(1000, 4096, 16, 16), (4096, 14336, 16, 56)])
def test_noalloc_matches_allocating_dropin(cuda_lib, rng, rows, cols, k, nnz):
    import gsdlq_b200.codebook as cb
    import gsdlq_b200.ops as ops
    import gsdlq_b200._lib as L
    lib = cuda_lib
    L.device_flags()  # start from a clear flag word
    import oracle
    t = rand_hex(rng, rows, cols, k=k, nnz=nnz, radius=8)
    h = ops.DeviceHex(t)
    xy = dev(cb.xy_table(8))
    x = rng.standard_normal(cols).astype(np.float32)
    xd = dev(x)
    tk = torch.zeros(16, device="cuda")
    ops.lowrank_proj(xd, h, tk)
    y_ref = torch.zeros(rows, device="cuda")
    assert _matvec(lib.gsdlq_hex2d_matvec, xd, h, xy, tk, y_ref) == 0
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    # the allocating entry point itself against the CPU oracle of the reference's matvec
    assert matvec_err(ref, oracle.CEngine.restatement().matvec(x, oracle_rec(t))) < MATVEC_TOL
    for call in range(2):  # the shared scratch must serve a second call after the first
        y = torch.full((rows,), float("nan"), device="cuda")
        assert _matvec(lib.gsdlq_hex2d_matvec_noalloc, xd, h, xy, tk, y) == 0
        torch.cuda.synchronize()
        assert matvec_err(y.cpu().numpy(), ref) < MATVEC_TOL, f"call {call}"
    assert L.device_flags() == 0


def test_noalloc_at_the_strip_limit(cuda_lib, rng):
    """The tallest matrix the packed linear's planner takes (127 strips of 16 rows per SM: its CTAs'
    shared-memory accumulators hold 128 strips), 64 columns, against the allocating drop-in, twice;
    its scratch fills most of the fixed array.  One strip more is refused (GSDLQ_ERR_UNSUPPORTED)."""
    import gsdlq_b200.codebook as cb
    import gsdlq_b200.ops as ops
    lib = cuda_lib
    max_strips = 127 * torch.cuda.get_device_properties(0).multi_processor_count
    assert 768 + 132 * max_strips <= 4 << 20  # the scratch this launch needs fits the fixed array
    rows, cols = 16 * max_strips, 64
    t = rand_hex(rng, rows, cols, k=4, nnz=1, radius=8)
    h = ops.DeviceHex(t)
    xy = dev(cb.xy_table(8))
    xd = dev(rng.standard_normal(cols).astype(np.float32))
    tk = torch.zeros(16, device="cuda")
    ops.lowrank_proj(xd, h, tk)
    y_ref = torch.zeros(rows, device="cuda")
    assert _matvec(lib.gsdlq_hex2d_matvec, xd, h, xy, tk, y_ref) == 0
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    for call in range(2):
        y = torch.full((rows,), float("nan"), device="cuda")
        assert _matvec(lib.gsdlq_hex2d_matvec_noalloc, xd, h, xy, tk, y) == 0
        torch.cuda.synchronize()
        assert matvec_err(y.cpu().numpy(), ref) < MATVEC_TOL, f"call {call}"
    h.rows = rows + 16  # claimed height only: refused before any buffer is read
    y = torch.zeros(16, device="cuda")
    assert _matvec(lib.gsdlq_hex2d_matvec_noalloc, xd, h, xy, tk, y) == -3


def test_noalloc_rejects_oversized_launch(cuda_lib, rng):
    """A matrix whose scratch would not fit the fixed array is refused before any launch."""
    import gsdlq_b200.codebook as cb
    import gsdlq_b200.ops as ops
    lib = cuda_lib
    t = rand_hex(rng, 64, 4096, k=0, nnz=0, radius=8)
    h = ops.DeviceHex(t)
    h.rows = 1 << 22  # claimed height only: the call must return before reading any buffer
    xy = dev(cb.xy_table(8))
    xd, y = torch.zeros(4096, device="cuda"), torch.zeros(64, device="cuda")
    assert _matvec(lib.gsdlq_hex2d_matvec_noalloc, xd, h, xy, None, y) == -3  # GSDLQ_ERR_UNSUPPORTED
