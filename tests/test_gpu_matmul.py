"""The batched packed linear (gsdlq_hex2d_matmul): every token's output against the oracle's
per-token matvec (the 1e-3 matvec bar), and against the batch-1 matvec drop-in."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from test_gpu_kernels import rand_hex, oracle_rec, rel_err, matvec_err, dev, MATVEC_TOL  # noqa: E402


@pytest.fixture(scope="module")
def env(cuda_lib):
    import gsdlq_b200.ops as ops
    import gsdlq_b200._lib as L
    L.device_flags()
    return ops, L


@pytest.mark.parametrize("rows,cols,k,nnz,radius", [
    (16, 64, 0, 0, 8), (100, 512, 16, 2, 8), (1024, 4096, 16, 16, 8), (4096, 4096, 8, 16, 6), (700, 14336, 16, 56, 8)])
@pytest.mark.parametrize("batch", [1, 3, 16, 24, 32, 40, 64, 100, 128])  # token groups 1-4: small kernel
def test_matmul_vs_oracle(env, restated, rng, rows, cols, k, nnz, radius, batch):
    ops, L = env
    import gsdlq_b200.codebook as cb
    t = rand_hex(rng, rows, cols, k=k, nnz=nnz, radius=radius)
    rec = oracle_rec(t)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    x[batch // 2] *= 40.0  # tokens of very different magnitude share the launch
    h = ops.DeviceHex(t)
    y = torch.full((batch, rows), 7.0, device="cuda")  # the entry point zeroes it
    work = ops.matmul_work(batch, cols)
    xy = dev(cb.xy_table(radius))
    for rep in range(2):
        ops.hex2d_matmul(dev(x), h, xy, y, work)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        for b in range(batch):
            yr = restated.matvec(np.ascontiguousarray(x[b]), rec, np.zeros(16, np.float32))
            assert matvec_err(got[b], yr) < MATVEC_TOL, (rep, b)
    assert L.device_flags() == 0


@pytest.mark.parametrize("batch", [1, 5, 40])
def test_matmul_widest_rows(env, restated, rng, batch):
    """65472 columns, the widest multiple of 64 a u16 kink column reaches, with a kink in every row's last
    column: the GEMM takes the width (its activations stream from global memory); the fused matvec cannot
    (GSDLQ_MATVEC_MAX_COLS), so the drop-in matvec hands such rows to the GEMM, and the no-allocation
    matvec refuses them."""
    ops, L = env
    import gsdlq_b200.codebook as cb
    rows, cols = 48, 65472
    t = rand_hex(rng, rows, cols, k=16, nnz=8, radius=8)
    kc = t.kink_cols.reshape(rows, 8).copy()
    kc[:, -1] = cols - 1
    t.kink_cols = np.sort(kc, axis=1).astype(np.uint16).reshape(-1)
    t.validate()
    rec = oracle_rec(t)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    h = ops.DeviceHex(t)
    y = torch.zeros((batch, rows), device="cuda")
    xy = dev(cb.xy_table(8))
    ops.hex2d_matmul(dev(x), h, xy, y, ops.matmul_work(batch, cols))
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for b in range(batch):
        yr = restated.matvec(np.ascontiguousarray(x[b]), rec, np.zeros(16, np.float32))
        assert matvec_err(got[b], yr) < MATVEC_TOL, b
    # the drop-in pair (projection, then matvec) on token 0, its x at an offset that is not 16-byte aligned
    tk, y1 = torch.zeros(16, device="cuda"), torch.full((rows,), 7.0, device="cuda")
    xbuf = torch.zeros(cols + 1, device="cuda")
    xbuf[1:].copy_(dev(x[0]))
    x0 = xbuf[1:]
    ops.lowrank_proj(x0, h, tk)
    ops.hex2d_matvec(x0, h, xy, tk, y1)
    torch.cuda.synchronize()
    yr = restated.matvec(np.ascontiguousarray(x[0]), rec, np.zeros(16, np.float32))
    assert matvec_err(y1.cpu().numpy(), yr) < MATVEC_TOL
    lib = L.load()
    assert lib.gsdlq_hex2d_matvec_noalloc(x0.data_ptr(), h.codes.data_ptr(), h.scales.data_ptr(), xy.data_ptr(),
                                          h.U.data_ptr(), tk.data_ptr(), h.row_ptr.data_ptr(),
                                          h.kink_cols.data_ptr(), h.kink_deltas.data_ptr(), y1.data_ptr(), rows,
                                          cols, 16, 217, None) == -3
    assert L.device_flags() == 0


def test_matmul_batch1_matches_matvec(env, rng):
    ops, L = env
    import gsdlq_b200.codebook as cb
    t = rand_hex(rng, 4096, 4096, k=16, nnz=16, radius=8)
    h = ops.DeviceHex(t)
    x = rng.standard_normal((1, 4096)).astype(np.float32)
    xd, xy = dev(x), dev(cb.xy_table(8))
    y1, tk = torch.zeros(4096, device="cuda"), torch.zeros(16, device="cuda")
    ops.lowrank_proj(xd[0], h, tk)
    ops.hex2d_matvec(xd[0], h, xy, tk, y1)
    y2, work = torch.zeros((1, 4096), device="cuda"), ops.matmul_work(1, 4096)
    ops.hex2d_matmul(xd, h, xy, y2, work)
    torch.cuda.synchronize()
    assert matvec_err(y2.cpu().numpy()[0], y1.cpu().numpy()) < MATVEC_TOL


def test_matmul_rejects_bad_arguments(env, rng):
    ops, L = env
    import gsdlq_b200.codebook as cb
    t = rand_hex(rng, 64, 128, k=0, nnz=0, radius=8)
    h = ops.DeviceHex(t)
    xy, work = dev(cb.xy_table(8)), ops.matmul_work(ops.MATMUL_MAX_BATCH, 128)
    wp, wb = ops._aligned(work)
    for batch in (0, ops.MATMUL_MAX_BATCH + 1):
        x = torch.zeros((max(batch, 1), 128), device="cuda")
        y = torch.zeros((max(batch, 1), 64), device="cuda")
        st = L.load().gsdlq_hex2d_matmul(ops.ptr(x), batch, ops.ptr(h.codes), ops.ptr(h.scales), ops.ptr(xy), None,
                                         None, None, ops.ptr(h.row_ptr), ops.ptr(h.kink_cols), ops.ptr(h.kink_deltas),
                                         ops.ptr(y), wp, wb, 64, 128, 0, h.n_pts, None)
        assert st == -1
    # a work buffer below the size the batch needs is refused
    x, y = torch.zeros((16, 128), device="cuda"), torch.zeros((16, 64), device="cuda")
    st = L.load().gsdlq_hex2d_matmul(ops.ptr(x), 16, ops.ptr(h.codes), ops.ptr(h.scales), ops.ptr(xy), None, None, None,
                                     ops.ptr(h.row_ptr), ops.ptr(h.kink_cols), ops.ptr(h.kink_deltas), ops.ptr(y), wp,
                                     ops.matmul_work_bytes(16, 128) - 16, 64, 128, 0, h.n_pts, None)
    assert st == -1
