"""Host logic of batched decode (no GPU): stacking packed matrices by rows for one fused GEMM."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def test_stack_rows_concatenates_codes_scales_and_kinks():
    import gsdlq_b200.packer as P
    from gsdlq_b200.ops import DeviceHex
    from gsdlq_b200.batch import _stack_rows
    a = P.random_packed_matrix(48, 256, "precision", seed=1)
    b = P.random_packed_matrix(16, 256, "precision", seed=2)
    ha, hb = DeviceHex(a, device="cpu"), DeviceHex(b, device="cpu")
    for h in (ha, hb):  # stacking is for matrices without a low-rank term
        h.k_dim, h.U, h.S, h.Vt = 0, None, None, None
    s = _stack_rows([ha, hb])
    assert (s.rows, s.cols, s.nnz) == (64, 256, a.kink_cols.size + b.kink_cols.size)
    np.testing.assert_array_equal(s.codes.numpy().view(np.uint8), np.concatenate([a.codes, b.codes]))
    np.testing.assert_array_equal(s.scales.numpy().view(np.uint16), np.concatenate([a.scales, b.scales]))
    rp = s.row_ptr.numpy().view(np.uint32)
    np.testing.assert_array_equal(rp, np.concatenate([a.row_ptr, b.row_ptr[1:] + a.row_ptr[-1]]))
    np.testing.assert_array_equal(s.kink_cols.numpy().view(np.uint16), np.concatenate([a.kink_cols, b.kink_cols]))
    np.testing.assert_array_equal(s.kink_deltas.numpy().view(np.float32),
                                  np.concatenate([a.kink_deltas, b.kink_deltas]))
    # rows keep their kinks: row 48 of the stack is row 0 of b
    assert list(s.kink_cols.numpy().view(np.uint16)[rp[48]:rp[49]]) == list(b.kink_cols[b.row_ptr[0]:b.row_ptr[1]])
