"""The C-ABI library loads without a GPU and exports every symbol include/gsdlq.h declares."""
import ctypes

import numpy as np
import pytest

from gsdlq_b200 import _lib as L


def test_library_exports_header_symbols():
    lib = L.load()
    names = L.header_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # every declared function has a typed binding
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


def test_host_functions_without_gpu(oracle_mod):
    lib = L.load()
    assert lib.gsdlq_version().startswith(b"0.")
    assert lib.gsdlq_status_string(-1) == b"invalid argument"
    for r, n in ((6, 127), (8, 217)):
        buf = np.zeros(512, np.float32)
        assert lib.gsdlq_codebook(r, buf.ctypes.data_as(ctypes.c_void_p), 256) == n
        assert np.array_equal(buf[:2 * n].reshape(n, 2), oracle_mod.codebook(r)[0])
    assert lib.gsdlq_codebook(0, None, 0) == -1


def test_rope_table_matches_reference_formula(restated):
    lib = L.load()
    S, hd, th = 64, 32, 1e6
    t = np.zeros((S, hd // 2, 2), np.float32)
    assert lib.gsdlq_rope_table(t.ctypes.data_as(ctypes.c_void_p), S, hd, th) == 0
    c, s = ctypes.c_float(), ctypes.c_float()
    for p in (0, 1, 37, 63):
        for i in (0, 5, 15):
            restated.lib.orc_rope_cos_sin(p, i, hd, ctypes.c_float(th), ctypes.byref(c), ctypes.byref(s))
            assert t[p, i, 0] == c.value and t[p, i, 1] == s.value


def test_argument_errors_before_launch():
    """Invalid shapes are rejected on the host (no GPU needed)."""
    lib = L.load()
    assert lib.gsdlq_hex2d_matvec(None, None, None, None, None, None, None, None, None, None, 16, 64, 0, 217,
                                  None) == -1
    assert lib.gsdlq_rmsnorm(None, None, None, 0, 1e-5, None) == -1
    assert lib.gsdlq_rope_and_store_kv(None, None, None, None, None, 0, 0, 1, 1, 64, 16, 1e4, 1, None) == -1
    job = L.LinearJob()
    job.n_mat = 0
    assert lib.gsdlq_linear(ctypes.byref(job), None, 0, None) == -1
