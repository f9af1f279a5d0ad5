"""The C-ABI library loads without a GPU and exports every symbol include/gsdlq.h declares."""
import ctypes
import os

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


def test_bindings_match_header_arity():
    """Every ctypes binding takes as many arguments as its declaration in include/gsdlq.h."""
    import re
    txt = re.sub(r"/\*.*?\*/", "", open(L.HEADER).read(), flags=re.S)
    for name, (args, _) in L.SIGNATURES.items():
        m = re.search(r"\b" + name + r"\s*\(([^)]*)\)\s*;", txt)
        assert m, name
        params = m.group(1).strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        assert n == len(args), (name, n, len(args))


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


def test_batched_and_noalloc_argument_errors_before_launch():
    """The batched linear and the no-allocation matvec refuse bad shapes and alignments on the host,
    before any CUDA call (the stand-in addresses below are never dereferenced)."""
    lib = L.load()
    A = ctypes.c_void_p(0x100000)        # a 256-byte-aligned stand-in address
    odd = ctypes.c_void_p(0x100001)

    def mm(x=A, batch=4, codes=A, y=A, work=A, rows=64, cols=128, k=0, n_pts=217, U=None, S=None, Vt=None, wb=1 << 30):
        return lib.gsdlq_hex2d_matmul(x, batch, codes, A, A, U, S, Vt, A, A, A, y, work, wb, rows, cols, k, n_pts, None)

    for kw in (dict(batch=0), dict(batch=129), dict(cols=100), dict(cols=65536), dict(cols=0), dict(rows=0),
               dict(k=17), dict(k=4), dict(n_pts=0), dict(n_pts=257), dict(codes=odd), dict(y=odd),
               dict(work=odd), dict(x=None), dict(codes=None), dict(x=ctypes.c_void_p(0x100008)),
               dict(work=ctypes.c_void_p(0x100100)), dict(wb=1024)):
        assert mm(**kw) == -1, kw

    def mv(x=A, codes=A, y=A, rows=64, cols=128, k=0, n_pts=217, U=None, tmp=None):
        return lib.gsdlq_hex2d_matvec_noalloc(x, codes, A, A, U, tmp, A, A, A, y, rows, cols, k, n_pts, None)

    for kw in (dict(n_pts=0), dict(n_pts=257), dict(k=4), dict(k=17, U=A, tmp=A), dict(cols=100), dict(rows=0),
               dict(codes=odd), dict(x=None), dict(y=None), dict(x=odd)):
        assert mv(**kw) == -1, kw
    # one strip more than the fixed scratch holds: refused as unsupported, still before any CUDA call
    assert mv(rows=16 * (31769 + 1), cols=64) == -3


def test_header_is_c99_and_links_from_c(tmp_path):
    """include/gsdlq.h compiles as pedantic C99, and a C program links libgsdlq_cuda.so and calls its
    host-only entry points (version, status strings, codebook, RoPE table) without a GPU."""
    import shutil
    import subprocess
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    inc, libdir = os.path.join(root, "include"), os.path.dirname(L.load()._name)
    src = tmp_path / "use_gsdlq.c"
    src.write_text(r'''
#include <stdio.h>
#include "gsdlq.h"
int main(void) {
  float xy[2 * 256];
  float rope[4 * 8 * 2];
  int n6 = gsdlq_codebook(6, xy, 256), n8 = gsdlq_codebook(8, xy, 256);
  int st = gsdlq_rope_table(rope, 4, 16, 10000.0f);
  printf("%s|%s|%d|%d|%d|%d\n", gsdlq_version(), gsdlq_status_string(GSDLQ_ERR_INVALID), n6, n8, st,
         gsdlq_hex2d_matvec(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 16, 64, 0, 217, 0));
  return 0;
}
''')
    exe = tmp_path / "use_gsdlq"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", inc, str(src), "-o", str(exe),
                        "-L", libdir, "-lgsdlq_cuda", "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    ver, msg, n6, n8, st, bad = out.stdout.strip().split("|")
    assert ver.startswith("0.") and msg == "invalid argument"
    assert (int(n6), int(n8), int(st), int(bad)) == (127, 217, 0, -1)
