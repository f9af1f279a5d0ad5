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
  size_t mm = 0, at = 0, sp = 0;
  int w1 = gsdlq_hex2d_matmul_work_size(16, 4096, &mm), w2 = gsdlq_attention_rows_work_size(128, 32, 128, &at);
  int w3 = gsdlq_sample_work_size(32768, &sp);
  printf("%s|%s|%d|%d|%d|%d|%d %zu|%d %zu|%d %zu\n", gsdlq_version(), gsdlq_status_string(GSDLQ_ERR_INVALID), n6,
         n8, st, gsdlq_hex2d_matvec(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 16, 64, 0, 217, 0), w1, mm, w2, at, w3, sp);
  return 0;
}
''')
    exe = tmp_path / "use_gsdlq"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", inc, str(src), "-o", str(exe),
                        "-L", libdir, "-lgsdlq_cuda", "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    ver, msg, n6, n8, st, bad, mm, at, sp = out.stdout.strip().split("|")
    assert ver.startswith("0.") and msg == "invalid argument"
    assert (int(n6), int(n8), int(st), int(bad)) == (127, 217, 0, -1)
    # the work sizes seen from C equal those seen through ctypes
    lib = L.load()
    for got, fn, args in ((mm, lib.gsdlq_hex2d_matmul_work_size, (16, 4096)),
                          (at, lib.gsdlq_attention_rows_work_size, (128, 32, 128)),
                          (sp, lib.gsdlq_sample_work_size, (32768,))):
        n = ctypes.c_size_t()
        assert fn(*args, ctypes.byref(n)) == 0
        status, size = got.split()
        assert int(status) == 0 and int(size) == n.value > 0


def test_row_batch_and_sampling_argument_errors_before_launch():
    """The prefill row kernels, the batched-decode kernels and the sampler refuse bad shapes, strides and
    alignments on the host before any CUDA call (the stand-in addresses are never dereferenced)."""
    lib = L.load()
    A = ctypes.c_void_p(0x100000)
    odd = ctypes.c_void_p(0x100004)      # 4-byte but not 16-byte aligned
    nb = ctypes.c_size_t()

    # work sizes are host arithmetic: the exact figures the callers allocate
    assert lib.gsdlq_sample_work_size(1000, ctypes.byref(nb)) == 0 and nb.value == 4000
    assert lib.gsdlq_sample_work_size(0, ctypes.byref(nb)) == -1
    assert lib.gsdlq_sample_work_size(10, None) == -1
    assert lib.gsdlq_attention_rows_work_size(5, 4, 64, ctypes.byref(nb)) == 0 and nb.value == 4 * 8 * 5 * 4 * 66
    assert lib.gsdlq_attention_rows_work_size(0, 4, 64, ctypes.byref(nb)) == -1
    work_ok = nb.value

    def smp(logits=A, n=100, u=A, work=A, wb=400, key=A, idx=None):
        return lib.gsdlq_sample_top_p(logits, n, 0.7, 0.9, u, None, work, wb, key, idx, None)

    for kw in (dict(logits=None), dict(n=0), dict(u=None), dict(work=None), dict(wb=396), dict(key=None),
               dict(work=ctypes.c_void_p(0x100002))):
        assert smp(**kw) == -1, kw

    def rows(q=A, k=A, v=A, out=A, work=A, wb=work_ok, pos0=0, n=5, nh=4, nkv=2, hd=64, max_seq=16):
        return lib.gsdlq_attention_rows(q, k, v, out, work, wb, 0, pos0, n, nh, nkv, hd, max_seq, 0.125, None)

    for kw in (dict(q=None), dict(n=0), dict(pos0=-1), dict(pos0=12), dict(nkv=3), dict(nh=16, nkv=1),
               dict(hd=96), dict(hd=32), dict(q=odd), dict(out=odd), dict(work=odd), dict(wb=work_ok - 4)):
        assert rows(**kw) == -1, kw

    seq = 2 * 16 * 2 * 64  # (layer + 1) * max_seq * n_kv * head_dim for layer 1

    def dec(q_stride=0, k=A, work=A, wb=1 << 20, layer=1, batch=3, nh=4, nkv=2, hd=64, seq_stride=seq):
        return lib.gsdlq_attention_decode_batch(A, q_stride, k, A, seq_stride, A, work, wb, layer, A, batch, nh, nkv,
                                                hd, 16, 0.125, None)

    for kw in (dict(batch=0), dict(layer=-1), dict(nh=6, nkv=2), dict(nh=16, nkv=1), dict(hd=32),
               dict(seq_stride=seq - 1), dict(seq_stride=seq + 1), dict(k=odd), dict(work=odd),
               dict(q_stride=-1), dict(q_stride=4 * 64 - 1), dict(wb=16)):
        assert dec(**kw) == -1, kw

    def rkb(row_stride=0, hd=64, seq_stride=seq, layer=1, batch=3):
        return lib.gsdlq_rope_kv_batch(A, A, A, row_stride, A, A, seq_stride, A, layer, A, batch, 4, 2, hd, 16, None)

    for kw in (dict(hd=63), dict(seq_stride=seq - 1), dict(row_stride=-1), dict(row_stride=100), dict(batch=0),
               dict(layer=-1)):
        assert rkb(**kw) == -1, kw
    assert lib.gsdlq_rope_kv_rows(A, A, A, A, A, A, 0, 10, 7, 4, 2, 64, 16, None) == -1   # 10 + 7 > 16
    assert lib.gsdlq_embed_rows(A, A, 0, 32, 64, A, None) == -1
    assert lib.gsdlq_rmsnorm_rows(A, A, A, 2, 0, 1e-5, None) == -1
    assert lib.gsdlq_swiglu_rows(A, A, 0, 64, None) == -1
    assert lib.gsdlq_argmax_rows(A, 2, 100, A, None, A, 16, None) == -1   # out_ids without positions
    assert lib.gsdlq_argmax_rows(A, 2, 100, A, A, A, 0, None) == -1
    assert lib.gsdlq_advance_eos(A, A, A, A, None, 0, 2, None, None) == -1


def test_matvec_width_limit_refused_before_launch():
    """Rows wider than GSDLQ_MATVEC_MAX_COLS (the fused matvec holds a whole input row in shared memory)
    are refused as unsupported by the no-allocation matvec, before any device work.  (The drop-in matvec
    takes them through the dequant-GEMM instead, so it is not called here with stand-in pointers.)"""
    import re
    lib = L.load()
    hdr = open(L.HEADER).read()
    limit = int(re.search(r"#define GSDLQ_MATVEC_MAX_COLS (\d+)", hdr).group(1))
    assert limit % 64 == 0 and 32768 <= limit < 65472
    A = ctypes.c_void_p(0x100000)
    for cols in (limit + 64, 65472):
        for rows in (16, 4096):
            assert lib.gsdlq_hex2d_matvec_noalloc(A, A, A, A, None, None, A, A, A, A, rows, cols, 0, 217,
                                                  None) == -3
