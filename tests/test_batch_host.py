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


def test_integer_coordinates_times_transformed_activations_equal_the_dequantised_product():
    """The small-batch GEMM multiplies each code's integer lattice coordinates (r0, r1) by the activations
    transformed as (a, b) = (x0, x0 / 2 + sqrt3/2 x1) and applies the group scale afterwards; that equals the
    reference's dequantised weights (xy[code] * scale) times x (gsd_lq_cpu_runtime.py dequant definition)."""
    import oracle
    rng = np.random.default_rng(3)
    for radius in (6, 8):
        xy, n_pts = oracle.codebook(radius)
        xy = np.asarray(xy, np.float64).reshape(-1, 2)[:n_pts]
        r1 = np.rint(xy[:, 1] / (np.sqrt(3.0) / 2.0))
        r0 = xy[:, 0] - 0.5 * r1
        assert np.all(r0 == np.rint(r0)) and np.all(np.abs(r0) <= radius) and np.all(np.abs(r1) <= radius)
        codes = rng.integers(0, n_pts, 32)
        x = rng.standard_normal((32, 2))
        s = 0.0123
        want = s * np.sum(xy[codes, 0] * x[:, 0] + xy[codes, 1] * x[:, 1])
        a, b = x[:, 0], 0.5 * x[:, 0] + (np.sqrt(3.0) / 2.0) * x[:, 1]
        got = s * np.sum(r0[codes] * a + r1[codes] * b)
        # equal up to the table's float32 rounding of r1 sqrt3/2 (2^-24 relative per entry)
        assert abs(got - want) <= 2e-7 * s * np.sum(np.abs(xy[codes]) * np.abs(x))


def test_bench_metric_and_config_names(monkeypatch):
    import importlib.util
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)

    class A:
        sweep, batch, model, mode, prompt, max_seq = False, 1, "mistral-7b", "precision", 1536, 2048
    a = A()
    assert bench.metric_name(a) == bench.METRIC  # the headline configuration keeps BASELINE's metric
    c = bench.workload_config(a, 1)
    assert c["global_batch"] == 1 and c["parallelism"] == "tp1" and "batch 1" in c["workload"]
    a.batch, a.model, a.mode, a.prompt = 16, "smollm2-1.7b", "turbo", 1024
    assert bench.metric_name(a) == "decode tok/s batch16 smollm2-1.7b-shape Turbo"
    c = bench.workload_config(a, 1)
    assert c["global_batch"] == 16 and "2048-entry KV cache" in c["workload"]
    a.sweep = True
    assert "GB/s" in bench.metric_name(a)
    assert bench.workload_config(a, 1)["shapes"] == [list(s) for s in bench.SWEEP_SHAPES]
