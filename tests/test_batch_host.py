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


def _run_bench(args, env_extra=None):
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(root, "bench.py")] + args, capture_output=True, text=True,
                          env=env, timeout=300, cwd=root)


def test_reference_arm_prints_the_contract_line():
    """bench.py --impl reference (the reference's C engine on the host cores) prints one JSON line with the
    contract's keys, its own cpu_baseline and an e2e that moves no bytes over PCIe; ranks other than 0 exit
    quietly."""
    import json
    r = _run_bench(["--impl", "reference", "--model", "tiny", "--prompt", "16", "--steps", "2", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    j = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in j, k
    assert j["impl"] == "reference" and j["unit"] == "tok/s" and j["value"] > 0 and j["n_gpus"] == 1
    assert j["steps"] == 2 and j["warmup"] == 3 and j["higher_is_better"] is True
    assert j["metric"] == "decode tok/s batch1 tiny-shape Precision" and j["config"]["global_batch"] == 1
    cb = j["cpu_baseline"]
    assert cb["value"] == j["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert j["e2e"] == {"value": j["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    r = _run_bench(["--impl", "reference", "--model", "tiny", "--prompt", "16", "--steps", "2", "--warmup", "3"],
                   {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0 and not r.stdout.strip(), (r.stdout, r.stderr[-2000:])


def _bench_module():
    import importlib.util
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("bench_mod_clocks", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


def test_clock_sampler_reads_nvidia_smi_lines(tmp_path, monkeypatch):
    """The bench's clock record (median SM clock, max clock, active slowdown reasons) from nvidia-smi's CSV
    stream, here a stand-in script on PATH; malformed lines are skipped; no nvidia-smi at all gives an
    explicit 'unavailable' record."""
    import os
    import time
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/sh\ncat <<'EOF'\n"
                    "0, 1965, 1965, 700.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
                    "0, 1950, 1965, 990.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n"
                    "0, [N/A], 1965, 991.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
                    "partial, line\n"
                    "0, 1800, 1965, 995.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n"
                    "EOF\nexec sleep 30\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    bench = _bench_module()
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    assert s.stop() == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    empty = tmp_path / "empty"
    empty.mkdir()
    monkeypatch.setenv("PATH", str(empty))
    s = bench.ClockSampler(0)
    s.start()
    r = s.stop()
    assert r["samples"] == 0 and r["sm_mhz"] is None and r["reasons"] == ["nvidia-smi unavailable"]


def test_prefill_roofline_counts_linear_and_causal_attention_flops():
    """The bench's prefill tensor roofline: 2 flops per layer weight per token plus 4 * heads * head_dim per
    causal query-key pair, counted here by brute force over the tokens."""
    import gsdlq_b200.packer as P
    bench = _bench_module()
    cfg = P.make_config("qwen2.5-1.5b")
    shapes = P.linear_shapes(cfg)
    T, L = 37, cfg["n_layers"]
    weights = L * sum(r * c for r, c in shapes.values())
    flops = 2 * weights * T + sum(L * 4 * cfg["n_heads"] * cfg["head_dim"] * (t + 1) for t in range(T))
    r = bench.prefill_roofline(cfg, T, 0.5, {"bf16_tflops": 1000.0}, "measured", sequences=3)
    assert r["flops"] == 3 * flops and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - 3 * flops / 0.5 / 1e12) < 1e-9 and abs(r["frac"] - r["achieved"] / 1000.0) < 1e-12


def test_batch_decoder_refuses_bad_setups_before_allocating():
    """BatchDecoder checks tensor parallelism, the batch range, the attention shapes and the cache length
    on the host, before it touches the device (a stand-in model: nothing here needs a GPU)."""
    import types
    import pytest
    from gsdlq_b200.batch import BatchDecoder
    ok = dict(tp=None, batched_prefill_supported=True, max_seq=256)
    with pytest.raises(NotImplementedError, match="one GPU"):
        BatchDecoder(types.SimpleNamespace(**{**ok, "tp": object()}), 4)
    for b in (0, 129):
        with pytest.raises(ValueError, match="batch must be"):
            BatchDecoder(types.SimpleNamespace(**ok), b)
    with pytest.raises(NotImplementedError, match="head_dim"):
        BatchDecoder(types.SimpleNamespace(**{**ok, "batched_prefill_supported": False}), 4)
    with pytest.raises(ValueError, match="max_seq"):
        BatchDecoder(types.SimpleNamespace(**ok), 4, max_seq=512)


def test_generate_refuses_bad_arguments_before_the_device():
    """GSDLQModel.generate's host checks (empty prompt, cache length, check interval, reuse position, device
    sampling under tensor parallelism) run before any device work: here on a stand-in model object."""
    import types
    import pytest
    from gsdlq_b200.model import GSDLQModel
    m = types.SimpleNamespace(max_seq=32, tp=None)
    gen = GSDLQModel.generate
    with pytest.raises(ValueError, match="at least one token"):
        gen(m, [], 4)
    with pytest.raises(ValueError, match="exceed max_seq"):
        gen(m, [1] * 30, 3)
    with pytest.raises(ValueError, match="exceed max_seq"):
        gen(m, [1, 2], -1)
    with pytest.raises(ValueError, match="check_every"):
        gen(m, [1, 2], 4, check_every=0)
    for sp in (-1, 2, 5):
        with pytest.raises(ValueError, match="start_pos"):
            gen(m, [1, 2], 4, start_pos=sp)
    with pytest.raises(NotImplementedError, match="whole vocabulary"):
        gen(types.SimpleNamespace(max_seq=32, tp=object()), [1, 2], 4, temperature=0.7)
