"""bench.py's workload definitions and CPU reference arms, on CPU: the
configurations are the ones the headline metric and the parity cases name, and
the reference arms run (on tiny stand-ins) and describe their sample."""
import os
import sys


sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from tikun_b200.sharding import ns_dense_flops  # noqa: E402


def test_workload_shapes():
    g = bench.WORKLOADS["gpt2-small-clip"]
    assert len(g["sizes"]) == 148 and sum(g["sizes"]) == 124_439_808 and g["max_norm"] == 1.0
    assert bench.WORKLOADS["flat-100m"]["sizes"] == [100_000_000]
    m2 = bench.MUON["muon-gpt2-d768"]
    assert len(m2["mats"]) == 72 and m2["adamw"][0] == 50257 * 768
    assert abs(sum(ns_dense_flops(r, c) for r, c in m2["mats"]) / 1e12 - 1.631) < 0.01
    m3 = bench.MUON["muon-1.3b-inbackward"]
    assert m3["inbackward"] and m3["layers"] == 24 and len(m3["mats"]) == 24 * 6
    m4 = bench.MUON["muon-llama3-8b"]
    assert len(m4["mats"]) == 224 and m4["adamw"][:2] == [128256 * 4096] * 2
    assert abs(sum(ns_dense_flops(r, c) for r, c in m4["mats"]) / 1e12 - 665.9) < 0.05


def test_ns_scratch_bytes_follow_the_library_layout():
    # two X^T and A, A', B: 2(2mn + 3m^2) bytes for 64-multiple shapes, plus
    # 256 f64 norm partials, the scale and the 256-byte tail
    m, n = 4096, 14336
    assert bench.ns_scratch_bytes(m, n) == 2 * (2 * m * n + 3 * m * m) + 8 * 256 + 256 + 256
    # split f16 operands: the 16-bit buffers twice as wide
    assert bench.ns_scratch_bytes(m, n, split=True) == 4 * (2 * m * n + 3 * m * m) + 8 * 256 + 512
    # padding: a 17 x 45 matrix uses 64-element rows
    assert bench.ns_scratch_bytes(17, 45) >= 2 * (2 * 45 * 64 + 3 * 17 * 64)


def test_cpu_reference_arms_run_on_tiny_workloads():
    tiny = dict(sizes=[1000, 17, 4097], kinds=["w", "b", "w"], max_norm=1.0, g_std=1e-2,
                desc="tiny")
    value, ms, warm, steps = bench.cpu_reference_run(tiny, 2, 1, 2)
    assert value > 0 and ms > 0 and (warm, steps) == (1, 2)
    # the chunked (non-reference) schedule processes the same elements
    cval, cms, _, _ = bench.cpu_reference_run(tiny, 2, 1, 2, chunk=1000)
    assert cval > 0 and cms > 0
    # a time budget far below one step cuts both phases to one step
    value, ms, warm, steps = bench.cpu_reference_run(tiny, 50, 5, 2, budget_s=1e-9)
    assert (warm, steps) == (1, 1)
    muon = dict(mats=[(64, 96), (96, 64), (256, 512)], adamw=[300, 64], layers=1,
                inbackward=False, desc="tiny muon")
    value, ms, sample = bench.cpu_muon_run(muon, 2, steps=2, warmup=1)
    assert value > 0 and ms > 0 and "one matrix per shape group" in sample
    assert "timed at" not in sample
    # a budget below the largest matrix forces a scaled-down timing, and long
    # AdamW leaves are cut and scaled by the element ratio
    secs, sample = bench.cpu_muon_sample(muon, 2, budget_flops=1e7, aw_cap=100)
    assert secs > 0 and "timed at" in sample and "first 100 elements" in sample


def test_reference_arm_prints_the_contract_line(monkeypatch, capsys):
    import json

    tiny = dict(sizes=[1000, 17, 4097], kinds=["w", "b", "w"], max_norm=1.0, g_std=1e-2,
                desc="tiny")
    monkeypatch.setitem(bench.WORKLOADS, "gpt2-small-clip", tiny)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--workload",
                                      "gpt2-small-clip", "--steps", "4", "--warmup", "3"])
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    bench.main()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 4 and d["warmup"] == 3
    # the same config dict the GPU arm prints for this workload
    assert d["config"] == bench.pointwise_config("gpt2-small-clip", tiny)
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["cpu_model"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # another rank under torchrun prints nothing and does no work
    monkeypatch.setenv("RANK", "1")
    bench.main()
    assert not [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]


def test_muon_reference_arm_prints_the_contract_line(monkeypatch, capsys):
    import json

    tiny = dict(mats=[(64, 96), (96, 64), (128, 128)], adamw=[300, 64], layers=1,
                inbackward=False, desc="tiny muon")
    monkeypatch.setitem(bench.MUON, "muon-gpt2-d768", tiny)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--workload",
                                      "muon-gpt2-d768", "--steps", "2", "--warmup", "3"])
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    bench.main()
    lines = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["cpu_baseline"]["cpu_model"]
    # the requested steps and warm-up, and the config dict the GPU arm prints
    assert d["steps"] == 2 and d["warmup"] == 3
    assert d["config"] == bench.muon_config("muon-gpt2-d768", tiny)
    assert d["e2e"]["h2d_bytes_per_step"] == 0


def test_default_workload_is_the_largest_single_gpu_config(monkeypatch):
    """With no --workload the bench runs the Llama-3-8B-shaped Muon+AdamW step."""
    import argparse

    seen = {}

    def fake_parse(self, args=None, namespace=None):
        ns = real_parse(self, [] if args is None else args, namespace)
        seen["workload"] = ns.workload
        raise SystemExit(0)

    real_parse = argparse.ArgumentParser.parse_args
    monkeypatch.setattr(argparse.ArgumentParser, "parse_args", fake_parse)
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    try:
        bench.main()
    except SystemExit:
        pass
    assert seen["workload"] == "muon-llama3-8b"
