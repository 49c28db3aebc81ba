"""The execution-plan report and compilation schema of the B200 lowering
(the reference's emit_inspect, tikun-py/src/lib.rs:88-113, and
CompilationSchema, tikun-core/src/schema.rs:78-184), on CPU."""
import json

import pytest

from tikun_b200 import _native
from tikun_b200.inspect import compilation_schema, emit_inspect, emit_schema


def test_schema_traffic_and_dispatch():
    ptrs, lens = [0x1000, 0x2040, 0x3008], [1000, 17, 4097]
    sc = compilation_schema(ptrs, lens, "adamw", 0.0, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    n = sum(lens)
    # schema.rs:127-129: 16 B read and 12 B written per AdamW element
    assert sc["performance_metrics"]["bytes_read_per_step"] == 16 * n
    assert sc["performance_metrics"]["bytes_written_per_step"] == 12 * n
    assert sc["memory_topography"]["total_parameters"] == n
    assert [s["cache_aligned"] for s in sc["memory_topography"]["slots"]] == [True, True, False]
    assert not sc["memory_topography"]["is_cache_aligned"]
    assert sc["target_architecture"].endswith("sm_100a)")
    # the clip adds the Tier-1 read of g
    clipped = compilation_schema(ptrs, lens, "AdamW", 1.0, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    assert clipped["performance_metrics"]["bytes_read_per_step"] == 20 * n
    assert clipped["execution_schedule"]["passes"][0]["pass_name"] == "sumsq_partials"
    # build_spec's dispatch: "lion", "sgd", anything else AdamW
    assert compilation_schema(ptrs, lens, "LION", 0, 1, 1, 1, 1, 0)["optimizer"]["algorithm"] == "Lion"
    assert compilation_schema(ptrs, lens, "sgd", 0, 1, 1, 1, 1, 0)["optimizer"]["algorithm"] == "SGD"
    assert compilation_schema(ptrs, lens, "adam", 0, 1, 1, 1, 1, 0)["optimizer"]["algorithm"] == "AdamW"
    json.loads(emit_schema(ptrs, lens, "adamw", 0.0, 1e-3, 0.9, 0.999, 1e-8, 0.01))


def test_inspect_report():
    ptrs = [64 * i for i in range(300)]
    lens = [768] * 300
    text = emit_inspect(ptrs, lens, "adamw", 1.0, 1e-3, 0.9, 0.999, 1e-8, 0.01)
    assert "Hardware Execution Plan" in text and "sm_100a" in text
    assert "2 x pointwise_kernel" in text  # 300 leaves, 224 per launch
    assert "... and 292 additional parameter slots" in text
    assert "load_p_g" in text and "store_p" in text
    with pytest.raises(_native.TikunValueError):
        emit_inspect([0], [1, 2], "adamw", 0.0, 1e-3, 0.9, 0.999, 1e-8, 0.01)


def test_optimizer_state_roundtrip_and_report_on_cpu():
    """state_dict/load_state_dict keep m1/m2 in parameter order (the step
    itself needs a GPU and is tested there); to_json gives the plan report."""
    import numpy as np

    from tikun_b200.universal import UniversalOptimizer, _extract_pointer_and_len

    ps = [np.zeros(10, np.float32), np.zeros(5, np.float32)]
    opt = UniversalOptimizer(ps, max_norm=1.0)
    ptr, n = _extract_pointer_and_len(ps[0])
    opt._state_for(ps[0], ptr, n)
    opt.m1_state[ptr][:] = 3.0
    opt.m2_state[ptr][:] = 2.0
    opt.step_count = 7
    sd = opt.state_dict()
    assert sd["step"] == 7 and sd["m1"][1] is None
    qs = [np.zeros(10, np.float32), np.zeros(5, np.float32)]
    opt2 = UniversalOptimizer(qs)
    opt2.load_state_dict(sd)
    p2, _ = _extract_pointer_and_len(qs[0])
    assert opt2.step_count == 7
    assert (opt2.m1_state[p2] == 3.0).all() and (opt2.m2_state[p2] == 2.0).all()
    with pytest.raises(ValueError):
        UniversalOptimizer([np.zeros(10, np.float32)]).load_state_dict(sd)
    assert "Hardware Execution Plan" in opt2.to_json()
    with pytest.raises(NotImplementedError):
        opt2.to_mlir()
