"""The step trace through the C ABI (qtts_step_trace_enable / _read), which
bench.py uses for its per-kernel roofline: one traced frame of the live frame
graph lists every launch of the frame in order with consistent stamps, and
tracing leaves the generated codes unchanged."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_step_trace_of_one_frame(pkg, model_dirs):
    e = pkg.HipTtsEngine.load_with_options(model_dirs["tiny"], pkg.EngineOptions(0, 128))
    try:
        ids = np.random.default_rng(31).integers(0, 4000, 10)
        opts = pkg.GenerateOptions(decode_audio=False, max_frames=9, seed=2)
        groups = e.info.num_code_groups
        plain = e.generate_codes_from_ids(ids, opts)
        e.step_trace_enable(True)
        traced = e.generate_codes_from_ids(ids, opts)
        rows = e.step_trace()
        e.step_trace_enable(False)
        again = e.generate_codes_from_ids(ids, opts)
    finally:
        e.close()
    assert list(traced.codes) == list(plain.codes) == list(again.codes)
    assert len(rows) > 20
    kinds = {r["name"].rsplit(" ", 2)[0] for r in rows}
    assert {"gemv", "gemv+swiglu", "gemv+resid", "cp head+select"} <= kinds
    # one head per acoustic group
    assert sum(r["name"].startswith("cp head") for r in rows) == groups - 1
    waits = [r["wait_ns"] for r in rows]
    assert all(w >= 0 for w in waits)
    assert waits == sorted(waits)  # each launch passes its wait after its predecessor's
    for r in rows:
        assert 0 <= r["entry_ns"] <= r["wait_ns"] <= r["exit_ns"], r
