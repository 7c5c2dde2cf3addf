"""The allocation-free talker decode step (qtts_talker_decode_step_static).

It exists for hosts that may not allocate device memory once running; it must
give the same hidden state, logits and token as qtts_talker_decode_step. Two
calls in a row are checked, so the second call sees the static working
memory the first one left behind. Collected last on purpose (file name)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2  # same tolerance as the other GPU parity tests


@pytest.mark.parametrize("shape", ["tiny", "tiny_proj"])
def test_static_scratch_step_matches_regular_step(pkg, model_dirs, oracles, shape):
    e = pkg.HipTtsEngine.load_with_options(model_dirs[shape], pkg.EngineOptions(0, 64))
    m = oracles[shape]
    ids = np.random.default_rng(21).integers(0, 4000, 9)
    pre, _, _ = m.prepare(list(ids))
    e.talker_prefill(pre.numpy())
    P = pre.shape[0]
    rng = np.random.default_rng(22)
    for off in (P, P + 1):  # two calls in a row
        x = (rng.standard_normal(e.hidden) * 0.05).astype(np.float32)
        h_ref, l_ref, t_ref = e.talker_decode_step(x, off)
        h_st, l_st, t_st = e.talker_decode_step_static(x, off)
        assert np.abs(h_st - h_ref).max() <= LOGIT_TOL
        assert np.abs(l_st - l_ref).max() <= LOGIT_TOL
        assert t_st == t_ref
    e.close()
