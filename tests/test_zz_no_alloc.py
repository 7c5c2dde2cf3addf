"""The allocation-free talker decode step (qtts_talker_decode_step_static).

It serves hosts that may not allocate device memory once running (a fixed
budget carved out at start-up, or a runtime where cudaMalloc would stall other
work on the device). It runs the same kernels as qtts_talker_decode_step, only
over a static device array, so its hidden state, logits and token must equal
the regular step's bit for bit; both are also checked against the CPU oracle.
Two calls in a row are checked, so the second call runs over the working
memory the first one left behind. Collected last on purpose (file name)."""
import numpy as np
import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2  # same tolerance as the other GPU parity tests


@pytest.mark.parametrize("shape", ["tiny", "tiny_proj"])
def test_static_scratch_step_matches_regular_step(pkg, model_dirs, oracles, shape):
    e = pkg.HipTtsEngine.load_with_options(model_dirs[shape], pkg.EngineOptions(0, 64))
    m = oracles[shape]
    ids = np.random.default_rng(21).integers(0, 4000, 9)
    pre, _, _ = m.prepare(list(ids))
    e.talker_prefill(pre.numpy())
    m.talker_prefill(pre)
    P = pre.shape[0]
    rng = np.random.default_rng(22)
    for off in (P, P + 1):  # two calls in a row
        x = (rng.standard_normal(e.hidden) * 0.05).astype(np.float32)
        h_ref, l_ref, t_ref = e.talker_decode_step(x, off)
        free0 = torch.cuda.mem_get_info(0)[0]
        h_st, l_st, t_st = e.talker_decode_step_static(x, off)
        free1 = torch.cuda.mem_get_info(0)[0]
        assert free1 == free0, "the static step changed the device's free memory"
        np.testing.assert_array_equal(h_st, h_ref)
        np.testing.assert_array_equal(l_st, l_ref)
        assert t_st == t_ref
        _, rh, rl = m.talker_step(torch.from_numpy(x), off)
        assert np.abs(h_st - rh.numpy()).max() <= LOGIT_TOL
        assert np.abs(l_st - rl).max() <= LOGIT_TOL
    e.close()


def test_static_step_rejects_oversized_talker(pkg, tmp_path):
    """A talker whose step activations exceed the static array is refused
    before anything is launched."""
    d = synth.write_model(tmp_path / "wide", "tiny_wide", 0)
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 16))
    x = np.zeros(e.hidden, np.float32)
    with pytest.raises(pkg.InvalidInput, match="static array"):
        e.talker_decode_step_static(x, 0)
    e.close()
