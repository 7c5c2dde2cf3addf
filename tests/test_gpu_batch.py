"""Batched serving (qtts_generate_codes_batch_from_ids): several requests
stepped in lockstep with tensor-core projections over all rows. Each request
is checked against the CPU oracle on its own, teacher-forced along the GPU's
codes (tokens identical wherever the oracle's top-2 gap exceeds 1e-2)."""
import numpy as np
import pytest

from oracle import qtts_oracle as O
from parity import check_codes

pytestmark = pytest.mark.gpu

GAP = 1e-2
GREEDY = O.SamplingConfig(False, 0, 1.0, 1.0)
SAMPLED = O.SamplingConfig(True, 50, 1.0, 0.9)
SHAPES = ["tiny", "tiny_proj"]
LENGTHS = [5, 12, 20]


@pytest.fixture(scope="module")
def engines(pkg, model_dirs):
    out = {s: pkg.HipTtsEngine.load_with_options(model_dirs[s], pkg.EngineOptions(0, 128))
           for s in SHAPES}
    yield out
    for e in out.values():
        e.close()


def requests(seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 4000, n) for n in LENGTHS]


def gaps_per_code(records):
    return [g for r in records for g in [r.talker_gap] + r.cp_gaps]


@pytest.mark.parametrize("shape", SHAPES)
def test_batch_greedy_matches_oracle(engines, oracles, pkg, shape):
    e, m = engines[shape], oracles[shape]
    reqs = requests(5)
    opts = [pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                                repetition_penalty=1.0, max_frames=12) for _ in reqs]
    outs = e.generate_codes_batch_from_ids(reqs, opts)
    assert len(outs) == len(reqs)
    for ids, out in zip(reqs, outs):
        assert out.frames == 12 and len(out.codes) == 12 * 16
        pre, tr, pad = m.prepare(list(ids))
        codes, _, recs = m.rollout(pre, tr, pad, 12, GREEDY, GREEDY, forced_codes=out.codes)
        gaps = gaps_per_code(recs)
        hard = [i for i, (a, b) in enumerate(zip(out.codes, codes)) if a != b and gaps[i] > GAP]
        assert not hard, (shape, hard[:10])


@pytest.mark.parametrize("shape", SHAPES)
def test_batch_sampled_per_request_seeds(engines, oracles, pkg, shape):
    e, m = engines[shape], oracles[shape]
    reqs = requests(6)
    opts = [pkg.GenerateOptions(decode_audio=False, max_frames=10, seed=b, rng="philox")
            for b in range(len(reqs))]
    outs = e.generate_codes_batch_from_ids(reqs, opts)
    for b, (ids, out) in enumerate(zip(reqs, outs)):
        pre, tr, pad = m.prepare(list(ids))
        codes, _, recs = m.rollout(pre, tr, pad, 10, SAMPLED, SAMPLED, penalty=1.05, seed=b,
                                   rng_kind="philox", forced_codes=out.codes)
        check_codes(out.codes, codes, recs, f"batch {shape} request {b}", sampled=True)


def test_batch_matches_single_requests(engines, pkg):
    """Each request of a batch against the same request generated alone. The
    prefill (and so frame 0's semantic token) runs the same kernels either way;
    later tokens come from different projection kernels and are free-running
    here, so their parity is the oracle tests' job, not this one's."""
    e = engines["tiny"]
    reqs = requests(7)
    opts = [pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                                repetition_penalty=1.0, max_frames=8) for _ in reqs]
    outs = e.generate_codes_batch_from_ids(reqs, opts)
    for ids, o, out in zip(reqs, opts, outs):
        single = e.generate_codes_from_ids(ids, o)
        assert out.frames == single.frames == 8
        assert out.codes[0] == single.codes[0]


def test_batch_errors(engines, pkg):
    e = engines["tiny"]
    with pytest.raises(pkg.InvalidInput):
        e.generate_codes_batch_from_ids([[1, 2]] * 17,
                                        [pkg.GenerateOptions(decode_audio=False)] * 17)
    with pytest.raises(pkg.InvalidInput):
        e.generate_codes_batch_from_ids(
            [[1, 2], [3, 4]],
            [pkg.GenerateOptions(decode_audio=False, top_k=50),
             pkg.GenerateOptions(decode_audio=False, top_k=40)])


@pytest.mark.parametrize("shape", ["0.6b", "1.7b"])
def test_batch_of_one_matches_single_full_size(pkg, full_model_dir, shape):
    """A one-request batch against the same request generated alone, greedy, at
    the full shapes: both must agree with the oracle's choices (gap-gated)."""
    from parity import check_codes

    d = full_model_dir(shape)
    e = pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 128))
    m = O.OracleModel(d, 128)
    ids = np.random.default_rng(31).integers(0, 150000, 20)
    opts = pkg.GenerateOptions(decode_audio=False, do_sample=False, subtalker_dosample=False,
                               repetition_penalty=1.0, max_frames=3)
    single = e.generate_codes_from_ids(ids, opts)
    (batch,) = e.generate_codes_batch_from_ids([ids], [opts])
    pre, tr, pad = m.prepare(list(ids))
    for label, out in (("single", single), ("batch of 1", batch)):
        codes, _, recs = m.rollout(pre, tr, pad, 3, GREEDY, GREEDY, forced_codes=out.codes)
        check_codes(out.codes, codes, recs, f"{shape} {label}")
    e.close()
