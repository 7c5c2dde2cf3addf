"""Full-size, full-length parity at the benchmarked configurations.

Each test runs one BASELINE configuration through the C ABI on the GPU and
checks every code against the CPU oracle, teacher-forced along the GPU's
codes (tests/parity.py: greedy tokens must match wherever the oracle's top-2
gap exceeds 1e-2; sampled tokens wherever the oracle's inverse-CDF target is
more than 2e-3 of the mass from a bucket edge). Each prints the fraction of
codes under the exemption.

* cfg 1 (north-star target): 0.6B, 32 ids, greedy, 240 frames
* cfg 2 (the bench line): 0.6B, 64 ids, 240 frames, top-k 50, T 0.9,
  penalty 1.05, subtalker top-k 50 T 0.9, Philox seed 0
* cfg 3: 1.7B, 128 ids, greedy, 240 frames
* cfg 4: 0.6B text stream, 8-id pushes, 6-frame chunks, min_start_tokens 1
* cfg 5: 16 requests at 1.7B, prompts uniform in [16, 256], config-1
  sampling, Philox seed = request index, 8 frames each
Random weights may reach EOS early; the oracle must then end at the same frame.
"""
import numpy as np
import pytest

from oracle import qtts_oracle as O
from parity import check_codes, check_end

pytestmark = pytest.mark.gpu

GREEDY = O.SamplingConfig(False, 0, 1.0, 1.0)
SAMPLED = O.SamplingConfig(True, 50, 1.0, 0.9)
VOCAB = 150000


def _ids(seed, n):
    return np.random.default_rng(seed).integers(0, VOCAB, n)


@pytest.fixture(scope="module")
def full(pkg, full_model_dir):
    made = {}

    def get(shape):
        if shape not in made:
            d = full_model_dir(shape)
            made[shape] = (pkg.HipTtsEngine.load_with_options(d, pkg.EngineOptions(0, 512)),
                           O.OracleModel(d, 512))
        return made[shape]

    yield get
    for e, _ in made.values():
        e.close()


def _rollout_check(pkg, e, m, ids, frames, t_cfg, s_cfg, penalty, seed, rng, label,
                   lookahead=None):
    sampled = t_cfg.do_sample or s_cfg.do_sample
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=frames, do_sample=t_cfg.do_sample,
                               top_k=t_cfg.top_k, top_p=t_cfg.top_p,
                               temperature=t_cfg.temperature, repetition_penalty=penalty,
                               subtalker_dosample=s_cfg.do_sample, subtalker_top_k=s_cfg.top_k,
                               subtalker_top_p=s_cfg.top_p,
                               subtalker_temperature=s_cfg.temperature, seed=seed, rng=rng)
    out = e.generate_codes_from_ids(ids, opts)
    pre, tr, pad = m.prepare(list(ids), lookahead)
    codes, ended, recs = m.rollout(pre, tr, pad, frames, t_cfg, s_cfg, penalty, seed, rng,
                                   forced_codes=out.codes)
    assert out.ended_by_eos == ended and out.frames == len(codes) // 16, label
    check_end(m, out.ended_by_eos, label, sampled)
    return check_codes(out.codes, codes, recs, label, sampled=sampled)


def test_cfg1_0p6b_greedy_240(full, pkg):
    e, m = full("0.6b")
    _rollout_check(pkg, e, m, _ids(0, 32), 240, GREEDY, GREEDY, 1.0, 0, "lcg",
                   "cfg1 0.6B greedy 240f")


def test_cfg2_0p6b_sampled_240(full, pkg):
    e, m = full("0.6b")
    _rollout_check(pkg, e, m, _ids(1, 64), 240, SAMPLED, SAMPLED, 1.05, 0, "philox",
                   "cfg2 0.6B sampled philox 240f")


def test_cfg2_lcg_reference_draw_order(full, pkg):
    """The same sampled config in the reference's own LCG draw order."""
    e, m = full("0.6b")
    _rollout_check(pkg, e, m, _ids(2, 64), 120, SAMPLED, SAMPLED, 1.05, 5, "lcg",
                   "cfg2 0.6B sampled lcg 120f")


def test_cfg3_1p7b_greedy_240(full, pkg):
    e, m = full("1.7b")
    _rollout_check(pkg, e, m, _ids(3, 128), 240, GREEDY, GREEDY, 1.0, 0, "lcg",
                   "cfg3 1.7B greedy 240f")


def test_cfg4_0p6b_text_stream(full, pkg):
    e, m = full("0.6b")
    ids = _ids(4, 256)
    frames = 120
    opts = pkg.GenerateOptions(decode_audio=False, max_frames=frames, seed=0, rng="philox")
    ts = e.start_text_stream_polling(opts, pkg.TextStreamOptions(min_start_tokens=1,
                                                                 min_resume_tokens=1))
    fed, got, chunks = 0, [], []
    ts.push_ids(ids[:8])
    fed = 8
    while True:
        r = ts.next_codes_chunk(6)
        if isinstance(r, pkg.NeedMoreText):
            if fed < len(ids):
                ts.push_ids(ids[fed:fed + 8])
                fed += 8
            else:
                ts.finish_text()
            continue
        if isinstance(r, pkg.Finished) or r is None:
            break
        chunks.append(r.frames)
        got.extend(r.codes)
    ts.close()
    assert all(c <= 6 for c in chunks) and sum(chunks) == len(got) // 16
    pre, tr, pad = m.prepare(list(ids), lookahead=1)
    codes, ended, recs = m.rollout(pre, tr, pad, frames, SAMPLED, SAMPLED, 1.05, 0, "philox",
                                   forced_codes=got)
    assert len(got) // 16 == len(codes) // 16
    check_codes(got, codes, recs, "cfg4 0.6B text stream 120f", sampled=True)


def test_cfg5_1p7b_batch16(full, pkg):
    e, m = full("1.7b")
    rng = np.random.default_rng(5)
    reqs = [rng.integers(0, VOCAB, int(rng.integers(16, 257))) for _ in range(16)]
    frames = 8
    opts = [pkg.GenerateOptions(decode_audio=False, max_frames=frames, seed=b, rng="philox")
            for b in range(16)]
    outs = e.generate_codes_batch_from_ids(reqs, opts)
    assert len(outs) == 16
    for b, (ids, out) in enumerate(zip(reqs, outs)):
        pre, tr, pad = m.prepare(list(ids))
        codes, ended, recs = m.rollout(pre, tr, pad, frames, SAMPLED, SAMPLED, 1.05, b, "philox",
                                       forced_codes=out.codes)
        assert out.ended_by_eos == ended and out.frames == len(codes) // 16
        check_end(m, out.ended_by_eos, f"cfg5 request {b}", True)
        check_codes(out.codes, codes, recs, f"cfg5 1.7B batch16 request {b} (P={pre.shape[0]})",
                    sampled=True)
