"""Regenerates tests/golden/tiny_seed0.json from the CPU oracle.

The fixture pins the oracle's own outputs on the seeded "tiny" synthetic
checkpoint (oracle/synth.py, seed 0) so that later changes to the oracle are
caught; it is produced by this script only:

    python tests/golden/make_golden.py
"""
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import qtts_oracle as O, synth  # noqa: E402

IDS = [17, 3999, 256, 1024, 7, 88, 2048, 3000]


def compute(model_dir) -> dict:
    m = O.OracleModel(model_dir, 128)
    pre, tr, pad = m.prepare(IDS)
    out = {"ids": IDS, "prefill_steps": int(pre.shape[0]),
           "prefill_sum": float(pre.double().sum()), "prefill_row0_head": pre[0, :8].tolist(),
           "trailing_sum": float(tr.double().sum()), "tts_pad_head": pad[:8].tolist()}
    _, hidden, logits = m.talker_prefill(pre)
    out["prefill_logits_head"] = logits[:8].tolist()
    out["prefill_token"] = O.argmax_device(m.penalise_and_suppress(logits, None, 1.0))
    g = O.SamplingConfig(False, 0, 1.0, 1.0)
    codes, ended, _ = m.rollout(pre, tr, pad, 6, g, g)
    out["greedy_codes"] = codes
    s = O.SamplingConfig(True, 50, 1.0, 0.9)
    codes, ended, _ = m.rollout(pre, tr, pad, 6, s, s, penalty=1.05, seed=0)
    out["sampled_lcg_codes"] = codes
    codes, ended, _ = m.rollout(pre, tr, pad, 4, s, s, penalty=1.05, seed=7, rng_kind="philox")
    out["sampled_philox_codes"] = codes
    th = torch.from_numpy(O.deterministic_hidden(m.tdims.hidden, 17, 15.0))
    se = torch.from_numpy(O.deterministic_hidden(m.tdims.hidden, 23, 11.0))
    toks, esum, _, _ = m.code_predictor(th, se, g, O.Lcg(0))
    out["cp_tokens"] = toks
    out["cp_embedding_sum_head"] = esum[:8].tolist()
    return out


if __name__ == "__main__":
    import tempfile
    d = synth.write_model(Path(tempfile.gettempdir()) / "qtts_golden_tiny", "tiny", 0)
    res = compute(d)
    (Path(__file__).parent / "tiny_seed0.json").write_text(json.dumps(res, indent=1))
    print("wrote tiny_seed0.json")
