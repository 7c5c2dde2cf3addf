"""Regenerates tests/golden/codec_seed0.json from the codec oracle.

The fixture pins the fp32 codec restatement (oracle/codec.py) on its seeded
synthetic weights (seed 0) and fixed codes, so later changes to the oracle
are caught; it is produced by this script only:

    python tests/golden/make_codec_golden.py
"""
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import codec as K  # noqa: E402

# Two frames: in-range codes, a negative code and codes past the codebook size.
CODES = [[5, 7, 2047, 0, 1, 2, 3, 4, 100, 200, 300, 400, 500, 600, 700, 800],
         [2049, -1, 9, 9, 9, 9, 1000, 1500, 1999, 42, 43, 44, 45, 46, 47, 48]]
STRIDE = 97  # waveform subsample


def compute(tensors) -> dict:
    st = K.CodecOracle(tensors).decode_stages(np.asarray(CODES).reshape(-1))
    out = {"codes": CODES, "stride": STRIDE}
    for name, v in st.items():
        v64 = v.astype(np.float64)
        out[name] = {"shape": list(v.shape), "sum": float(v64.sum()),
                     "abs_sum": float(np.abs(v64).sum())}
    out["waveform_samples"] = st["waveform"][::STRIDE].astype(float).tolist()
    return out


if __name__ == "__main__":
    res = compute(K.generate(0))
    (Path(__file__).parent / "codec_seed0.json").write_text(json.dumps(res, indent=1))
    print("wrote codec_seed0.json")
