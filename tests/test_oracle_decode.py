"""Pins the binary64 decode oracle to FP32Model.token outputs (tests/golden/decode_small.npz)."""
import numpy as np

import oracle
from anvilq_b200 import decoder


def test_decode_oracle_matches_reference_token(golden_dir):
    g = np.load(golden_dir / "decode_small.npz")
    shape = tuple(int(v) for v in g["shape"])
    w = decoder.synthetic_weights(shape, seed=29)
    o = oracle.DecodeOracle(w)
    tokens = [int(t) for t in g["tokens"]]
    for pos in range(len(g["logits"])):
        logits = o.step(tokens[pos], pos)
        err, cos = oracle.normalized_error(logits, g["logits"][pos])
        # binary64 restatement against the reference's binary32 arithmetic
        assert err <= 1e-4 and cos >= 0.999999, (pos, err, cos)
        assert oracle.greedy(logits) == tokens[pos + 1]
