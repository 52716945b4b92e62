"""The golden-model drop-ins with the reference's call signatures, on the GPU,
against outputs the reference itself produced (tests/golden/, made by
tests/golden/make_golden.py):

* attention(q, keys, values)           fp64_reference.attention (anvil-q1-fp/tests/fp64_reference.py:164-170)
* pack_lanes / unpack_lanes            awq_prepare.py:84-99 (bit-exact)
* GpuModel(checkpoint, shape).token    FP32Model.token (anvil-q1/tests/official_weights.py:451-509)
"""
import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import decoder, golden_api
from anvilq_b200.checkpoint import CheckpointError

pytestmark = pytest.mark.gpu

# attention: per-operator tolerance of anvil-q1-fp/design/SPEC.md:311-317 (cosine >= 0.9999,
# max|y - ref| / max(1, max|ref|) <= 0.002); decode logits: the decode-step tolerance of
# tests/test_gpu_decode.py (normalized error <= 1e-2, cosine >= 0.999).
TOL_ATTN = (2e-3, 0.9999)
TOL_DECODE = (1e-2, 0.999)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def test_attention_signature_against_reference_outputs(dev, golden_dir):
    g = np.load(golden_dir / "attention.npz")
    checked = 0
    for key in [str(s) for s in g["case_names"]]:
        q, k, v, ref = g[key + "_q"], g[key + "_k"], g[key + "_v"], g[key + "_y"]
        if q.shape[1] not in (64, 128):
            with pytest.raises(ValueError):
                golden_api.attention(q, k, v)
            continue
        y = golden_api.attention(q, k, v)
        assert y.shape == ref.shape and y.dtype == np.float64
        err, cos = oracle.normalized_error(y, ref)
        assert err <= TOL_ATTN[0] and cos >= TOL_ATTN[1], (key, err, cos)
        checked += 1
    assert checked >= 4
    with pytest.raises(ValueError):
        golden_api.attention(np.zeros((6, 64)), np.zeros((3, 4, 64)), np.zeros((3, 4, 64)))   # 6 % 4 != 0


def test_pack_lanes_bit_exact(dev, golden_dir):
    g = np.load(golden_dir / "pack.npz")
    words = golden_api.pack_lanes(g["lanes_codes"])
    assert words.dtype == np.dtype("<u4") and words.shape == g["lanes_words"].shape
    assert (words == g["lanes_words"]).all()
    codes = golden_api.unpack_lanes(words, g["lanes_codes"].shape[0])
    assert codes.dtype == np.uint8 and (codes == g["lanes_codes"]).all()
    rng = np.random.default_rng(11)
    c = rng.integers(0, 16, size=(64, 40)).astype(np.uint8)
    w = golden_api.pack_lanes(c)
    assert (w == oracle.pack_lanes(c)).all()
    assert (golden_api.unpack_lanes(w, 64) == c).all()
    for bad in (np.zeros((12, 4), np.uint8), np.full((8, 4), 16), np.full((8, 4), -1), np.zeros(8)):
        with pytest.raises(ValueError):
            golden_api.pack_lanes(bad)
    with pytest.raises(ValueError):
        golden_api.unpack_lanes(w, 63)


def test_gpu_model_token_against_reference_logits(dev, golden_dir):
    """GpuModel.token over the same checkpoint object FP32Model read when the
    fixture was made: same logits within tolerance, same greedy tokens."""
    g = np.load(golden_dir / "decode_small.npz")
    shape = tuple(int(v) for v in g["shape"])
    ckpt = decoder.synthetic_weights(shape, seed=29).checkpoint()
    model = golden_api.GpuModel(ckpt, shape)
    tokens = [int(t) for t in g["tokens"]]
    for pos in range(len(g["logits"])):
        logits = model.token(tokens[pos], pos, new_sequence=pos == 0)
        assert len(logits) == shape[7]
        err, cos = oracle.normalized_error(np.asarray(logits), g["logits"][pos])
        assert err <= TOL_DECODE[0] and cos >= TOL_DECODE[1], (pos, err, cos)
        assert int(np.argmax(logits)) == tokens[pos + 1]
    # the reference's sequencing rules
    with pytest.raises(CheckpointError):
        model.token(tokens[0], 0)                       # not the next position
    with pytest.raises(CheckpointError):
        model.token(tokens[0], 1, new_sequence=True)    # a new sequence starts at 0
    with pytest.raises(CheckpointError):
        model.token(shape[7], len(g["logits"]))         # token outside the vocabulary
    first = model.token(tokens[0], 0, new_sequence=True)   # restart reproduces position 0
    err, cos = oracle.normalized_error(np.asarray(first), g["logits"][0])
    assert err <= TOL_DECODE[0] and cos >= TOL_DECODE[1]
