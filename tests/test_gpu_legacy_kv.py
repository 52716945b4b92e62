"""Legacy KV-cache codecs of the Q16.16 datapath (INT8 / INT4 symmetric, INT4
asymmetric): the oracle against the reference's own cache_block outputs
(tests/golden/legacy_kv.npz), and the CUDA encoder / decoder against the oracle
bit for bit."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import _lib, ops


def test_oracle_matches_reference_cache_block(golden_dir):
    g = np.load(golden_dir / "legacy_kv.npz")
    for i in range(int(g["count"])):
        block = [int(v) for v in g[f"b{i}_in"]]
        for fmt in (1, 2, 3):
            meta, codes, decoded = oracle.legacy_kv_block(block, fmt)
            assert meta == int(g[f"b{i}_f{fmt}_meta"]), (i, fmt)
            assert codes == [int(c) for c in g[f"b{i}_f{fmt}_codes"]], (i, fmt)
            assert decoded == [int(d) for d in g[f"b{i}_f{fmt}_decoded"]], (i, fmt)


def test_oracle_spec_worked_values():
    # anvil-q4/design/SPEC.md:256-258: INT8 raw +-509 -> e3, codes +-64, reconstruction +-512;
    # symmetric INT4 raw +-29 -> e3, codes +-4, reconstruction +-32
    assert oracle.legacy_kv_block([509, -509], 1) == (3, [64, -64], [512, -512])
    assert oracle.legacy_kv_block([29, -29], 2) == (3, [4, -4], [32, -32])


def test_oracle_payload_layout():
    """Ascending bytes / nibbles per word, W words per block, padding zero."""
    vals = np.array([[1, 2, 3, 4, 5, -6, 7]], np.int64)
    payload, meta, decoded = oracle.legacy_kv_encode(vals, 1, 7, 7, 2)   # INT4, one block of 7, W = 1
    assert meta[0, 0] == 0 and list(decoded[0]) == [1, 2, 3, 4, 5, -6, 7]
    assert payload[0, 0] == sum(((c & 15) << (4 * k)) for k, c in enumerate([1, 2, 3, 4, 5, -6, 7, 0]))
    payload, meta, _ = oracle.legacy_kv_encode(vals, 1, 7, 4, 1)         # INT8, blocks of 4 and 3
    assert payload.shape == (1, 2) and payload[0, 1] == (5 | ((-6 & 255) << 8) | (7 << 16))


def test_entry_points_validate_on_the_host():
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)
    assert lib.anvilq_legacy_kv_encode(fake, fake, fake, 1, 1, 8, 65, 1, None) == -5    # block > 64
    assert lib.anvilq_legacy_kv_encode(fake, fake, fake, 1, 1, 8, 8, 4, None) == -5    # no format 4
    assert lib.anvilq_legacy_kv_encode(None, fake, fake, 1, 1, 8, 8, 1, None) == -1
    assert lib.anvilq_legacy_kv_decode(fake, fake, fake, 1, 1, 8, 8, 1, None, None) == -1   # dev_err needed


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _values(rng, R, n):
    """Q16.16 rows with per-row magnitudes 2^0..2^31 and a few one-sided rows and extremes."""
    out = np.empty((R, n), np.int64)
    for r in range(R):
        mag = 1 << int(rng.integers(0, 32))
        v = rng.integers(-mag, mag, size=n, dtype=np.int64)
        if r % 5 == 1:
            v = np.abs(v)
        if r % 7 == 3:
            v[rng.integers(0, n)] = -(1 << 31)
        out[r] = np.clip(v, -(1 << 31), (1 << 31) - 1)
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [1, 2, 3])
@pytest.mark.parametrize("H,D,block", [(2, 64, 64), (8, 128, 24), (1, 100, 32), (4, 7, 7), (2, 128, 64), (3, 50, 1)])
def test_encode_decode_match_oracle(dev, fmt, H, D, block):
    rng = np.random.default_rng(fmt * 1000 + H * 10 + D + block)
    R = 12
    vals = _values(rng, R, H * D)
    payload_ref, meta_ref, decoded_ref = oracle.legacy_kv_encode(vals, H, D, block, fmt)
    x = torch.from_numpy(vals.astype(np.int32)).to(dev)
    payload, meta = ops.legacy_kv_encode(x, H, D, block, fmt)
    y = ops.legacy_kv_decode(payload, meta, H, D, block, fmt)
    ops.raise_device_errors(dev)
    assert np.array_equal(payload.cpu().numpy().view(np.uint32), payload_ref)
    assert np.array_equal(meta.cpu().numpy().view(np.uint32), meta_ref)
    assert np.array_equal(y.cpu().numpy(), decoded_ref)


@pytest.mark.gpu
def test_decode_flags_forbidden_codes_padding_and_metadata(dev):
    H, D, block = 1, 6, 8                       # one block of 6 values, W = 2 (INT8): 2 padding bytes
    x = torch.tensor([[1, -2, 3, -4, 5, -6]], dtype=torch.int32, device=dev)
    payload, meta = ops.legacy_kv_encode(x, H, D, block, 1)
    ops.legacy_kv_decode(payload, meta, H, D, block, 1)
    ops.raise_device_errors(dev)                # a clean block decodes without an error
    cases = []
    p = payload.clone(); p[0, 0] = (p[0, 0] & ~0xFF) | 0x80           # code -128 (forbidden in INT8)
    cases.append((p, meta, 1))
    p = payload.clone(); p[0, 1] = p[0, 1] | (1 << 24)                # nonzero padding byte
    cases.append((p, meta, 1))
    m = meta.clone(); m[0, 0] = 26                                    # exponent past the INT8 range
    cases.append((payload, m, 1))
    m = meta.clone(); m[0, 0] = m[0, 0] | (3 << 8)                    # zero point in a symmetric block
    cases.append((payload, m, 1))
    m = meta.clone(); m[0, 0] = m[0, 0] | (1 << 12)                   # reserved bit
    cases.append((payload, m, 1))
    for p, m, fmt in cases:
        ops.legacy_kv_decode(p, m, H, D, block, fmt)
        with pytest.raises(_lib.AnvilqError, match="legacy cache"):
            ops.raise_device_errors(dev)


@pytest.mark.gpu
def test_golden_api_cache_block_matches_reference(dev, golden_dir):
    """golden_api.cache_block (the reference's signature, GPU codec) returns the
    reference's own (metadata, codes, decoded) for every fixture block."""
    from anvilq_b200 import golden_api
    g = np.load(golden_dir / "legacy_kv.npz")
    for i in range(int(g["count"])):
        block = [int(v) for v in g[f"b{i}_in"]]
        for fmt in (1, 2, 3):
            meta, codes, decoded = golden_api.cache_block(block, fmt)
            assert meta == int(g[f"b{i}_f{fmt}_meta"]), (i, fmt)
            assert codes == [int(c) for c in g[f"b{i}_f{fmt}_codes"]], (i, fmt)
            assert decoded == [int(d) for d in g[f"b{i}_f{fmt}_decoded"]], (i, fmt)
