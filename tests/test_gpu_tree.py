"""Tree attention of speculative draft nodes (per-node causal attention over the
committed prefix and the node's ancestors) against the binary64 golden
attention over each node's rows, and the ancestor-contract checks."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from anvilq_b200 import _lib, ops

TOL_ERR, TOL_COS = 2e-3, 0.9999   # the attention tolerance (anvil-q1-fp/design/SPEC.md:311-317)


def random_tree(rng, M):
    """Ancestor masks of a random draft tree: node m's parent is an earlier node
    (or the prefix), and its mask is its parent's plus itself."""
    masks = []
    for m in range(M):
        parent = int(rng.integers(-1, m)) if m else -1
        masks.append((masks[parent] if parent >= 0 else 0) | (1 << m))
    return masks


def test_tree_oracle_contract_and_chain():
    assert oracle.tree_is_valid([1, 3, 7, 15])          # a chain
    assert oracle.tree_is_valid([1, 3, 5, 11])          # 0 -> {1, 2}, 1 -> 3
    assert oracle.tree_is_valid([1, 2])                 # two children of the prefix
    assert not oracle.tree_is_valid([1, 1])             # node 1 misses itself
    assert not oracle.tree_is_valid([3])                # node 0 sees a later node
    assert not oracle.tree_is_valid([1, 3, 6])          # node 2 sees 1 but not 1's ancestor 0
    rng = np.random.default_rng(1)
    for M in (1, 4, 16, 32):
        assert oracle.tree_is_valid(random_tree(rng, M))
    # a chain's tree attention is causal attention over the extended sequence
    q = rng.standard_normal((3, 4, 64))
    k = rng.standard_normal((10, 2, 64))
    v = rng.standard_normal((10, 2, 64))
    t = oracle.tree_attention_f64(q, k, v, [1, 3, 7], 7)
    for m in range(3):
        np.testing.assert_allclose(t[m], oracle.attention_f64(q[m], k[:8 + m], v[:8 + m]), rtol=1e-12)


def test_tree_entry_point_validates_on_the_host():
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)
    args = lambda P, M, T: (fake, fake, fake, fake, P, fake, M, 8, 2, 64, T, 0.0, fake, 1 << 20, fake, None)
    assert lib.anvilq_tree_attention(*args(0, 33, 64)) == -5      # more than 32 nodes
    assert lib.anvilq_tree_attention(*args(60, 8, 64)) == -5      # prefix + nodes past the cache
    assert lib.anvilq_tree_attention(*args(0, 4, 40)) == -5       # Tmax not a multiple of 16
    assert lib.anvilq_tree_attention(*args(-1, 4, 64)) == -5
    assert lib.anvilq_tree_attention(None, fake, fake, fake, 0, fake, 4, 8, 2, 64, 64, 0.0, fake, 1 << 20, fake,
                                     None) == -1


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.gpu
@pytest.mark.parametrize("M,Hq,Hkv,D,P,Tmax", [
    (4, 14, 2, 64, 1000, 1024),      # Qwen2.5-0.5B heads, 4 draft nodes
    (16, 32, 8, 128, 4000, 4096),    # Llama-7B-class heads, 16 nodes
    (32, 32, 8, 128, 200, 256),      # the widest tree, short prefix
    (8, 32, 8, 128, 0, 64),          # no committed prefix
    (2, 32, 8, 128, 30000, 32768),   # long prefix: several clusters per node
])
def test_tree_attention_matches_golden(dev, M, Hq, Hkv, D, P, Tmax):
    rng = np.random.default_rng(M * 100 + P)
    q = rng.standard_normal((M, Hq, D), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((Tmax, Hkv, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((Tmax, Hkv, D), dtype=np.float32).astype(np.float16)
    masks = random_tree(rng, M)
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    anc = to(np.array(masks, np.uint32).view(np.int32))
    out = ops.tree_attention(to(q), to(k), to(v), anc, P)
    ops.raise_device_errors(dev)
    ref = oracle.tree_attention_f64(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64), masks, P)
    err, cos = oracle.normalized_error(out.float().cpu().numpy(), ref)
    assert err <= TOL_ERR and cos >= TOL_COS, (err, cos)


@pytest.mark.gpu
def test_tree_chain_equals_decode_attention(dev):
    """A chain of M nodes is causal decode attention over prefix + m + 1 rows:
    node m's result equals the decode kernel's at that length (within the
    tolerance: the tail is merged in fp32 from the prefix's fp16 output)."""
    M, Hq, Hkv, D, P, Tmax = 4, 32, 8, 128, 777, 1024
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    q = torch.randn((M, Hq, D), generator=g, device=dev, dtype=torch.float16)
    k = torch.randn((Tmax, Hkv, D), generator=g, device=dev, dtype=torch.float16)
    v = torch.randn((Tmax, Hkv, D), generator=g, device=dev, dtype=torch.float16)
    anc = torch.tensor([(1 << (m + 1)) - 1 for m in range(M)], dtype=torch.int32, device=dev)
    out = ops.tree_attention(q, k, v, anc, P)
    ref = ops.gqa_decode(q, k[None].expand(M, -1, -1, -1).contiguous(), v[None].expand(M, -1, -1, -1).contiguous(),
                         torch.arange(P + 1, P + M + 1, dtype=torch.int32, device=dev))
    ops.raise_device_errors(dev)
    err, cos = oracle.normalized_error(out.float().cpu().numpy(), ref.float().cpu().numpy())
    assert err <= TOL_ERR and cos >= TOL_COS, (err, cos)


@pytest.mark.gpu
def test_broken_ancestor_masks_are_device_errors(dev):
    M, Hq, Hkv, D, P, Tmax = 3, 8, 2, 64, 16, 64
    q = torch.zeros((M, Hq, D), dtype=torch.float16, device=dev)
    k = torch.zeros((Tmax, Hkv, D), dtype=torch.float16, device=dev)
    for masks in ([1, 1, 7], [1, 3, 6], [3, 3, 7]):   # no self / missing ancestor's ancestor / later node
        assert not oracle.tree_is_valid(masks)
        anc = torch.tensor(masks, dtype=torch.int32, device=dev)
        ops.tree_attention(q, k, k, anc, P)
        with pytest.raises(_lib.AnvilqError, match="ancestor"):
            ops.raise_device_errors(dev)
