"""Decode attention over a paged KV cache (the Anvil-Q4 page table,
anvil-q4/design/SPEC.md:205-208) against the same attention over the
contiguous cache holding the same logical rows: bit-identical, since both run
the same split plan over the same logical capacity."""
import ctypes

import numpy as np
import pytest
import torch

from anvilq_b200 import _lib, ops

VALID = np.int64(1) << 31


def entry(page: int, valid: bool = True) -> int:
    """A page-table word (bit 31 valid, bits 30:0 the page) as the int32 the table tensor holds."""
    return int(np.array([(VALID if valid else 0) | page], np.int64).astype(np.uint32).view(np.int32)[0])


def _case(dev, B, Hq, Hkv, D, page_tokens, max_pages, num_pages, seed):
    rng = np.random.default_rng(seed)
    Tmax = page_tokens * max_pages
    seqlens = np.array([Tmax] + list(rng.integers(1, Tmax + 1, size=B - 1)), np.int32)
    k = rng.standard_normal((B, Tmax, Hkv, D), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((B, Tmax, Hkv, D), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((B, Hq, D), dtype=np.float32).astype(np.float16)
    # every logical page of every sequence gets its own physical page, shuffled
    # over a pool larger than needed; pages past a sequence's length stay unmapped
    phys = rng.permutation(num_pages)[:B * max_pages].reshape(B, max_pages)
    table = np.zeros((B, max_pages), np.int64)
    k_pool = np.zeros((num_pages, page_tokens, Hkv, D), np.float16)
    v_pool = np.zeros_like(k_pool)
    for b in range(B):
        for j in range((seqlens[b] + page_tokens - 1) // page_tokens):
            table[b, j] = VALID | phys[b, j]
            k_pool[phys[b, j]] = k[b, j * page_tokens:(j + 1) * page_tokens]
            v_pool[phys[b, j]] = v[b, j * page_tokens:(j + 1) * page_tokens]
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return (to(q), to(k), to(v), to(seqlens), to(k_pool), to(v_pool),
            to(table.astype(np.uint32).view(np.int32)), table)


def test_paged_entry_point_validates_on_the_host():
    lib = _lib.load()
    fake = ctypes.c_void_p(1 << 20)   # never dereferenced: rejected before any launch
    # page_tokens must be a positive multiple of 16
    for pt in (0, 8, 24):
        assert lib.anvilq_gqa_decode_paged(fake, fake, fake, fake, fake, fake, 1, 8, 2, 64, pt, 4, 4, 0.0,
                                           fake, 1 << 20, fake, None) == -5
    assert lib.anvilq_gqa_decode_paged(None, fake, fake, fake, fake, fake, 1, 8, 2, 64, 16, 4, 4, 0.0,
                                       fake, 1 << 20, fake, None) == -1


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,D,page_tokens,max_pages,num_pages", [
    (3, 32, 8, 128, 16, 64, 256),      # 1024-token capacity in 16-token pages
    (4, 14, 2, 64, 64, 40, 200),       # 2560 tokens in 64-token pages
    (2, 32, 8, 128, 256, 128, 300),    # 32768 tokens: several clusters per pair
])
def test_paged_matches_contiguous(dev, B, Hq, Hkv, D, page_tokens, max_pages, num_pages):
    q, k, v, seqlens, k_pool, v_pool, table, _ = _case(dev, B, Hq, Hkv, D, page_tokens, max_pages, num_pages, 7 + B)
    ref = ops.gqa_decode(q, k, v, seqlens)
    out = ops.gqa_decode_paged(q, k_pool, v_pool, table, seqlens)
    ops.raise_device_errors(dev)
    assert torch.equal(out, ref)
    # a graph replay reads the table and lengths anew: remap one page and shorten a sequence
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(dev)
    out2 = torch.empty_like(out)
    with torch.cuda.stream(s):
        ops.gqa_decode_paged(q, k_pool, v_pool, table, seqlens, out=out2)
    s.synchronize()
    with torch.cuda.graph(g, stream=s):
        ops.gqa_decode_paged(q, k_pool, v_pool, table, seqlens, out=out2)
    seqlens[0] = page_tokens + 3
    used = {int(e) & 0x7FFFFFFF for e in table.cpu().numpy().astype(np.int64).ravel() if int(e) < 0}
    spare = next(pg for pg in range(num_pages) if pg not in used)
    old = int(table[0, 1].item()) & 0x7FFFFFFF
    k_pool[spare].copy_(k_pool[old])
    v_pool[spare].copy_(v_pool[old])
    k_pool[old].zero_()
    v_pool[old].zero_()
    table[0, 1] = entry(spare)
    g.replay()
    torch.cuda.synchronize(dev)
    ops.raise_device_errors(dev)
    ref2 = ops.gqa_decode(q, k, v, seqlens)
    assert torch.equal(out2, ref2)


@pytest.mark.gpu
def test_absent_live_page_is_a_device_error(dev):
    q, k, v, seqlens, k_pool, v_pool, table, host = _case(dev, 2, 32, 8, 128, 16, 8, 32, 3)
    seqlens.fill_(5 * 16)                      # live pages 0..4 of both sequences
    bad = table.clone()
    bad[1, 3] = entry(int(host[1, 3] & 0x7FFFFFFF), valid=False)   # valid bit cleared on a live page
    ops.gqa_decode_paged(q, k_pool, v_pool, bad, seqlens)
    with pytest.raises(_lib.AnvilqError, match="page"):
        ops.raise_device_errors(dev)
    bad = table.clone()
    bad[0, 2] = entry(32)                      # a page past the pool (32 pages)
    ops.gqa_decode_paged(q, k_pool, v_pool, bad, seqlens)
    with pytest.raises(_lib.AnvilqError, match="page"):
        ops.raise_device_errors(dev)
    # entries past the live pages are never read: leaving them invalid is fine
    ok = table.clone()
    ok[:, 5:] = 0
    out = ops.gqa_decode_paged(q, k_pool, v_pool, ok, seqlens)
    ops.raise_device_errors(dev)
    assert torch.equal(out, ops.gqa_decode(q, k, v, seqlens))
