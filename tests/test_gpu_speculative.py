"""Two-token speculative verification with the GPU decoder as the target.

What the verifier commits must be the plain greedy decode of the same model,
bit for bit (same kernels, same cache), whether a draft is accepted whole,
cut after its first token (its second token's cache row then gets rewritten
by the next run) or rejected without a target run."""
import pytest
import torch

from anvilq_b200 import decoder
from anvilq_b200.speculative import BatchedDecoderTarget, DecoderTarget, SpeculativeVerifier

pytestmark = pytest.mark.gpu

SHAPE = (2, 128, 256, 2, 1, 64, 128, 64, 32)   # (L, H, I, QH, KVH, D, G, V, SEQ)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _greedy(w, dev, first, n):
    return [first] + decoder.Decoder(w, dev, max_seq=32).generate(first, n)


@pytest.mark.parametrize("graph,batched", [(False, False), (True, False), (False, True)])
def test_verifier_commits_the_greedy_decode(dev, graph, batched):
    w = decoder.synthetic_weights(SHAPE, seed=41)
    seq = _greedy(w, dev, 9, 20)                  # seq[p] is the token at position p
    d = decoder.Decoder(w, dev, max_seq=32)
    if graph:
        d.reset(9)
        d.capture()
    v = SpeculativeVerifier(BatchedDecoderTarget(d) if batched else DecoderTarget(d))
    r = v.verify(seq[0], seq[1], 0, new_sequence=True)
    assert (r.accepted, r.error, r.prediction) == (2, False, seq[2])
    wrong = lambda t: (t + 1) % SHAPE[7]
    pos, i = 2, 0
    while pos < 18:
        case = i % 3
        i += 1
        if case == 0:         # a draft whose second token is wrong: one token accepted
            r = v.verify(seq[pos], wrong(seq[pos + 1]), pos)
            assert (r.accepted, r.error, r.target_runs, r.prediction) == (1, False, 1, seq[pos + 1])
            # the rejected token's cache row (written by the batched pass) is rewritten by the next run
        elif case == 1:       # a draft that misses the prediction: nothing runs
            r = v.verify(wrong(seq[pos]), seq[pos + 1], pos)
            assert (r.accepted, r.error, r.target_runs) == (0, False, 0)
            r = v.verify(seq[pos], seq[pos + 1], pos)
            assert (r.accepted, r.error) == (2, False)
        else:
            r = v.verify(seq[pos], seq[pos + 1], pos)
            assert (r.accepted, r.error, r.target_runs) == (2, False, 1 if batched else 2)
        pos = v.committed_tokens
        assert v.prediction == seq[pos], pos


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_verify_tokens_equal_sequential_decode_steps(dev, M):
    """One batched pass over M tokens gives the greedy choice after each token,
    as M decode steps do, and leaves the cache ready for the next step."""
    w = decoder.synthetic_weights(SHAPE, seed=43)
    seq = _greedy(w, dev, 5, 24)
    d = decoder.Decoder(w, dev, max_seq=32)
    P = 6
    d.reset(seq[0])
    for _ in range(P):                 # commit tokens 0 .. P-1 by plain steps
        d.step()
    d.stream.synchronize()
    got = d.verify_tokens(seq[P:P + M], P)
    assert got == seq[P + 1:P + M + 1]
    # continue with a plain step after the verified tokens
    d.set_position(seq[P + M], P + M)
    d.step()
    d.stream.synchronize()
    assert int(d.token.item()) == seq[P + M + 1]


@pytest.mark.parametrize("shape_id", [0, 1])
def test_tree_draft_commits_the_greedy_path(dev, shape_id):
    """A draft tree (branching at several depths, wrong siblings before and
    after the right ones) verified in one batched pass: the accepted path is the
    plain greedy decode, the next prediction is its next token, and after the
    accepted K/V rows are moved into place plain decode steps continue exactly
    as the sequential decode does."""
    from anvilq_b200.speculative import speculate_tree
    w = decoder.synthetic_weights(SHAPE, seed=47 + shape_id)
    seq = _greedy(w, dev, 3, 24)
    V = SHAPE[7]
    wrong = lambda t, k=1: (t + k) % V
    P = 5
    d = decoder.Decoder(w, dev, max_seq=32)
    d.reset(seq[0])
    for _ in range(P):                 # commit tokens 0 .. P-1 by plain steps
        d.step()
    d.stream.synchronize()
    first = int(d.token.item())        # the decoder's greedy choice for position P
    assert first == seq[P]
    if shape_id == 0:   # wrong root first; the right chain 1 -> 3 -> 5 with wrong siblings 2, 4, 6
        tokens = [wrong(seq[P]), seq[P], wrong(seq[P + 1]), seq[P + 1], wrong(seq[P + 2], 2), seq[P + 2],
                  wrong(seq[P + 3])]
        parents = [-1, -1, 1, 1, 3, 3, 5]
        want = 3
    else:               # a bushy tree: two right levels, then only wrong children
        tokens = [seq[P], wrong(seq[P + 1]), seq[P + 1], wrong(seq[P + 1], 2), wrong(seq[P + 2]), wrong(seq[P + 2], 3)]
        parents = [-1, 0, 0, 0, 2, 2]
        want = 2
    accepted, nxt = speculate_tree(d, tokens, parents, P, first)
    assert accepted == seq[P:P + want]
    assert nxt == seq[P + want]
    # continue with plain steps after the accepted tokens
    d.set_position(nxt, P + want)
    for k in range(3):
        d.step()
        d.stream.synchronize()
        assert int(d.token.item()) == seq[P + want + 1 + k], k
