"""Two-token greedy speculative verification: the controller's decisions
(anvil-q4/rtl/anvil_q4_speculative.sv:1-94) against a host-side fake target.

The fake target is a fixed greedy "model": after token t at position p it
predicts (7 t + p) mod V, and it records every run, so the tests can check both
the answer and which target runs the verifier spent."""
import pytest

from anvilq_b200 import _lib
from anvilq_b200.speculative import SpeculativeVerifier


class FakeTarget:
    def __init__(self, vocabulary=50, capacity=16, fail_at=None, bad_argmax_at=None):
        self.vocabulary = vocabulary
        self.context_capacity = capacity
        self.runs = []
        self.fail_at = fail_at
        self.bad_argmax_at = bad_argmax_at

    def next(self, token, pos):
        return (7 * token + pos) % self.vocabulary

    def run(self, token, pos):
        self.runs.append((token, pos))
        if self.fail_at == pos:
            raise _lib.AnvilqError("target fault")
        if self.bad_argmax_at == pos:
            return self.vocabulary
        return self.next(token, pos)


def test_new_sequence_accepts_both_tokens_when_the_draft_is_greedy():
    t = FakeTarget()
    v = SpeculativeVerifier(t)
    t1 = t.next(3, 0)
    r = v.verify(3, t1, 0, new_sequence=True)
    assert (r.accepted, r.error, r.commit_length, r.target_runs) == (2, False, 2, 2)
    assert r.prediction == t.next(t1, 1)
    assert t.runs == [(3, 0), (t1, 1)]
    assert (v.committed_tokens, v.prediction, v.sequence_valid) == (2, t.next(t1, 1), True)


def test_mismatching_second_token_accepts_one_and_skips_the_second_run():
    t = FakeTarget()
    v = SpeculativeVerifier(t)
    wrong = (t.next(3, 0) + 1) % t.vocabulary
    r = v.verify(3, wrong, 0, new_sequence=True)
    assert (r.accepted, r.error, r.commit_length, r.prediction) == (1, False, 1, t.next(3, 0))
    assert t.runs == [(3, 0)]
    assert v.committed_tokens == 1


def test_continuation_whose_first_token_misses_the_prediction_accepts_nothing():
    t = FakeTarget()
    v = SpeculativeVerifier(t)
    v.verify(3, 0, 0, new_sequence=True)              # commits 1, prediction p
    p = v.prediction
    n = len(t.runs)
    r = v.verify((p + 1) % t.vocabulary, 0, 1)
    assert (r.accepted, r.error, r.commit_length, r.prediction, r.target_runs) == (0, False, 0, p, 0)
    assert len(t.runs) == n and v.committed_tokens == 1 and v.prediction == p


def test_continuation_chain_commits_the_greedy_sequence():
    """Drafting the true greedy continuation commits two tokens per verification,
    and the committed tokens are exactly the plain greedy decode."""
    t = FakeTarget(vocabulary=97, capacity=64)
    v = SpeculativeVerifier(t)
    seq = [5]
    for p in range(20):
        seq.append(t.next(seq[-1], p))
    r = v.verify(seq[0], seq[1], 0, new_sequence=True)
    assert r.accepted == 2 and v.prediction == seq[2]
    while v.committed_tokens < 16:
        pos = v.committed_tokens
        # the draft: the standing prediction (= seq[pos]) and its greedy successor
        r = v.verify(v.prediction, t.next(v.prediction, pos), pos)
        assert r.accepted == 2 and not r.error and r.target_runs == 2
        # tokens [0, pos + 2) committed; the prediction is the next greedy token
        assert v.committed_tokens == pos + 2 and v.prediction == seq[pos + 2]
    assert t.runs == [(seq[p], p) for p in range(16)]


@pytest.mark.parametrize("draft", [
    (50, 0, 0, True),        # token0 outside the vocabulary
    (0, 50, 0, True),        # token1 outside the vocabulary
    (1, 2, 3, True),         # a new sequence must start at 0
    (1, 2, 0, False),        # continuation without a valid sequence
    (1, 2, 15, True),        # pos >= capacity - 1
    (1, 2, -1, True),
])
def test_invalid_drafts_are_errors_that_run_nothing(draft):
    t = FakeTarget()
    v = SpeculativeVerifier(t)
    r = v.verify(*draft[:3], new_sequence=draft[3])
    assert (r.accepted, r.error, r.commit_length, r.target_runs) == (0, True, 0, 0)
    assert t.runs == [] and v.committed_tokens == 0 and not v.sequence_valid


def test_continuation_at_the_wrong_position_is_an_error():
    t = FakeTarget()
    v = SpeculativeVerifier(t)
    v.verify(3, 0, 0, new_sequence=True)
    r = v.verify(v.prediction, 0, v.committed_tokens + 1)
    assert r.error and r.accepted == 0 and v.committed_tokens == 1


def test_degenerate_vocabulary_and_capacity_are_errors():
    for vocab, cap in ((0, 16), (50, 1)):
        t = FakeTarget(vocabulary=vocab, capacity=cap)
        r = SpeculativeVerifier(t).verify(0, 0, 0, new_sequence=True)
        assert r.error and t.runs == []


@pytest.mark.parametrize("kind", ["fault", "argmax"])
@pytest.mark.parametrize("at", [0, 1])
def test_target_failure_in_either_run_commits_nothing(kind, at):
    t = FakeTarget(**({"fail_at": at} if kind == "fault" else {"bad_argmax_at": at}))
    v = SpeculativeVerifier(t)
    r = v.verify(3, t.next(3, 0), 0, new_sequence=True)
    assert (r.accepted, r.error, r.commit_length) == (0, True, 0)
    assert len(t.runs) == at + 1
    assert v.committed_tokens == 0 and not v.sequence_valid and v.prediction is None


class FakePairTarget(FakeTarget):
    """A target that runs both draft tokens in one batched pass."""

    def __init__(self, fail_second=False, **kw):
        super().__init__(**kw)
        self.fail_second = fail_second

    def run_pair(self, token0, token1, pos):
        self.runs.append(((token0, pos), (token1, pos + 1)))
        a0 = self.vocabulary if self.bad_argmax_at == pos else self.next(token0, pos)
        a1 = self.vocabulary if self.bad_argmax_at == pos + 1 else self.next(token1, pos + 1)
        return a0, None if self.fail_second else a1


def test_batched_target_gives_the_same_commits_in_one_pass():
    t = FakePairTarget()
    v = SpeculativeVerifier(t)
    t1 = t.next(3, 0)
    r = v.verify(3, t1, 0, new_sequence=True)
    assert (r.accepted, r.error, r.prediction, r.target_runs) == (2, False, t.next(t1, 1), 1)
    r = v.verify(v.prediction, (t.next(v.prediction, 2) + 1) % t.vocabulary, 2)
    assert (r.accepted, r.prediction, r.target_runs) == (1, t.next(t.next(t1, 1), 2), 1)
    assert len(t.runs) == 2


def test_batched_target_ignores_the_second_choice_when_the_first_misses():
    # an out-of-vocabulary second choice only matters when token1 was accepted
    t = FakePairTarget(bad_argmax_at=1)
    r = SpeculativeVerifier(t).verify(3, (t.next(3, 0) + 1) % 50, 0, new_sequence=True)
    assert (r.accepted, r.error) == (1, False)
    t = FakePairTarget(bad_argmax_at=1)
    r = SpeculativeVerifier(t).verify(3, t.next(3, 0), 0, new_sequence=True)
    assert (r.accepted, r.error) == (0, True)


def test_batched_target_whose_second_half_failed():
    """The token1 half failing only matters when token1 was accepted: with
    a0 != token1 the reference controller (WAIT0) never runs token1 and
    commits one token, so the batched pass must too."""
    t = FakePairTarget(fail_second=True)
    v = SpeculativeVerifier(t)
    r = v.verify(3, (t.next(3, 0) + 1) % 50, 0, new_sequence=True)
    assert (r.accepted, r.error, r.commit_length, r.prediction) == (1, False, 1, t.next(3, 0))
    assert v.committed_tokens == 1 and v.sequence_valid
    t = FakePairTarget(fail_second=True)
    v = SpeculativeVerifier(t)
    r = v.verify(3, t.next(3, 0), 0, new_sequence=True)
    assert (r.accepted, r.error, r.commit_length) == (0, True, 0)
    assert v.committed_tokens == 0 and not v.sequence_valid


def test_accept_tree_walks_the_greedy_path():
    """accept_tree: from the prefix's prediction, each accepted child's own
    prediction selects the next; siblings that differ are skipped, the lowest
    matching index wins, and the walk stops at the first miss."""
    from anvilq_b200.speculative import accept_tree
    #        prefix -> 0:(5)  1:(7)
    #        0 -> 2:(6)  3:(9);  3 -> 4:(1);  1 -> 5:(2)
    tokens = [5, 7, 6, 9, 1, 2]
    parents = [-1, -1, 0, 0, 3, 1]
    preds = [9, 2, 0, 1, 4, 3]
    path, acc, nxt = accept_tree(tokens, parents, preds, first=5)
    assert path == [0, 3, 4] and acc == [5, 9, 1] and nxt == 4
    path, acc, nxt = accept_tree(tokens, parents, preds, first=7)
    assert path == [1, 5] and acc == [7, 2] and nxt == 3
    path, acc, nxt = accept_tree(tokens, parents, preds, first=8)   # no root matches
    assert path == [] and acc == [] and nxt == 8
    # two equal siblings: the lower index is taken
    path, _, _ = accept_tree([5, 5], [-1, -1], [1, 2], first=5)
    assert path == [0]


def test_accept_tree_rejects_bad_parents():
    from anvilq_b200.speculative import accept_tree
    with pytest.raises(ValueError):
        accept_tree([1, 2], [-1, 1], [0, 0], first=1)   # a node is its own parent
    with pytest.raises(ValueError):
        accept_tree([1, 2], [-1, -2], [0, 0], first=1)

