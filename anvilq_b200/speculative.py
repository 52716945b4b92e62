"""Two-token greedy speculative verification over the device-resident decoder.

Restates the verifier of the Anvil-Q4 chip (anvil-q4/rtl/anvil_q4_speculative.sv:1-94;
contract anvil-q4/design/SPEC.md:271-272: "Two-token greedy speculative
verification commits only the accepted prefix; ties choose the lowest
vocabulary index") as a host-side controller whose target runs are whole decode
steps of ``decoder.Decoder`` (one CUDA graph per token on the GPU).

A draft is (token0, token1, pos, new_sequence).  The verifier

* rejects it as an error -- nothing runs, nothing commits -- when a token is
  outside the vocabulary, the vocabulary is empty, the context holds fewer than
  two tokens, ``pos >= capacity - 1``, a continuation arrives without a valid
  sequence, or the position is not the sequence's next one (0 for a new
  sequence, else the committed length) (:59-63);
* accepts nothing, without running the target, when a continuation's token0
  differs from the standing prediction (:64-65);
* otherwise runs the target on token0 at pos: one token is accepted and the
  next prediction is its argmax; when that argmax equals token1 the target
  also runs on token1 at pos + 1, two tokens are accepted and the prediction is
  the second argmax (:68-84).  A target error, or an argmax outside the
  vocabulary, turns the whole verification into an error with nothing accepted.

A successful verification commits ``accepted`` tokens (0, 1 or 2) and the new
prediction; an error commits nothing (:39-41).  Greedy choices break ties toward
the lowest vocabulary index, as the decoder's argmax does.

The target of a continuation never re-runs committed tokens: the decoder keeps
its KV cache, so running token0 at pos writes cache row pos and reads rows
[0, pos]; a rejected token1 leaves no trace because the committed length (the
next draft position) does not cover the row it would have written.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import _lib


@dataclass
class Verification:
    """What the verifier answers for one draft (the RTL's verify_* / commit_* outputs)."""
    accepted: int          # verify_accepted: 0, 1 or 2 draft tokens confirmed
    error: bool            # verify_error: nothing accepted, nothing committed
    commit_length: int     # tokens committed to the sequence (== accepted unless error)
    prediction: int        # commit_prediction: greedy token after the committed prefix (when committed)
    target_runs: int       # target passes spent (decode steps, or batched two-token passes)


class DecoderTarget:
    """The target model: one greedy decode step of ``decoder.Decoder`` at a given
    token and position, returning its argmax (device error bits raise)."""

    def __init__(self, dec):
        self.dec = dec
        self.vocabulary = int(dec.shape[7])
        self.context_capacity = int(dec.max_seq)

    def run(self, token: int, pos: int) -> int:
        d = self.dec
        d.set_position(token, pos)
        d.step()
        d.stream.synchronize()
        d.check_errors()
        return int(d.token.item())


class BatchedDecoderTarget(DecoderTarget):
    """The target as ONE pass over both draft tokens (``Decoder.verify_tokens``):
    token0 at pos and token1 at pos + 1 through M = 2 row GEMMs, so the weights
    stream once for the pair.  run_pair returns the greedy choice after each;
    the verifier uses the second only when the first equals token1, which is
    exactly when the reference's controller would have run it.

    run_pair contract: it raises when the token0 half failed; a target that
    can tell a failure of the token1 half alone returns None as the second
    choice (the first stays valid).  This one cannot tell the halves apart
    (device error bits cover the whole pass), so any error raises."""

    def run_pair(self, token0: int, token1: int, pos: int):
        a0, a1 = self.dec.verify_tokens([token0, token1], pos)
        return a0, a1


class SpeculativeVerifier:
    """Sequence state plus the two-token verification of anvil_q4_speculative.sv.

    ``committed_tokens`` counts the tokens whose KV rows are committed;
    ``prediction`` is the greedy token expected after them (None until a target
    run produced one)."""

    def __init__(self, target, vocabulary: int | None = None, context_capacity: int | None = None):
        self.target = target
        self.vocabulary = int(target.vocabulary if vocabulary is None else vocabulary)
        self.context_capacity = int(target.context_capacity if context_capacity is None else context_capacity)
        self.committed_tokens = 0
        self.sequence_valid = False
        self.prediction: int | None = None

    def _invalid(self, token0: int, token1: int, pos: int, new_sequence: bool) -> bool:
        V, cap = self.vocabulary, self.context_capacity
        return (not 0 <= token0 < V or not 0 <= token1 < V or V == 0 or cap < 2 or pos >= cap - 1
                or pos < 0 or (not new_sequence and not self.sequence_valid)
                or (pos != 0 if new_sequence else pos != self.committed_tokens))

    def verify(self, token0: int, token1: int, pos: int, new_sequence: bool = False) -> Verification:
        """Verify one draft and commit its accepted prefix."""
        token0, token1, pos = int(token0), int(token1), int(pos)
        if self._invalid(token0, token1, pos, new_sequence):
            return Verification(0, True, 0, 0, 0)
        prediction = self.prediction
        if not new_sequence and prediction is not None and token0 != prediction:
            return self._commit(pos, 0, prediction, 0)
        runs = 0
        try:
            if hasattr(self.target, "run_pair"):   # both target runs in one batched pass
                runs = 1
                a0, a1 = self.target.run_pair(token0, token1, pos)   # a1 None: token1's half failed
                if not 0 <= a0 < self.vocabulary:
                    return Verification(0, True, 0, 0, runs)
                if a0 != token1:
                    # the reference never runs token1 here (WAIT0 -> commit 1), so
                    # whatever happened to the second half does not matter
                    return self._commit(pos, 1, a0, runs)
                if a1 is None or not 0 <= a1 < self.vocabulary:
                    return Verification(0, True, 0, 0, runs)
                return self._commit(pos, 2, a1, runs)
            runs += 1
            a0 = self.target.run(token0, pos)
            if not 0 <= a0 < self.vocabulary:
                return Verification(0, True, 0, 0, runs)
            if a0 != token1:
                return self._commit(pos, 1, a0, runs)
            runs += 1
            a1 = self.target.run(token1, pos + 1)
            if not 0 <= a1 < self.vocabulary:
                return Verification(0, True, 0, 0, runs)
            return self._commit(pos, 2, a1, runs)
        except _lib.AnvilqError:
            # a target that failed commits nothing; its partial cache writes lie
            # beyond the committed length and are overwritten later
            return Verification(0, True, 0, 0, runs)

    def _commit(self, pos: int, accepted: int, prediction, runs: int) -> Verification:
        self.committed_tokens = pos + accepted
        self.sequence_valid = True
        if prediction is not None:
            self.prediction = int(prediction)
        return Verification(accepted, False, accepted, 0 if prediction is None else int(prediction), runs)


__all__ = ["Verification", "DecoderTarget", "BatchedDecoderTarget", "SpeculativeVerifier"]


# ---- draft trees --------------------------------------------------------------
def accept_tree(tokens, parents, predictions, first: int):
    """The longest greedy-accepted path of a draft tree.

    ``tokens[m]`` continues node ``parents[m]`` (-1: the committed prefix);
    ``predictions[m]`` is the target's greedy choice after node m (as returned
    by ``Decoder.verify_tree``) and ``first`` its choice after the prefix.  From
    the prefix, a child is accepted when its token is the standing prediction
    (among several, the lowest node index), which then becomes that child's
    prediction; the walk stops at the first node with no accepted child.
    Returns (path, tokens committed, next prediction): the path as node
    indices, the accepted tokens, and the prediction after the last one --
    exactly what sequential greedy decoding from the prefix would produce for
    those positions (the tree's batched evaluation of anvil-q3-ht2/design/SPEC.md:71-86,
    with the accept rule of the two-token verifier, anvil-q4/rtl/anvil_q4_speculative.sv:64-84)."""
    if len(tokens) != len(parents) or len(predictions) != len(tokens):
        raise ValueError("tokens, parents and predictions must have one entry per node")
    children = {}
    for m, par in enumerate(parents):
        if not -1 <= int(par) < m:
            raise ValueError(f"node {m}: parent {par} must be -1 or an earlier node")
        children.setdefault(int(par), []).append(m)
    path, cur, pred = [], -1, int(first)
    while True:
        nxt = next((m for m in children.get(cur, []) if int(tokens[m]) == pred), None)
        if nxt is None:
            break
        path.append(nxt)
        cur, pred = nxt, int(predictions[nxt])
    return path, [int(tokens[m]) for m in path], pred


def speculate_tree(decoder, tokens, parents, pos: int, first: int):
    """Verify a draft tree at `pos` on ``decoder`` (one batched pass), keep the
    accepted path's K/V rows where sequential decoding would have put them and
    return (accepted tokens, next prediction).  ``first`` is the decoder's
    greedy choice after the committed prefix [0, pos)."""
    preds = decoder.verify_tree(tokens, parents, pos)
    path, accepted, pred = accept_tree(tokens, parents, preds, first)
    decoder.commit_tree_path(path, pos)
    return accepted, pred
