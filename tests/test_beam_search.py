"""Beam search: golden searches over small Markov chains, sampler contracts, scorers and constraints.

The chains and expected beams are the ones the reference's ``tests/beam_search_test.py`` uses, so a
pass here means the two implementations agree on them.
"""
import math

import pytest
import torch

from olmo_b200.beam_search import (
    BeamSearch,
    DeterministicSampler,
    GumbelSampler,
    LengthNormalizedSequenceLogProbabilityScorer,
    MultinomialSampler,
    RepeatedNGramBlockingConstraint,
    TopKSampler,
    TopPSampler,
)

END = 5
#              START  1    2    3    4   END
CHAIN = torch.tensor(
    [
        [0.0, 0.4, 0.3, 0.2, 0.1, 0.0],
        [0.0, 0.0, 1.0, 0.0, 0.0, 0.0],
        [0.0, 0.0, 0.0, 1.0, 0.0, 0.0],
        [0.0, 0.0, 0.0, 0.0, 1.0, 0.0],
        [0.0, 0.0, 0.0, 0.0, 0.0, 1.0],
        [0.2, 0.1, 0.2, 0.2, 0.2, 0.1],
    ]
)
SHORT = torch.tensor(
    [
        [0.0, 0.1, 0.0, 0.0, 0.0, 0.9],
        [0.0, 0.0, 0.1, 0.0, 0.0, 0.9],
        [0.0, 0.0, 0.0, 0.1, 0.0, 0.9],
        [0.0, 0.0, 0.0, 0.0, 0.1, 0.9],
        [0.0, 0.0, 0.0, 0.0, 0.0, 1.0],
        [0.2, 0.1, 0.2, 0.2, 0.2, 0.1],
    ]
)
LOOPY = torch.tensor(
    [
        [0.0, 1.0, 0.0, 0.0, 0.0, 0.0],
        [0.0, 0.0, 0.4, 0.6, 0.0, 1e-9],
        [0.0, 0.0, 0.0, 1.0, 0.0, 1e-9],
        [0.0, 1.0, 0.0, 0.0, 0.0, 1e-9],
        [0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
        [0.0, 0.0, 0.0, 0.0, 0.0, 1.0],
    ]
)
DENSE = torch.tensor(
    [
        [0.0, 0.4, 0.3, 0.2, 0.1, 0.0],
        [0.0, 0.4, 0.3, 0.2, 0.1, 0.1],
        [0.0, 0.0, 0.4, 0.3, 0.2, 0.1],
        [0.0, 0.0, 0.3, 0.4, 0.2, 0.1],
        [0.0, 0.0, 0.2, 0.3, 0.4, 0.1],
        [0.2, 0.1, 0.2, 0.2, 0.2, 0.1],
    ]
)


def quiet():
    import warnings

    ctx = warnings.catch_warnings()
    ctx.__enter__()
    warnings.simplefilter("ignore")

    class _C:
        def __enter__(self_inner):
            return None

        def __exit__(self_inner, *a):
            return ctx.__exit__(*a)

    return _C()


def markov(matrix, with_timestep=False):
    def two(last, state):
        return torch.log(matrix[last]), state

    def three(last, state, timestep):
        return two(last, state)

    return three if with_timestep else two


def run(search, matrix=CHAIN, batch=5, state=None, with_timestep=True):
    seqs, scores = search.search(torch.zeros(batch, dtype=torch.long), state or {}, markov(matrix, with_timestep))
    assert seqs.shape[:2] == (batch, search.beam_size)
    assert scores.shape == (batch, search.beam_size)
    return seqs, scores


def expect(seqs, scores, want_seqs, want_probs):
    assert seqs[0].tolist() == want_seqs
    torch.testing.assert_close(scores[0], torch.log(torch.tensor(want_probs)), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("with_timestep", [True, False])
def test_top_beams_of_simple_chain(with_timestep):
    with quiet():
        seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=3), with_timestep=with_timestep)
    expect(seqs, scores, [[1, 2, 3, 4, 5], [2, 3, 4, 5, 5], [3, 4, 5, 5, 5]], [0.4, 0.3, 0.2])


def test_state_follows_surviving_beams():
    """State rows must be re-indexed by parent beam: the step function checks its own foo tensor."""
    batch, beam = 3, 3
    seen = []

    def step(last, state, t):
        # every row of "tag" was written as the token that row's beam had produced at t-1
        if t > 0:
            seen.append(bool((state["tag"] == state["prev"]).all()))
        log_probs = torch.log(CHAIN[last])
        return log_probs, {"tag": last.clone(), "prev": last.clone(), "none": None}

    search = BeamSearch(END, max_steps=6, beam_size=beam)
    with quiet():
        search.search(torch.zeros(batch, dtype=torch.long), {"tag": torch.zeros(batch), "prev": torch.zeros(batch)}, step)
    assert seen and all(seen)


def test_state_shapes_through_search():
    batch, beam = 2, 3
    shapes = []

    def step(last, state, t):
        shapes.append(tuple(state["h"].shape))
        return torch.log(CHAIN[last]), state

    with quiet():
        BeamSearch(END, max_steps=4, beam_size=beam).search(
            torch.zeros(batch, dtype=torch.long), {"h": torch.zeros(batch, 7, 2)}, step
        )
    assert shapes[0] == (batch, 7, 2)
    assert all(s == (batch * beam, 7, 2) for s in shapes[1:])


def test_batch_of_one_and_greedy():
    with quiet():
        seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=3), batch=1)
    expect(seqs, scores, [[1, 2, 3, 4, 5], [2, 3, 4, 5, 5], [3, 4, 5, 5, 5]], [0.4, 0.3, 0.2])
    seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=1))
    expect(seqs, scores, [[1, 2, 3, 4, 5]], [0.4])


def test_single_step_and_early_stop():
    seqs, scores = run(BeamSearch(END, max_steps=1, beam_size=3))
    expect(seqs, scores, [[1], [2], [3]], [0.4, 0.3, 0.2])
    with quiet():
        seqs, scores = run(BeamSearch(END, max_steps=3, beam_size=3))
    expect(seqs, scores, [[1, 2, 3], [2, 3, 4], [3, 4, 5]], [0.4, 0.3, 0.2])


def test_short_sequences_and_min_steps():
    seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=5), matrix=SHORT)
    expect(
        seqs,
        scores,
        [[5, 5, 5, 5, 5], [1, 5, 5, 5, 5], [1, 2, 5, 5, 5], [1, 2, 3, 5, 5], [1, 2, 3, 4, 5]],
        [0.9, 0.09, 0.009, 0.0009, 0.0001],
    )
    for min_steps, want, probs in [
        (0, [[5]], [0.9]),
        (1, [[1, 5]], [0.09]),
        (2, [[1, 2, 5]], [0.009]),
    ]:
        search = BeamSearch(END, max_steps=10, beam_size=1, min_steps=min_steps)
        if min_steps == 0:
            with quiet():
                seqs, scores = run(search, matrix=SHORT)
        else:
            seqs, scores = run(search, matrix=SHORT)
        expect(seqs, scores, want, probs)
    seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=3, min_steps=2), matrix=SHORT)
    expect(seqs, scores, [[1, 2, 5, 5, 5], [1, 2, 3, 5, 5], [1, 2, 3, 4, 5]], [0.009, 0.0009, 0.0001])


def test_per_node_beam_size_and_bad_arguments():
    for k in (1, 2):
        with quiet():
            seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=3, per_node_beam_size=k))
        expect(seqs, scores, [[1, 2, 3, 4, 5], [2, 3, 4, 5, 5], [3, 4, 5, 5, 5]], [0.4, 0.3, 0.2])
    with pytest.raises(ValueError):
        run(BeamSearch(END, max_steps=10, beam_size=20))  # per-node width exceeds the vocabulary
    for kwargs in (dict(max_steps=0), dict(beam_size=0), dict(per_node_beam_size=0), dict(min_steps=-1), dict(max_steps=3, min_steps=4)):
        with pytest.raises(ValueError):
            BeamSearch(END, **kwargs)


def test_warnings_for_dead_ends_and_empty_output():
    with pytest.warns(RuntimeWarning, match="Negligible"):
        run(BeamSearch(END, max_steps=10, beam_size=5), batch=1)
    with pytest.warns(RuntimeWarning, match="Empty sequences"):
        seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=1), matrix=SHORT)
    assert seqs.shape == (5, 1, 1) and seqs.flatten().tolist() == [5] * 5


@pytest.mark.parametrize(
    "sampler",
    [TopPSampler(p=0.8), TopKSampler(k=3), TopKSampler(k=5, temperature=0.7, with_replacement=True), MultinomialSampler()],
)
def test_search_with_stochastic_node_samplers(sampler):
    torch.manual_seed(0)
    search = BeamSearch(END, max_steps=10, beam_size=2 if isinstance(sampler, MultinomialSampler) else 3, sampler=sampler)
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        seqs, scores = run(search)
    assert seqs.shape[-1] <= 10
    # beams come back best-first and every sequence follows the chain's only legal path
    assert bool((scores[:, :-1] >= scores[:, 1:]).all())
    first = seqs[..., 0]
    for t in range(1, seqs.shape[-1]):
        prev, cur = seqs[..., t - 1], seqs[..., t]
        ok = (cur == torch.clamp(prev + 1, max=END)) | (prev == END)
        live = torch.isfinite(scores) & (scores > -1e30)
        assert bool(ok[live].all())
    assert bool(((first >= 1) & (first <= 4)).all())


@pytest.mark.parametrize("p", [-1.0, 1.2])
def test_top_p_rejects_bad_p(p):
    with pytest.raises(ValueError):
        TopPSampler(p=p)


@pytest.mark.parametrize("k", [0, 7])
def test_top_k_rejects_bad_k(k):
    with pytest.raises(ValueError):
        run(BeamSearch(END, max_steps=5, beam_size=1, sampler=TopKSampler(k=k)))


LOGP = torch.log(torch.tensor([[0.1, 0.3, 0.3, 0.3, 0.0, 0.0], [0.0, 0.0, 0.4, 0.3, 0.2, 0.1]]))


def test_node_samplers_pick_from_support():
    torch.manual_seed(1)
    for sampler in (MultinomialSampler(), TopKSampler(k=4, temperature=2.0), TopPSampler(p=0.9, temperature=2.0)):
        probs, classes, state = sampler.sample_nodes(LOGP, 3, {"foo": "bar"})
        assert probs.shape == classes.shape == (2, 3)
        assert state == {"foo": "bar"}
        assert bool(torch.isfinite(probs).all())
        torch.testing.assert_close(probs, LOGP.gather(1, classes))
    # a tight nucleus keeps exactly the required number of tokens
    probs, classes, _ = TopPSampler(p=0.1).sample_nodes(LOGP, 2, {})
    assert sorted(classes[1].tolist()) == [2, 3]
    # top-k with k == per-node width returns exactly the top set
    probs, classes, _ = TopKSampler(k=3).sample_nodes(LOGP, 3, {})
    assert sorted(classes[0].tolist()) == [1, 2, 3] and sorted(classes[1].tolist()) == [2, 3, 4]
    probs, classes, _ = DeterministicSampler().sample_nodes(LOGP, 2, {})
    assert classes[1].tolist() == [2, 3]


def test_gumbel_sampler_contract_and_search():
    torch.manual_seed(2)
    sampler = GumbelSampler()
    state = sampler.init_state(LOGP, batch_size=2, num_classes=6)
    assert state["G_phi_S"].shape == (2, 6)
    beam_scores, beams, state = sampler.sample_beams(LOGP, 3, state)
    assert beams.shape == (2, 3) and state["G_phi_S"].shape == (6,) and state["phi_S"].shape == (6,)
    assert bool((beam_scores[:, :-1] >= beam_scores[:, 1:]).all())
    torch.testing.assert_close(beam_scores, LOGP.gather(1, beams))
    step_scores = torch.log_softmax(torch.randn(6, 6), dim=-1)
    node_scores, nodes, state2 = sampler.sample_nodes(step_scores, 2, state)
    assert nodes.shape == (6, 2) and state2["G_phi_S"].shape == (6, 2)
    # children never exceed their parent's perturbed score
    assert bool((state2["G_phi_S"] <= state["G_phi_S"].unsqueeze(-1) + 1e-4).all())

    # conditioned Gumbels: the row maximum equals the requested ceiling
    phi = torch.randn(4, 50)
    T = torch.randn(4, 1)
    g = sampler.gumbel_with_max(phi, T)
    torch.testing.assert_close(g.max(dim=-1, keepdim=True).values, T, atol=1e-4, rtol=1e-4)

    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        seqs, scores = run(BeamSearch(END, max_steps=10, beam_size=3, sampler=GumbelSampler()))
    # sampling without replacement: the three beams of a batch element are distinct sequences
    for b in range(seqs.shape[0]):
        assert len({tuple(s) for s in seqs[b].tolist()}) == 3


def test_length_normalised_scorer():
    with quiet():
        seqs, scores = run(
            BeamSearch(END, max_steps=10, beam_size=3, final_sequence_scorer=LengthNormalizedSequenceLogProbabilityScorer())
        )
    # lengths include one end token: 5, 4, 3
    want = torch.tensor([math.log(0.4) / 5, math.log(0.3) / 4, math.log(0.2) / 3])
    order = want.argsort(descending=True)
    torch.testing.assert_close(scores[0], want[order], rtol=1e-5, atol=1e-6)
    # a strong penalty prefers long sequences; scores come back sorted either way
    with quiet():
        seqs, scores = run(
            BeamSearch(
                END,
                max_steps=10,
                beam_size=3,
                final_sequence_scorer=LengthNormalizedSequenceLogProbabilityScorer(length_penalty=2.0),
            )
        )
    assert seqs[0, 0].tolist() == [1, 2, 3, 4, 5]
    # unfinished sequences are not credited an end token
    with quiet():
        seqs, scores = run(
            BeamSearch(END, max_steps=3, beam_size=3, final_sequence_scorer=LengthNormalizedSequenceLogProbabilityScorer())
        )
    got = {tuple(s): v for s, v in zip(seqs[0].tolist(), scores[0].tolist())}
    assert got[(1, 2, 3)] == pytest.approx(math.log(0.4) / 3, rel=1e-5)
    assert got[(3, 4, 5)] == pytest.approx(math.log(0.2) / 3, rel=1e-5)


def test_ngram_constraint_state_and_mask():
    c = RepeatedNGramBlockingConstraint(ngram_size=3)
    state = c.init_state(batch_size=2)
    scores = torch.zeros(2, 1, 6)
    assert bool((c.apply(state, scores) == 0).all())
    # two beams per batch element with explicit histories
    state = c.update_state(state, torch.tensor([[1, 1], [2, 2]]))
    state = c.update_state(state, torch.tensor([[2, 3], [3, 3]]), last_backpointer=torch.tensor([[0, 1], [0, 1]]))
    state = c.update_state(state, torch.tensor([[4, 1], [2, 3]]), last_backpointer=torch.tensor([[0, 0], [1, 1]]))
    state = c.update_state(state, torch.tensor([[1, 2], [3, 3]]), last_backpointer=torch.tensor([[1, 1], [0, 1]]))
    assert state["history"].tolist() == [[[1, 2, 1, 1], [1, 2, 1, 2]], [[2, 3, 2, 3], [2, 3, 3, 3]]]
    floor = torch.finfo(torch.float32).min
    masked = c.apply(state, torch.zeros(2, 2, 6))
    blocked = {(b, k): [v for v in range(6) if masked[b, k, v] == floor] for b in range(2) for k in range(2)}
    # [1,2,1,2]: prefix (1,2) was followed by 1;  [2,3,2,3]: (2,3) followed by 2;  [2,3,3,3]: (3,3) followed by 3
    assert blocked == {(0, 0): [], (0, 1): [1], (1, 0): [2], (1, 1): [3]}


def test_ngram_blocking_end_to_end():
    def go(n, steps, matrix=LOOPY):
        search = BeamSearch(END, max_steps=steps, beam_size=2, constraints=[RepeatedNGramBlockingConstraint(n)] if n else [])
        return run(search, matrix=matrix)

    expect(*go(0, 5), [[1, 3, 1, 3, 1], [1, 2, 3, 1, 3]], [0.36, 0.24])
    expect(*go(1, 3), [[1, 2, 3], [1, 3, 5]], [0.4, 0.6e-9])
    expect(*go(1, 5, DENSE), [[1, 2, 3, 4, 5], [1, 2, 4, 3, 5]], [0.4 * 0.3 * 0.3 * 0.2 * 0.1, 0.4 * 0.3 * 0.2 * 0.3 * 0.1])
    expect(*go(2, 4), [[1, 2, 3, 1], [1, 3, 1, 2]], [0.4, 0.24])
    expect(*go(3, 5), [[1, 2, 3, 1, 3], [1, 2, 3, 1, 2]], [0.24, 0.16])
    # finished beams keep emitting the end token even though a unigram constraint would block it
    expect(*go(1, 10), [[1, 3, 5, 5], [1, 2, 3, 5]], [0.6e-9, 0.4e-9])


def test_wide_beam_equals_exhaustive_enumeration_on_random_chains():
    """Property test: with a beam as wide as the number of distinct sequences, beam search is exhaustive, so on a random
    Markov chain its ranked output must equal a brute-force enumeration of all sequences (a sequence stops at the end
    token; the score is the sum of its transition log-probabilities up to and including the end token)."""
    import itertools

    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=25, deadline=None)
    @given(vocab=st.integers(2, 4), steps=st.integers(1, 3), seed=st.integers(0, 10**6), batch=st.integers(1, 2))
    def check(vocab, steps, seed, batch):
        g = torch.Generator().manual_seed(seed)
        chain = torch.softmax(3 * torch.randn(vocab, vocab, generator=g), dim=-1).log()  # row: last token, column: next
        end = vocab - 1
        starts = torch.randint(0, vocab - 1, (batch,), generator=g)

        def brute(start):
            found = {}
            for seq in itertools.product(range(vocab), repeat=steps):
                score, last, out = 0.0, start, []
                for tok in seq:
                    score += float(chain[last, tok])
                    out.append(tok)
                    last = tok
                    if tok == end:
                        break
                out = tuple(out + [end] * (steps - len(out)))  # a finished beam keeps emitting the end token at no cost
                found[out] = score
            return sorted(found.items(), key=lambda kv: -kv[1])

        beam = vocab**steps
        search = BeamSearch(end, max_steps=steps, beam_size=beam, per_node_beam_size=vocab)
        with quiet():
            preds, scores = search.search(starts, {}, lambda last, state, t: (chain[last], state))
        for b in range(batch):
            want = brute(int(starts[b]))
            got = [(tuple(int(x) for x in preds[b, i]), float(scores[b, i])) for i in range(beam) if float(scores[b, i]) > -1e30]  # spare beams carry -inf or the 'negligible' floor
            seen = {}
            for seq, score in got:  # duplicates of a finished sequence may fill spare beams; keep the first (best) of each
                seen.setdefault(seq, score)
            ranked = list(seen.items())
            assert [s for _, s in ranked] == sorted((s for _, s in ranked), reverse=True)
            assert len(ranked) == len(want)
            for (seq_a, score_a), (seq_b, score_b) in zip(ranked, want):
                assert score_a == pytest.approx(score_b, abs=1e-4)
            assert dict(ranked).keys() == dict(want).keys()
            assert ranked[0][0] == want[0][0] or ranked[0][1] == pytest.approx(want[1][1], abs=1e-5)

    check()
