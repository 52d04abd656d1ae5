"""
Beam search decoding with pluggable samplers, final-sequence scorers and constraints.

The public surface (class names, constructor arguments, tensor shapes of every hook) follows the
reference's ``olmo/beam_search.py:44-1078`` so that user-written samplers, scorers, constraints and
step functions plug in unchanged.  The implementation differs:

* the search keeps one ``[batch, beam, t]`` token history that is re-indexed by the surviving
  beams' parents after every step, instead of storing per-step predictions plus back-pointers and
  rebuilding sequences at the end;
* the repeated-n-gram constraint is evaluated with tensor ops over that kind of history (no Python
  dictionaries per beam), so it stays on the device.

Terminology: a *node* is one candidate next token of one beam, a *beam* is one partial sequence.
"""
from __future__ import annotations

import warnings
from abc import abstractmethod
from inspect import signature
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "Sampler",
    "DeterministicSampler",
    "MultinomialSampler",
    "TopKSampler",
    "TopPSampler",
    "GumbelSampler",
    "FinalSequenceScorer",
    "SequenceLogProbabilityScorer",
    "LengthNormalizedSequenceLogProbabilityScorer",
    "Constraint",
    "RepeatedNGramBlockingConstraint",
    "BeamSearch",
]

StateType = Dict[str, torch.Tensor]
StepFunctionType = Callable[..., Tuple[torch.Tensor, StateType]]
ConstraintStateType = Any


def _lowest(t: torch.Tensor) -> float:
    return torch.finfo(t.dtype).min


# ---------------------------------------------------------------------------------------- samplers


class Sampler:
    """
    Chooses candidates during the search.

    ``sample_nodes(log_probs[group, vocab], k, state)`` picks ``k`` next tokens per beam;
    ``sample_beams(log_probs[batch, beam * k], beam_size, state)`` picks the surviving beams.  Both
    return ``(chosen log-probs, chosen indices, new state)``.  ``init_state`` may prepare tensors
    that the two calls pass along.  (``olmo/beam_search.py:44-99``)
    """

    def init_state(self, start_class_log_probabilities: torch.Tensor, batch_size: int, num_classes: int) -> StateType:
        return {}

    @abstractmethod
    def sample_nodes(
        self, log_probs: torch.Tensor, per_node_beam_size: int, state: StateType
    ) -> Tuple[torch.Tensor, torch.Tensor, StateType]:
        raise NotImplementedError

    def sample_beams(
        self, log_probs: torch.Tensor, beam_size: int, state: StateType
    ) -> Tuple[torch.Tensor, torch.Tensor, StateType]:
        values, indices = log_probs.topk(beam_size, dim=-1)
        return values, indices, {}


class DeterministicSampler(Sampler):
    """Plain beam search: the highest-scoring nodes and beams win."""

    def sample_nodes(self, log_probs, per_node_beam_size, state):
        values, indices = log_probs.topk(per_node_beam_size, dim=-1)
        return values, indices, {}


def _tempered_probs(log_probs: torch.Tensor, temperature: float) -> torch.Tensor:
    if temperature == 1.0:
        return log_probs.exp()
    return F.softmax(log_probs / temperature, dim=-1)


class MultinomialSampler(Sampler):
    """Draw nodes from the (optionally tempered) categorical distribution; beams by top-k."""

    def __init__(self, temperature: float = 1.0, with_replacement: bool = False) -> None:
        self.temperature = temperature
        self.with_replacement = with_replacement

    def sample_nodes(self, log_probs, per_node_beam_size, state):
        draws = torch.multinomial(
            _tempered_probs(log_probs, self.temperature), per_node_beam_size, replacement=self.with_replacement
        )
        return log_probs.gather(1, draws), draws, state


class TopKSampler(Sampler):
    """Draw nodes from the ``k`` most likely tokens, renormalised.  (``olmo/beam_search.py:148-203``)"""

    def __init__(self, k: int = 1, temperature: float = 1.0, with_replacement: bool = False):
        self.k = k
        self.temperature = temperature or 1.0
        self.with_replacement = with_replacement

    def sample_nodes(self, log_probs, per_node_beam_size, state):
        vocab = log_probs.shape[1]
        if not (per_node_beam_size <= self.k <= vocab):
            raise ValueError("k must be at least per_node_beam_size and at most the vocabulary size")
        head, head_ids = log_probs.topk(self.k, dim=-1)
        weights = F.softmax(head / self.temperature, dim=-1)
        pick = torch.multinomial(weights, per_node_beam_size, replacement=self.with_replacement)
        chosen = head_ids.gather(-1, pick)
        return log_probs.gather(1, chosen), chosen, state


class TopPSampler(Sampler):
    """
    Nucleus sampling: draw nodes from the smallest set of tokens whose probability mass reaches
    ``p`` (always keeping at least ``per_node_beam_size`` tokens when drawing without replacement).
    (``olmo/beam_search.py:205-288``)
    """

    def __init__(self, p: float = 0.9, temperature: float = 1.0, with_replacement: bool = False):
        if not 0.0 <= p <= 1.0:
            raise ValueError("p must lie in [0, 1]")
        self.p = p
        self.temperature = temperature or 1.0
        self.with_replacement = with_replacement

    def sample_nodes(self, log_probs, per_node_beam_size, state):
        if per_node_beam_size > log_probs.shape[1]:
            raise ValueError("per_node_beam_size cannot exceed the vocabulary size")
        scaled = log_probs if self.temperature == 1.0 else F.log_softmax(log_probs / self.temperature, dim=-1)
        ordered, order = scaled.sort(dim=-1, descending=True)
        mass_before = ordered.exp().cumsum(dim=-1) - ordered.exp()
        # a token is outside the nucleus when the tokens ranked above it already hold mass >= p
        outside = mass_before >= self.p
        outside[..., 0] = False
        if not self.with_replacement:
            outside[..., :per_node_beam_size] = False
        weights = F.softmax(ordered.masked_fill(outside, _lowest(log_probs)), dim=-1)
        pick = torch.multinomial(weights, per_node_beam_size, replacement=self.with_replacement)
        chosen = order.gather(-1, pick)
        return log_probs.gather(1, chosen), chosen, state


class GumbelSampler(Sampler):
    """
    Stochastic beam search (Kool et al., 2019): beams are sampled without replacement by perturbing
    sequence log-probabilities with Gumbel noise whose maximum over each beam's children is tied to
    the parent's perturbed score.  State carries ``G_phi_S`` (perturbed scores) and ``phi_S`` (true
    scores).  (``olmo/beam_search.py:291-421``)
    """

    def __init__(self, temperature: float = 1.0):
        self.temperature = temperature

    def init_state(self, start_class_log_probabilities, batch_size, num_classes):
        ceiling = start_class_log_probabilities.new_zeros((batch_size, num_classes))
        return {"G_phi_S": self.gumbel_with_max(start_class_log_probabilities, ceiling)}

    def sample_nodes(self, log_probs, per_node_beam_size, state):
        scaled = log_probs if self.temperature == 1.0 else F.log_softmax(log_probs / self.temperature, dim=-1)
        child_scores = state["phi_S"].unsqueeze(-1) + scaled
        perturbed = self.gumbel_with_max(child_scores, state["G_phi_S"].unsqueeze(-1))
        top_perturbed, chosen = perturbed.topk(per_node_beam_size, dim=-1)
        return log_probs.gather(1, chosen), chosen, {"G_phi_S": top_perturbed}

    def sample_beams(self, log_probs, beam_size, state):
        batch = log_probs.shape[0]
        perturbed = state["G_phi_S"].reshape_as(log_probs)
        kept_perturbed, kept = perturbed.topk(beam_size, dim=-1)
        kept_scores = log_probs.gather(1, kept)
        # order survivors by their true score so that beam 0 is the most likely one
        kept_scores, by_score = kept_scores.sort(dim=-1, descending=True)
        kept = kept.gather(1, by_score)
        kept_perturbed = kept_perturbed.gather(1, by_score)
        return (
            kept_scores,
            kept,
            {"G_phi_S": kept_perturbed.reshape(batch * beam_size), "phi_S": kept_scores.reshape(batch * beam_size)},
        )

    def gumbel(self, phi: torch.Tensor) -> torch.Tensor:
        """One ``Gumbel(phi)`` sample per element."""
        return phi - torch.log(-torch.log(torch.rand_like(phi)))

    def gumbel_with_max(self, phi: torch.Tensor, T: torch.Tensor) -> torch.Tensor:
        """``Gumbel(phi)`` samples conditioned on their row maximum being ``T`` (numerically stable form)."""
        g = self.gumbel(phi)
        row_max = g.max(dim=-1, keepdim=True).values
        v = T - g + torch.log1p(-torch.exp(g - row_max))
        return T - F.relu(v) - torch.log1p(torch.exp(-v.abs()))


# ----------------------------------------------------------------------------------------- scorers


class FinalSequenceScorer:
    """Ranks finished beams.  ``score(predictions[b, k, t], log_probabilities[b, k], end_index) -> [b, k]``."""

    @abstractmethod
    def score(self, predictions: torch.Tensor, log_probabilities: torch.Tensor, end_index: int) -> torch.Tensor:
        raise NotImplementedError


class SequenceLogProbabilityScorer(FinalSequenceScorer):
    """Score = summed token log-probability."""

    def score(self, predictions, log_probabilities, end_index):
        return log_probabilities


class LengthNormalizedSequenceLogProbabilityScorer(FinalSequenceScorer):
    """
    Score = log-probability / length ** ``length_penalty``; the length counts one end token if the
    sequence finished.  (``olmo/beam_search.py:462-491``)
    """

    def __init__(self, length_penalty: float = 1.0):
        self.length_penalty = length_penalty

    def score(self, predictions, log_probabilities, end_index):
        content = (predictions != end_index).sum(dim=2)
        finished = (predictions[:, :, -1] == end_index).to(content.dtype)
        return log_probabilities / (content + finished) ** self.length_penalty


# ------------------------------------------------------------------------------------- constraints


class Constraint:
    """
    Vetoes candidate tokens.  ``init_state(batch_size)`` builds per-batch state for a single start
    beam; ``apply(state, log_probs[batch, beam, vocab])`` returns the masked log-probs;
    ``update_state(state, last_prediction[batch, beam], last_backpointer)`` re-indexes the state by
    the surviving beams' parents and records the new tokens.  (``olmo/beam_search.py:494-590``)
    """

    @abstractmethod
    def init_state(self, batch_size: int) -> ConstraintStateType:
        raise NotImplementedError

    @abstractmethod
    def apply(self, state: ConstraintStateType, class_log_probabilities: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    @abstractmethod
    def update_state(
        self,
        state: ConstraintStateType,
        last_prediction: torch.Tensor,
        last_backpointer: Optional[torch.Tensor] = None,
    ) -> ConstraintStateType:
        raise NotImplementedError


class RepeatedNGramBlockingConstraint(Constraint):
    """
    Forbid producing any n-gram twice within a beam.  State is the beam's token history
    ``[batch, beam, t]`` (``None`` before the first token).
    """

    def __init__(self, ngram_size: int) -> None:
        if ngram_size < 1:
            raise ValueError("ngram_size must be positive")
        self.ngram_size = ngram_size

    def init_state(self, batch_size: int) -> ConstraintStateType:
        return {"history": None, "batch_size": batch_size}

    def apply(self, state, class_log_probabilities):
        history = state["history"]
        n = self.ngram_size
        if history is None or history.shape[-1] < n:
            if n == 1 and history is not None and history.shape[-1] >= 1:
                pass
            else:
                return class_log_probabilities
        t = history.shape[-1]
        if n == 1:
            banned_tokens = history  # every token produced so far
            hit = torch.ones_like(history, dtype=torch.bool)
        else:
            windows = history.unfold(-1, n, 1)  # [b, k, t-n+1, n] : all complete n-grams so far
            tail = history[..., t - (n - 1) :]  # the prefix the next token would extend
            hit = (windows[..., : n - 1] == tail.unsqueeze(-2)).all(dim=-1)
            banned_tokens = windows[..., n - 1]
        floor = _lowest(class_log_probabilities)
        mask = torch.zeros_like(class_log_probabilities, dtype=torch.bool)
        # beams of the history line up with beams of the scores except on the very first call,
        # where the history has one beam per batch element
        mask.scatter_(-1, banned_tokens.expand(*mask.shape[:2], -1), hit.expand(*mask.shape[:2], -1))
        return class_log_probabilities.masked_fill(mask, floor)

    def update_state(self, state, last_prediction, last_backpointer=None):
        history = state["history"]
        if history is None:
            new_history = last_prediction.unsqueeze(-1)
        else:
            if last_backpointer is None:
                parents = history.expand(-1, last_prediction.shape[1], -1)
            else:
                parents = history.gather(1, last_backpointer.unsqueeze(-1).expand(-1, -1, history.shape[-1]))
            new_history = torch.cat([parents, last_prediction.unsqueeze(-1)], dim=-1)
        return {"history": new_history, "batch_size": state["batch_size"]}


# ------------------------------------------------------------------------------------------ search


class BeamSearch:
    """
    Batched beam search over a user-supplied step function.

    :param end_index: id of the end-of-sequence token; a beam that emits it keeps emitting it.
    :param max_steps: number of tokens to generate at most.
    :param beam_size: beams kept per batch element.
    :param per_node_beam_size: candidate tokens considered per beam and step (default ``beam_size``).
    :param sampler: candidate selection policy (default :class:`DeterministicSampler`).
    :param min_steps: the end token is forbidden for this many leading steps.
    :param final_sequence_scorer: ranks the finished beams (default: summed log-probability).
    :param constraints: vetoes applied to every step's scores.

    (``olmo/beam_search.py:649-1078``)
    """

    def __init__(
        self,
        end_index: int,
        *,
        max_steps: int = 50,
        beam_size: int = 10,
        per_node_beam_size: Optional[int] = None,
        sampler: Optional[Sampler] = None,
        min_steps: Optional[int] = None,
        final_sequence_scorer: Optional[FinalSequenceScorer] = None,
        constraints: Optional[List[Constraint]] = None,
    ) -> None:
        if max_steps <= 0:
            raise ValueError("max_steps must be positive")
        if beam_size <= 0:
            raise ValueError("beam_size must be positive")
        if per_node_beam_size is not None and per_node_beam_size <= 0:
            raise ValueError("per_node_beam_size must be positive")
        if min_steps is not None and not (0 <= min_steps <= max_steps):
            raise ValueError("min_steps must lie in [0, max_steps]")
        self._end_index = end_index
        self.max_steps = max_steps
        self.beam_size = beam_size
        self.per_node_beam_size = per_node_beam_size or beam_size
        self.sampler = sampler or DeterministicSampler()
        self.min_steps = min_steps or 0
        self.final_sequence_scorer = final_sequence_scorer or SequenceLogProbabilityScorer()
        self.constraints = constraints or []

    # -- state bookkeeping ---------------------------------------------------------------------

    def _fan_out(self, state: StateType, batch: int) -> None:
        """``[batch, ...]`` -> ``[batch * beam, ...]`` with every beam starting from the same state."""
        for key, value in state.items():
            if value is not None:
                state[key] = value.repeat_interleave(self.beam_size, dim=0)

    def _follow_parents(self, state: StateType, parents: torch.Tensor) -> None:
        """Re-index ``[batch * beam, ...]`` state tensors by the parent beam of every survivor."""
        batch = parents.shape[0]
        flat = (parents + torch.arange(batch, device=parents.device).unsqueeze(1) * self.beam_size).reshape(-1)
        for key, value in state.items():
            if value is not None:
                state[key] = value.index_select(0, flat)

    def _constrain(self, scores: torch.Tensor, batch: int, constraint_states: List[ConstraintStateType]):
        if not self.constraints:
            return scores
        shaped = scores.reshape(batch, -1, scores.shape[-1])
        for constraint, cstate in zip(self.constraints, constraint_states):
            shaped = constraint.apply(cstate, shaped)
        return shaped.reshape(scores.shape)

    # -- public --------------------------------------------------------------------------------

    def search(
        self, start_predictions: torch.Tensor, start_state: StateType, step: StepFunctionType
    ) -> Tuple[torch.Tensor, torch.Tensor]:
        """
        :param start_predictions: ``[batch]`` start tokens.
        :param start_state: tensors of shape ``[batch, ...]`` handed to ``step``.
        :param step: ``step(last_tokens[group], state[, timestep]) -> (log_probs[group, vocab], state)``
            with ``group`` equal to ``batch`` on the first call and ``batch * beam_size`` after it.
        :returns: ``(predictions[batch, beam, <=max_steps], scores[batch, beam])``, best beam first.
        """
        if len(signature(step).parameters) < 3:
            two_arg = step

            def step(tokens, state, timestep):  # type: ignore[no-redef]
                return two_arg(tokens, state)

        return self._search(start_predictions, start_state, step)

    def _search(self, start_predictions, start_state, step):
        batch = start_predictions.shape[0]
        B, K, end = self.beam_size, self.per_node_beam_size, self._end_index
        constraint_states = [c.init_state(batch) for c in self.constraints]

        first_scores, state = step(start_predictions, start_state, 0)
        vocab = first_scores.shape[1]
        if K > vocab:
            raise ValueError(
                f"Vocab size ({vocab:d}) too small relative to per_node_beam_size ({K:d}).\n"
                f"Please decrease beam_size or per_node_beam_size."
            )
        sampler_state = self.sampler.init_state(first_scores, batch, vocab)
        first_scores = self._constrain(first_scores, batch, constraint_states)
        if self.min_steps >= 1:
            first_scores[:, end] = _lowest(first_scores)

        if B > vocab:
            # More beams than first tokens: take every token once and fill the spare beams with finished sequences of
            # score -inf, which can never displace a real candidate.  (Only meaningful for the deterministic sampler;
            # the stochastic ones keep per-beam state that cannot be padded.)
            if type(self.sampler) is not DeterministicSampler:
                raise ValueError(f"beam_size ({B:d}) exceeds the vocabulary size ({vocab:d}); decrease beam_size")
            beam_scores, tokens, sampler_state = self.sampler.sample_beams(first_scores, vocab, sampler_state)
            beam_scores = torch.cat([beam_scores, beam_scores.new_full((batch, B - vocab), float("-inf"))], dim=1)
            tokens = torch.cat([tokens, tokens.new_full((batch, B - vocab), end)], dim=1)
        else:
            beam_scores, tokens, sampler_state = self.sampler.sample_beams(first_scores, B, sampler_state)
        if B == 1 and bool((tokens == end).all()):
            warnings.warn(
                "Empty sequences predicted. You may want to increase the beam size or ensure "
                "your step function is working properly.",
                RuntimeWarning,
            )
            return tokens.unsqueeze(-1), beam_scores

        history = tokens.unsqueeze(-1)  # [batch, beam, 1]
        # once a beam has ended, the only continuation with non-negligible probability is `end`
        ended_row = first_scores.new_full((vocab,), _lowest(first_scores))
        ended_row[end] = 0.0

        self._fan_out(state, batch)
        for i, c in enumerate(self.constraints):
            constraint_states[i] = c.update_state(constraint_states[i], tokens)

        for t in range(1, self.max_steps):
            last = history[..., -1].reshape(batch * B)
            if bool((last == end).all()):
                break
            scores, state = step(last, state, t)
            scores = self._constrain(scores, batch, constraint_states)
            if t + 1 <= self.min_steps:
                scores[:, end] = _lowest(scores)
            scores = torch.where((last == end).unsqueeze(-1), ended_row, scores)

            node_scores, node_tokens, sampler_state = self.sampler.sample_nodes(scores, K, sampler_state)
            totals = (node_scores.reshape(batch, B, K) + beam_scores.unsqueeze(-1)).reshape(batch, B * K)
            beam_scores, kept, sampler_state = self.sampler.sample_beams(totals, B, sampler_state)
            tokens = node_tokens.reshape(batch, B * K).gather(1, kept)
            parents = torch.div(kept, K, rounding_mode="trunc")

            history = torch.cat(
                [history.gather(1, parents.unsqueeze(-1).expand(-1, -1, history.shape[-1])), tokens.unsqueeze(-1)],
                dim=-1,
            )
            self._follow_parents(state, parents)
            for i, c in enumerate(self.constraints):
                constraint_states[i] = c.update_state(constraint_states[i], tokens, last_backpointer=parents)

        if not self.constraints and (
            not bool(torch.isfinite(beam_scores).all()) or bool((beam_scores == _lowest(beam_scores)).any())
        ):
            warnings.warn(
                "Negligible log probabilities encountered ('-inf' or equivalent). "
                "Some final sequences may not make sense. "
                "This can happen when the beam size is larger than the number of valid (non-zero "
                "probability) transitions that the step function produces.",
                RuntimeWarning,
            )

        final = self.final_sequence_scorer.score(history, beam_scores, end)
        final, order = final.sort(dim=1, descending=True)
        return history.gather(1, order.unsqueeze(-1).expand_as(history)), final
