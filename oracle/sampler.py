"""Restatement of the WeDLM commit rule (test infrastructure only).

* ``SamplingParams`` and presets      ``src/decoding/sampler.rs:12-44``, ``src/bin/cli.rs:113-137``
* ``compute_entropies_with_probs``    ``src/decoding/sampler.rs:125-154``
* ``sample_from_probs_at_indices``    ``src/decoding/sampler.rs:160-200`` (T = 0 branch; the
  T > 0 branches ``sample_from_probs`` / ``sample_nucleus``, ``sampler.rs:306-351``, with the
  uniform draw passed in, since the reference's ``thread_rng`` is unseeded)
* ``select_by_entropy_with_distance`` ``src/decoding/sampler.rs:446-493``
* streaming dynamic cap (entropy EMA) ``src/decoding/wedlm.rs:517-535``
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np


@dataclass
class SamplingParams:
    """``SamplingParams`` (``sampler.rs:12-44``); default values as ``Default``."""

    temperature: float = 0.2
    top_p: float = 1.0
    entropy_threshold: float = 0.6
    distance_penalty: float = 0.02
    max_tokens_per_step: int = 4
    margin_threshold: float = 0.0

    @staticmethod
    def preset(name: str, temperature: float = 0.0) -> "SamplingParams":
        """``Preset::to_params`` (``cli.rs:113-137``)."""
        table = {"quality": (0.5, 0.10, 4), "balanced": (0.8, 0.05, 8), "fast": (1.0, 0.05, 6)}
        tau, lam, cap = table[name]
        return SamplingParams(temperature=temperature, entropy_threshold=tau,
                              distance_penalty=lam, max_tokens_per_step=cap)


def scale_logits(logits: np.ndarray, temperature: float) -> np.ndarray:
    """Logits are divided by T only when ``T > 0 && T != 1`` (``sampler.rs:127-131``)."""
    x = np.asarray(logits, dtype=np.float32)
    if temperature > 0.0 and temperature != 1.0:
        x = (x / np.float32(temperature)).astype(np.float32)
    return x


def compute_entropies_with_probs(logits: np.ndarray, temperature: float) -> Tuple[np.ndarray, np.ndarray]:
    """``compute_entropies_with_probs`` (``sampler.rs:125-154``).

    Softmax over the (scaled) logits, then ``H = sum_{p>0} -p ln p``.  The sum is
    accumulated in float64 here; the reference accumulates in f32, which differs
    from the exact value by O(sqrt(V) * 2^-24) relative.
    """
    x = scale_logits(logits, temperature).astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    p = e / e.sum(axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        t = np.where(p > 0, -p * np.log(np.where(p > 0, p, 1.0)), 0.0)
    H = t.sum(axis=-1).astype(np.float32)
    return H, p.astype(np.float32)


def row_stats(logits: np.ndarray, temperature: float):
    """Per-row (entropy, argmax, max-prob) from the logits in one pass.

    Argmax follows ``sampler.rs:183-190``: ``Iterator::max_by`` returns the LAST
    maximum, so ties resolve to the largest index.  The max probability is
    ``exp(x_max - m) / sum exp(x - m)``.
    """
    x = scale_logits(logits, temperature).astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    S = e.sum(axis=-1)
    T = (e * x).sum(axis=-1)
    H = (m[:, 0] + np.log(S) - T / S).astype(np.float32)
    xr = x[:, ::-1]
    am = (x.shape[1] - 1 - np.argmax(xr, axis=-1)).astype(np.int32)
    maxp = (1.0 / S).astype(np.float32)
    return H, am, maxp


def shard_partials(logits_shard: np.ndarray, vocab_offset: int, temperature: float):
    """Per-row partial softmax statistics of one vocabulary shard (columns
    ``vocab_offset ..``): max m, S = sum exp(x - m), T = sum exp(x - m) * x, and the
    shard's last-max argmax as a global column.  The split of ``row_stats`` over
    shards that the vocab-sharded LM head uses; ``combine_partials`` merges them."""
    x = scale_logits(logits_shard, temperature).astype(np.float64)
    m = x.max(axis=-1)
    e = np.exp(x - m[:, None])
    S = e.sum(axis=-1)
    T = (e * x).sum(axis=-1)
    am = vocab_offset + (x.shape[1] - 1 - np.argmax(x[:, ::-1], axis=-1))
    return m, S, T, am.astype(np.int64)


def combine_partials(parts):
    """Merge shard partials (list of ``shard_partials`` results, in vocabulary order):
    m = max m_r, S = sum S_r e^(m_r - m), T = sum T_r e^(m_r - m), H = m + ln S - T / S;
    the argmax is the largest value, ties to the largest global column; max-prob 1 / S."""
    m = np.max(np.stack([p[0] for p in parts]), axis=0)
    S = sum(p[1] * np.exp(p[0] - m) for p in parts)
    T = sum(p[2] * np.exp(p[0] - m) for p in parts)
    H = (m + np.log(S) - T / S).astype(np.float32)
    am = parts[0][3].copy()
    best = parts[0][0].copy()
    for p in parts[1:]:
        take = p[0] >= best  # later shards hold larger columns: ties go to them
        am = np.where(take, p[3], am)
        best = np.where(take, p[0], best)
    return H, am.astype(np.int32), (1.0 / S).astype(np.float32)


_MASK64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    """The SplitMix64 output function (Steele, Lea and Flood, OOPSLA 2014)."""
    x = (x + 0x9E3779B97F4A7C15) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def sampling_uniform(seed: int, seq: int, step: int, row: int) -> np.float32:
    """The seeded draw of the device sampler for mask row ``row`` of sequence ``seq`` at
    decode step ``step`` (1-based): a 24-bit uniform in [0, 1), the precision of the
    reference's ``rng.gen::<f32>()``."""
    h = splitmix64(seed & _MASK64)
    h = splitmix64(h ^ (seq & _MASK64))
    h = splitmix64(h ^ (step & _MASK64))
    h = splitmix64(h ^ (row & _MASK64))
    return np.float32((h >> 40) * 2.0 ** -24)


def sample_from_probs(probs: np.ndarray, r: float) -> int:
    """``sample_from_probs`` (``sampler.rs:306-317``) with the draw ``r`` given: the first
    index whose running sum exceeds r; the last index when rounding leaves none.  The
    running sums are float64 here; the reference's f32 running sum differs from the exact
    one by O(V * 2^-24)."""
    c = np.cumsum(np.asarray(probs, np.float64))
    hit = np.nonzero(float(r) < c)[0]
    return int(hit[0]) if hit.size else int(len(c) - 1)


def sample_nucleus(probs: np.ndarray, top_p: float, r: float) -> int:
    """``sample_nucleus`` (``sampler.rs:320-351``) with the draw ``r`` given: probabilities
    sorted descending (stable, so ties keep index order), the smallest prefix whose running
    sum reaches top_p, renormalised, and the first member whose running sum exceeds
    r * total; the most probable token when rounding leaves none.  Sums in float64, as in
    ``sample_from_probs``."""
    p = np.asarray(probs, np.float64)
    order = np.argsort(-p, kind="stable")
    ps = p[order]
    c = np.cumsum(ps)
    reach = np.nonzero(c >= float(np.float32(top_p)))[0]
    cut = int(reach[0]) + 1 if reach.size else len(ps)
    run = c[:cut]
    total = run[-1]
    target = float(r) * total
    hit = np.nonzero(target < run)[0]
    return int(order[hit[0]]) if hit.size else int(order[0])


def greedy_argmax_last(probs_row: np.ndarray) -> int:
    """T = 0 branch of ``sample_from_probs_at_indices`` (``sampler.rs:183-190``)."""
    r = np.asarray(probs_row)
    return int(r.shape[0] - 1 - np.argmax(r[::-1]))


def select_by_entropy_with_distance(entropies: Sequence[float], mask_indices: Sequence[int],
                                    entropy_threshold: float, distance_penalty: float,
                                    max_positions: int) -> List[int]:
    """``select_by_entropy_with_distance`` (``sampler.rs:446-493``).

    ``adj_i = H_i + lambda * (pos_i - min pos)`` (f32 arithmetic); keep ``adj < tau``
    in ascending logical position (stable sort), ``take(max_positions)``; if none,
    the first minimum of ``adj`` in logical order.
    """
    if len(entropies) == 0 or len(mask_indices) == 0:
        return []
    leftmost = min(mask_indices)
    lam = np.float32(distance_penalty)
    items = []
    for i, h in enumerate(entropies):
        lp = mask_indices[i] if i < len(mask_indices) else i
        dist = np.float32(max(lp - leftmost, 0))
        adj = np.float32(np.float32(h) + np.float32(lam * dist))
        items.append((i, lp, adj))
    items.sort(key=lambda t: t[1])  # stable, like sort_by_key
    tau = np.float32(entropy_threshold)
    res = [i for (i, _, a) in items if a < tau][:max_positions]
    if not res and items:
        best = items[0]
        for it in items[1:]:
            if it[2] < best[2]:
                best = it
        res = [best[0]]
    return res


ENTROPY_EMA_ALPHA = np.float32(0.3)


def update_running_entropy(running: float, entropies: Sequence[float]) -> np.float32:
    """Entropy EMA (``wedlm.rs:517-522``): ``r = 0.3 * mean(H) + 0.7 * r`` in f32."""
    if len(entropies) == 0:
        return np.float32(running)
    s = np.float32(0.0)
    for h in entropies:  # sequential f32 sum, like Iterator::sum::<f32>
        s = np.float32(s + np.float32(h))
    avg = np.float32(s / np.float32(len(entropies)))
    return np.float32(ENTROPY_EMA_ALPHA * avg + (np.float32(1.0) - ENTROPY_EMA_ALPHA) * np.float32(running))


def effective_cap(running: float, tau: float, cap: int) -> int:
    """Dynamic per-step cap (``wedlm.rs:526-535``)."""
    r, t = np.float32(running), np.float32(tau)
    if r < t * np.float32(0.4):
        return cap * 2
    if r < t * np.float32(0.7):
        return (cap * 3 + 1) // 2
    return cap
