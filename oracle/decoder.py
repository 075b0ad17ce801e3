"""Restatement of the WeDLM decode loops (test infrastructure only).

* ``compute_block_reorder_into``  ``src/decoding/reorder.rs:57-90``
* ``topological_reorder_cpu``     ``src/decoding/reorder.rs:98-139``
* ``WeDLMDecoder::generate_streaming`` ``src/decoding/wedlm.rs:336-590``
  (commit-before-predict, cache truncate, EMA cap, refill)
* ``WeDLMDecoder::generate_block`` / ``commit_block_to_cache`` /
  ``generate_with_stats``         ``src/decoding/wedlm.rs:106-296,610-714``

The model is any object with ``forward_with_positions(ids, positions, caches)``
returning ``(logits [S, V], new_caches)`` and ``prefill_cache(ids)``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from .sampler import (SamplingParams, compute_entropies_with_probs, effective_cap,
                      greedy_argmax_last, sample_from_probs, sample_nucleus,
                      sampling_uniform, scale_logits, select_by_entropy_with_distance,
                      update_running_entropy)

ENTROPY_SOFT_THRESHOLD = 8.0   # wedlm.rs:29
ENTROPY_HARD_THRESHOLD = 12.0  # wedlm.rs:32
MAX_CACHED_LENGTH = 16384      # wedlm.rs:35
CACHE_CHECK_INTERVAL = 32      # wedlm.rs:38


@dataclass
class BlockReorderResult:
    """``BlockReorderResult`` (``reorder.rs:21-30``)."""

    reordered_block: List[int] = field(default_factory=list)
    positions: List[int] = field(default_factory=list)
    block_permutation: List[int] = field(default_factory=list)
    num_filled: int = 0


def compute_block_reorder(block_tokens: Sequence[int], mask_positions: Sequence[int],
                          prefix_len: int) -> BlockReorderResult:
    """``compute_block_reorder_into`` (``reorder.rs:57-90``): filled indices in
    ascending order, then ``mask_positions`` in the given order; positions are
    ``prefix_len + block_pos``."""
    r = BlockReorderResult()
    mset = set(mask_positions)
    r.block_permutation = [i for i in range(len(block_tokens)) if i not in mset]
    r.num_filled = len(r.block_permutation)
    r.block_permutation += list(mask_positions)
    r.reordered_block = [block_tokens[p] for p in r.block_permutation]
    r.positions = [prefix_len + p for p in r.block_permutation]
    return r


def topological_reorder_cpu(ids: Sequence[int], mask_positions: Sequence[int]):
    """``topological_reorder_cpu`` (``reorder.rs:98-139``)."""
    mset = set(mask_positions)
    known = [i for i in range(len(ids)) if i not in mset]
    unknown = [i for i in range(len(ids)) if i in mset]
    perm = known + unknown
    inv = [0] * len(ids)
    for new, old in enumerate(perm):
        inv[old] = new
    return [ids[i] for i in perm], perm, inv, len(known)


@dataclass
class BlockStats:
    """``BlockStats`` (``wedlm.rs:41-58``)."""

    steps: int = 0
    tokens_generated: int = 0
    avg_confidence: float = 0.0
    avg_entropy: float = 0.0
    max_entropy: float = 0.0
    high_entropy_count: int = 0
    block_size_reductions: int = 0
    cache_refreshes: int = 0
    prefix_cached: bool = False


@dataclass
class StepTrace:
    """What one streaming step did (for step-by-step parity checks)."""

    n_commit: int
    reordered_tokens: List[int]
    reordered_positions: List[int]
    num_filled: int
    mask_logical_indices: List[int]
    entropies: List[float]
    effective_max: int
    selected: List[int]
    sampled: List[int]


class OracleDecoder:
    """``WeDLMDecoder`` restated; the cache is a Python list of per-layer (K, V)."""

    def __init__(self, model, mask_token_id: int, eos_token_id: int, seed: int = 0,
                 seq_index: int = 0):
        self.model = model
        self.mask = int(mask_token_id)
        self.eos = int(eos_token_id)
        self.cache = None
        self.cache_len = 0
        self.trace: List[StepTrace] = []
        # T > 0: the seeded draws of the device sampler (``sampling_uniform``)
        self.seed = int(seed)
        self.seq_index = int(seq_index)

    def _truncate(self, new_len: int):
        """``truncate_cache`` (``wedlm.rs:308-323``)."""
        if new_len >= self.cache_len:
            return
        self.cache = [(k[:, :new_len], v[:, :new_len]) for (k, v) in self.cache]
        self.cache_len = new_len

    def _sample(self, probs, selected, params, step: int, logits=None):
        """``sample_from_probs_at_indices`` (``sampler.rs:160-200``).  T > 0 draws
        ``sampling_uniform(seed, seq_index, step, row)`` in place of the reference's
        unseeded ``thread_rng``, over float64 probabilities of ``logits`` (the mask rows)."""
        if params.temperature == 0.0:
            return [greedy_argmax_last(probs[i]) for i in selected]
        x = scale_logits(np.asarray(logits), params.temperature).astype(np.float64)
        e = np.exp(x - x.max(axis=-1, keepdims=True))
        probs = e / e.sum(axis=-1, keepdims=True)
        out = []
        for i in selected:
            u = sampling_uniform(self.seed, self.seq_index, step, i)
            if params.top_p >= 1.0:
                out.append(sample_from_probs(probs[i], u))
            else:
                out.append(sample_nucleus(probs[i], params.top_p, u))
        return out

    def generate_streaming(self, prompt_ids: Sequence[int], max_new_tokens: int,
                           window_size: int, params: SamplingParams):
        """``generate_streaming`` (``wedlm.rs:336-590``).  Returns
        ``(prompt ++ output ids, BlockStats)``."""
        prompt = [int(t) for t in prompt_ids]
        P = len(prompt)
        stats = BlockStats(prefix_cached=True)
        self.cache = self.model.prefill_cache(prompt)
        self.cache_len = P
        self.trace = []
        committed_len = P
        next_pos = P
        out: List[int] = []
        running = np.float32(params.entropy_threshold)
        init = min(window_size, max_new_tokens)
        win = [self.mask] * init
        win_pos = list(range(next_pos, next_pos + init))
        next_pos += init
        while len(out) < max_new_tokens:
            stats.steps += 1
            n_commit = 0
            for t in win:
                if t == self.mask:
                    break
                n_commit += 1
            mask_logical = [i for i, t in enumerate(win) if t == self.mask]
            if len(win) == 0:
                break
            ro = compute_block_reorder(win, mask_logical, 0)
            rpos = [win_pos[i] for i in ro.block_permutation]
            num_filled, num_mask = ro.num_filled, len(mask_logical)
            logits, new_cache = self.model.forward_with_positions(ro.reordered_block, rpos, self.cache)
            self.cache = new_cache
            self.cache_len = committed_len + len(win)
            remaining = max(max_new_tokens - len(out), 0)
            n_commit = min(n_commit, remaining)
            self._truncate(committed_len + n_commit)
            tr = StepTrace(n_commit, list(ro.reordered_block), list(rpos), num_filled,
                           list(mask_logical), [], 0, [], [])
            self.trace.append(tr)
            if n_commit > 0:
                toks = win[:n_commit]
                del win[:n_commit]
                del win_pos[:n_commit]
                eos_at = next((i for i, t in enumerate(toks) if t == self.eos), None)
                to_add = toks if eos_at is None else toks[:eos_at + 1]
                out.extend(to_add)
                stats.tokens_generated += len(to_add)
                committed_len += len(to_add)
                if eos_at is not None:
                    break
                for _ in range(n_commit):
                    if len(out) + len(win) >= max_new_tokens:
                        break
                    win.append(self.mask)
                    win_pos.append(next_pos)
                    next_pos += 1
            if num_mask == 0:
                continue
            mlog = np.asarray(logits)[num_filled:num_filled + num_mask]
            H, probs = compute_entropies_with_probs(mlog, params.temperature)
            running = update_running_entropy(running, H)
            eff = effective_cap(running, params.entropy_threshold, params.max_tokens_per_step)
            sel = select_by_entropy_with_distance(H, mask_logical, params.entropy_threshold,
                                                  params.distance_penalty, eff)
            toks = self._sample(probs, sel, params, stats.steps, mlog)
            tr.entropies, tr.effective_max, tr.selected, tr.sampled = list(H), eff, sel, toks
            for i, s in enumerate(sel):
                post = max(mask_logical[s] - n_commit, 0)
                if post < len(win):
                    win[post] = toks[i]
                    e = float(H[s])
                    stats.avg_entropy += e
                    stats.max_entropy = max(stats.max_entropy, e)
                    if e > ENTROPY_SOFT_THRESHOLD:
                        stats.high_entropy_count += 1
        if stats.tokens_generated > 0:
            stats.avg_entropy /= stats.tokens_generated
            stats.avg_confidence = max(1.0 - stats.avg_entropy / 10.0, 0.0)
        return prompt + out, stats

    # -- block mode --------------------------------------------------------------
    def generate_block(self, prefix_ids: Sequence[int], block_size: int, params: SamplingParams):
        """``generate_block`` (``wedlm.rs:106-259``): re-forwards the block against the
        fixed prefix cache each step; the block K/V are discarded."""
        prefix = [int(t) for t in prefix_ids]
        P = len(prefix)
        stats = BlockStats(prefix_cached=True)
        if self.cache is None or self.cache_len != P:
            self.cache = self.model.prefill_cache(prefix)
            self.cache_len = P
        block = [self.mask] * block_size
        mask_pos = list(range(block_size))
        while mask_pos:
            stats.steps += 1
            ro = compute_block_reorder(block, mask_pos, P)
            logits, _ = self.model.forward_with_positions(ro.reordered_block, ro.positions, self.cache)
            nf, nm = ro.num_filled, len(mask_pos)
            mlog = np.asarray(logits)[nf:nf + nm]
            H, probs = compute_entropies_with_probs(mlog, params.temperature)
            orig = [ro.block_permutation[i] for i in range(nf, block_size)]
            sel = select_by_entropy_with_distance(H, orig, params.entropy_threshold,
                                                  params.distance_penalty, params.max_tokens_per_step)
            if not sel:
                break
            toks = self._sample(probs, sel, params, stats.steps, mlog)
            fill = []
            for i, s in enumerate(sel):
                fill.append((ro.block_permutation[nf + s], toks[i]))
                e = float(H[s])
                stats.avg_entropy += e
                stats.max_entropy = max(stats.max_entropy, e)
                if e > ENTROPY_SOFT_THRESHOLD:
                    stats.high_entropy_count += 1
            stats.tokens_generated += len(fill)
            for p, t in fill:
                block[p] = t
            filled = {p for p, _ in fill}
            mask_pos = [p for p in mask_pos if p not in filled]
            if any(t == self.eos for _, t in fill):
                break
        if stats.tokens_generated > 0:
            stats.avg_entropy /= stats.tokens_generated
            stats.avg_confidence = max(1.0 - stats.avg_entropy / 10.0, 0.0)
        return prefix + block, block, stats

    def commit_block_to_cache(self, block_tokens: Sequence[int]):
        """``commit_block_to_cache`` (``wedlm.rs:268-296``): sequential positions."""
        n = len(block_tokens)
        pos = list(range(self.cache_len, self.cache_len + n))
        _, self.cache = self.model.forward_with_positions(list(block_tokens), pos, self.cache)
        self.cache_len += n

    def generate_with_stats(self, prompt_ids: Sequence[int], max_new_tokens: int,
                            block_size: int, params: SamplingParams):
        """``generate_with_stats`` (``wedlm.rs:610-705``) with adaptive block size and
        cache refresh (``wedlm.rs:710-714``)."""
        all_ids = [int(t) for t in prompt_ids]
        total = 0
        since_check = 0
        eff_bs = block_size
        cum = BlockStats()
        self.cache, self.cache_len = None, 0
        while total < max_new_tokens:
            cur = min(max_new_tokens - total, eff_bs)
            new_ids, blk, bs = self.generate_block(all_ids, cur, params)
            cum.steps += bs.steps
            cum.tokens_generated += bs.tokens_generated
            cum.high_entropy_count += bs.high_entropy_count
            cum.max_entropy = max(cum.max_entropy, bs.max_entropy)
            if cum.tokens_generated > 0:
                prev = cum.tokens_generated - bs.tokens_generated
                cum.avg_entropy = (cum.avg_entropy * prev + bs.avg_entropy * bs.tokens_generated) / cum.tokens_generated
            if bs.max_entropy > ENTROPY_HARD_THRESHOLD:
                eff_bs = 1
                cum.block_size_reductions += 1
            elif bs.max_entropy > ENTROPY_SOFT_THRESHOLD:
                eff_bs = max(eff_bs // 2, 1)
                cum.block_size_reductions += 1
            elif eff_bs < block_size and bs.avg_entropy < ENTROPY_SOFT_THRESHOLD / 2.0:
                eff_bs = min(eff_bs * 2, block_size)
            all_ids = new_ids
            total += cur
            since_check += 1
            if any(t == self.eos for t in blk):
                break
            self.commit_block_to_cache(blk)
            if self.cache_len > MAX_CACHED_LENGTH:
                self.cache = self.model.prefill_cache(all_ids)
                self.cache_len = len(all_ids)
                cum.cache_refreshes += 1
            if since_check >= CACHE_CHECK_INTERVAL:
                since_check = 0
                if cum.high_entropy_count > CACHE_CHECK_INTERVAL // 2:
                    self.cache = self.model.prefill_cache(all_ids)
                    self.cache_len = len(all_ids)
                    cum.cache_refreshes += 1
                    cum.high_entropy_count = 0
        cum.avg_confidence = max(1.0 - cum.avg_entropy / 10.0, 0.0)
        cum.prefix_cached = True
        return all_ids, cum
