"""Speculative-decoding control flow restated (oracle; test infrastructure only).

Reference: tree_utils.py (generate_tree_buffers :72-175,
evaluate_posterior_greedy :182-214, build_tree_attention_mask :501-552) and
speculative_decoding.py (greedy branch of speculative_decode :240-398,
autoregressive_generate :401-451).  Models are duck-typed callables working
on Python lists / numpy arrays.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Sequence

import numpy as np


def generate_tree_buffers(tree_choices: Sequence[Sequence[int]]) -> Dict:
    """tree_utils.py:72-175 (numpy)."""
    sc = sorted([list(c) for c in tree_choices], key=lambda x: (len(x), x))
    T = len(sc) + 1
    depth_counts: List[int] = []
    prev = 0
    for path in sc:
        if len(path) != prev:
            depth_counts.append(0)
        depth_counts[len(path) - 1] += 1
        prev = len(path)
    mask = np.eye(T)
    mask[:, 0] = 1
    start = 0
    for i, cnt in enumerate(depth_counts):
        for j in range(cnt):
            cur = sc[start + j]
            if len(cur) == 1:
                continue
            anc = [sc.index(cur[: c + 1]) + 1 for c in range(len(cur) - 1)]
            mask[j + start + 1, anc] = 1
        start += cnt
    pos = np.zeros(T, dtype=np.int64)
    start = 0
    for i, cnt in enumerate(depth_counts):
        pos[start + 1: start + cnt + 1] = i + 1
        start += cnt
    nest, seen = [], []
    for i in range(len(sc)):
        cur = sc[-i - 1]
        if cur in seen:
            continue
        ri = []
        for c in range(len(cur)):
            ri.append(sc.index(cur[: c + 1]))
            seen.append(cur[: c + 1])
        nest.append(ri)
    ml = max(len(x) for x in nest)
    ri = np.array([x + [-2] * (ml - len(x)) for x in nest], dtype=np.int64) + 1
    ri = np.concatenate([np.zeros((ri.shape[0], 1), np.int64), ri], axis=1)
    big = ri.max() + 5
    order = sorted(ri.tolist(), key=lambda r: [v if v >= 0 else big for v in r])
    return {
        "tree_attn_mask": mask[None, None],
        "tree_position_ids": pos,
        "retrieve_indices": np.array(order, dtype=np.int64),
        "sorted_tree_choices": sc,
        "tree_len": T,
        "depth_counts": depth_counts,
    }


def evaluate_posterior_greedy(logits: np.ndarray, candidates: np.ndarray):
    """tree_utils.py:182-214: longest prefix where cand[:, i+1] == argmax(logits[:, i])."""
    post = (candidates[:, 1:] == np.argmax(logits[:, :-1], axis=-1)).astype(np.int64)
    acc = np.cumprod(post, axis=1).sum(axis=1)
    al = int(acc.max())
    best = 0 if al == 0 else int(np.argmax(acc))
    return best, al, logits[best, al]


def build_tree_attention_mask(prefix_len: int, tree_attn_mask: np.ndarray) -> np.ndarray:
    """tree_utils.py:501-552 with a -inf stand-in for finfo.min (boolean form:
    True = may attend)."""
    T = tree_attn_mask.shape[-1]
    tot = prefix_len + T
    allow = np.zeros((tot, tot), dtype=bool)
    allow[:prefix_len, :prefix_len] = np.tril(np.ones((prefix_len, prefix_len), dtype=bool))
    allow[prefix_len:, :prefix_len] = True
    allow[prefix_len:, prefix_len:] = tree_attn_mask[0, 0].astype(bool)
    return allow


def speculative_decode_greedy(draft_gen: Callable, target_fwd: Callable, input_ids: List[int],
                              max_new_tokens: int, draft_length: int, eos_token_id: int):
    """Greedy branch of speculative_decode (speculative_decoding.py:282-380).
    draft_gen(ids, k) -> list of k draft tokens; target_fwd(ids) -> logits [len(ids), V]."""
    gen: List[int] = []
    total_draft = total_acc = steps = 0
    cur = list(input_ids)
    while len(gen) < max_new_tokens:
        steps += 1
        k = min(draft_length, max_new_tokens - len(gen))
        draft = draft_gen(cur, k)
        logits = target_fwd(cur + list(draft))
        L = len(cur)
        acc = 0
        for i in range(k):
            t = int(np.argmax(logits[L - 1 + i]))
            if t == draft[i]:
                acc += 1
                gen.append(draft[i])
                if draft[i] == eos_token_id:
                    break
            else:
                gen.append(t)
                break
        if acc == k and len(gen) < max_new_tokens:
            gen.append(int(np.argmax(logits[L + k - 1])))
        total_draft += k
        total_acc += acc
        cur = list(input_ids) + gen
        if gen[-1] == eos_token_id:
            break
    stats = {
        "total_tokens_generated": len(gen),
        "total_draft_tokens": total_draft,
        "total_accepted_tokens": total_acc,
        "num_steps": steps,
        "mean_acceptance_length": total_acc / max(steps, 1),
        "acceptance_rate": total_acc / max(total_draft, 1),
    }
    return list(input_ids) + gen, stats


def autoregressive_greedy(target_fwd: Callable, input_ids: List[int], max_new_tokens: int,
                          eos_token_id: int):
    """speculative_decoding.py:401-451 (greedy)."""
    cur = list(input_ids)
    for _ in range(max_new_tokens):
        t = int(np.argmax(target_fwd(cur)[-1]))
        cur.append(t)
        if t == eos_token_id:
            break
    return cur
