"""Tree speculative decoding utilities (drop-in for the reference tree_utils.py).

Same public functions and return structures: ``TREE_PRESETS`` (tree_utils.py:
26-60), ``generate_tree_buffers`` (:72-175), ``evaluate_posterior_greedy``
(:182-214), ``evaluate_posterior_sampling`` (:217-282), ``evaluate_posterior``
(:285-306), ``generate_draft_tree`` (:313-494) and
``build_tree_attention_mask`` (:501-552).  Additions for the B200 path:
``tree_bitmasks`` turns a tree attention mask into the per-node ancestor
bitmasks the attention kernel takes, and ``binary_tree_choices`` builds the
depth-d / branching-b tree of the benchmark configuration.
"""
from __future__ import annotations

import random
from itertools import product
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

# The preset trees must be the reference's (they come from EAGLE's mc_sim
# choices) so that a caller selecting a preset gets the same tree here.
TREE_CHOICES_DEFAULT = [
    [0], [1], [2], [3],
    [0, 0], [0, 1], [0, 2], [1, 0], [1, 1], [2, 0], [2, 1], [3, 0],
    [0, 0, 0], [0, 0, 1], [0, 0, 2], [0, 1, 0], [0, 1, 1], [0, 2, 0], [0, 2, 1], [1, 0, 0],
    [0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 0, 2],
    [0, 0, 0, 0, 0], [0, 0, 0, 0, 1],
]
TREE_CHOICES_SMALL = [
    [0], [1], [2],
    [0, 0], [0, 1], [1, 0],
    [0, 0, 0], [0, 0, 1],
    [0, 0, 0, 0],
]
TREE_CHOICES_LARGE = [
    [0], [1], [2], [3], [4],
    [0, 0], [0, 1], [0, 2], [0, 3], [1, 0], [1, 1], [1, 2], [2, 0], [2, 1], [3, 0], [3, 1], [4, 0],
    [0, 0, 0], [0, 0, 1], [0, 0, 2], [0, 1, 0], [0, 1, 1], [0, 2, 0], [1, 0, 0], [1, 0, 1], [1, 1, 0], [2, 0, 0],
    [0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 0, 2], [0, 0, 1, 0], [0, 1, 0, 0], [1, 0, 0, 0],
    [0, 0, 0, 0, 0], [0, 0, 0, 0, 1],
]
TREE_PRESETS = {"default": TREE_CHOICES_DEFAULT, "small": TREE_CHOICES_SMALL, "large": TREE_CHOICES_LARGE}


def binary_tree_choices(depth: int = 4, branch: int = 2) -> List[List[int]]:
    """Every index path of length 1..depth with indices < branch (2+4+8+16 = 30
    nodes for the depth-4 / branching-2 tree)."""
    return [list(p) for d in range(1, depth + 1) for p in product(range(branch), repeat=d)]


def pad_path(path: List[int], length: int, pad_value: int = -2) -> List[int]:
    return path + [pad_value] * (length - len(path))


def generate_tree_buffers(tree_choices, device="cuda") -> Dict:
    """Tree attention mask [1,1,T,T], depth position ids [T], retrieve indices
    [leaves, D+1] (tree_utils.py:72-175)."""
    sc = sorted([list(c) for c in tree_choices], key=lambda c: (len(c), c))
    T = len(sc) + 1
    index = {tuple(c): i + 1 for i, c in enumerate(sc)}  # node index of each path (root = 0)
    depth_counts: List[int] = []
    for c in sc:
        while len(depth_counts) < len(c):
            depth_counts.append(0)
        depth_counts[len(c) - 1] += 1
    mask = torch.eye(T, T)
    mask[:, 0] = 1
    pos = torch.zeros(T, dtype=torch.long)
    for c in sc:
        i = index[tuple(c)]
        for d in range(1, len(c)):
            mask[i, index[tuple(c[:d])]] = 1
        pos[i] = len(c)
    # one retrieval row per maximal path, scanning from the deepest node backwards
    rows, covered = [], set()
    for c in reversed(sc):
        if tuple(c) in covered:
            continue
        rows.append([index[tuple(c[:d + 1])] - 1 for d in range(len(c))])
        covered.update(tuple(c[:d + 1]) for d in range(len(c)))
    width = max(len(r) for r in rows)
    ri = torch.tensor([pad_path(r, width) for r in rows], dtype=torch.long) + 1
    ri = torch.cat([torch.zeros(ri.shape[0], 1, dtype=torch.long), ri], dim=1)
    big = int(ri.max()) + 5
    ri = torch.tensor(sorted(ri.tolist(), key=lambda r: [v if v >= 0 else big for v in r]), dtype=torch.long)
    buf = {
        "tree_attn_mask": mask[None, None],
        "tree_position_ids": pos,
        "retrieve_indices": ri,
        "sorted_tree_choices": sc,
        "tree_len": T,
        "depth_counts": depth_counts,
    }
    return {k: (v.clone().to(device) if isinstance(v, torch.Tensor) else v) for k, v in buf.items()}


def tree_bitmasks(tree_attn_mask: torch.Tensor) -> torch.Tensor:
    """[1,1,T,T] 0/1 mask -> int64 [T]: bit j of entry i set when node i sees node j
    (T <= 64), the form the attention kernel takes."""
    m = tree_attn_mask.reshape(tree_attn_mask.shape[-2], tree_attn_mask.shape[-1]).bool().cpu()
    T = m.shape[0]
    if T > 64:
        raise ValueError("tree masks of more than 64 nodes are not supported")
    out = []
    for i in range(T):
        v = 0
        for j in range(T):
            if m[i, j]:
                v |= 1 << j
        out.append(v - (1 << 64) if v >= (1 << 63) else v)
    return torch.tensor(out, dtype=torch.int64)


def evaluate_posterior_greedy(logits: torch.Tensor, candidates: torch.Tensor):
    """Longest candidate prefix matching the target's argmax (tree_utils.py:182-214)."""
    match = (candidates[:, 1:].to(logits.device) == torch.argmax(logits[:, :-1], dim=-1)).int()
    lengths = torch.cumprod(match, dim=1).sum(dim=1)
    accept = lengths.max()
    if accept == 0:
        best = torch.tensor(0, dtype=torch.long, device=candidates.device)
    else:
        best = torch.argmax(lengths).to(torch.long)
    return best, accept.item(), logits[best, accept]


def evaluate_posterior_sampling(logits: torch.Tensor, candidates: torch.Tensor, temperature: float = 1.0):
    """Rejection sampling over candidate paths (tree_utils.py:217-282)."""
    accept_length = 1
    accept_cand = candidates[0][:1]
    best_candidate = 0
    adjustflag = False
    gtp = None
    for i in range(1, candidates.shape[1]):
        if i != accept_length:
            break
        adjustflag = False
        is_eq = (candidates[:, :accept_length] == accept_cand).all(dim=1)
        fi = torch.nonzero(is_eq, as_tuple=True)[0][0]
        gt_logits = logits[fi, i - 1][None]
        if temperature > 1e-5:
            gt_logits = gt_logits / temperature
        gtp = torch.softmax(gt_logits[0], dim=0)
        seen = []
        for j in range(candidates.shape[0]):
            if not is_eq[j]:
                continue
            x = candidates[j, i]
            xi = x.item()
            if xi in seen or xi == -1:
                continue
            seen.append(xi)
            r = random.random()
            if r <= gtp[xi] / 1.0:  # uniform draft proposal, as in the reference
                accept_cand = torch.cat((accept_cand, x[None]), dim=0)
                accept_length += 1
                best_candidate = j
                break
            gtp[xi] = 0
            gtp = gtp / (gtp.sum() + 1e-10)
            adjustflag = True
    if adjustflag and accept_length != candidates.shape[1]:
        sample_p = gtp
    else:
        gt_logits = logits[best_candidate, accept_length - 1][None]
        if temperature > 1e-5:
            gt_logits = gt_logits / temperature
        sample_p = torch.softmax(gt_logits[0], dim=0)
    return torch.tensor(best_candidate), accept_length - 1, sample_p


def evaluate_posterior(logits, candidates, greedy: bool = True, temperature: float = 1.0):
    if greedy:
        return evaluate_posterior_greedy(logits, candidates)
    return evaluate_posterior_sampling(logits, candidates, temperature)


@torch.no_grad()
def generate_draft_tree(draft_model, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor],
                        tree_buffers: Dict, top_k: int = 10, temperature: float = 1.0) -> torch.Tensor:
    """Tree of draft candidates (tree_utils.py:313-494): the root's top-k fill depth
    1; every node that has children in the tree is expanded by one draft forward
    and its top-k become the children's tokens.  Returns (1, tree_len) token ids.

    A draft model exposing ``expand_tree`` (the CUDA draft model) expands a whole
    depth level in one tree-masked forward; any other model is called once per
    expanded node on the full prefix, as the reference does."""
    if hasattr(draft_model, "expand_tree"):
        return draft_model.expand_tree(input_ids, tree_buffers, top_k=top_k, temperature=temperature)
    sc = tree_buffers["sorted_tree_choices"]
    T = tree_buffers["tree_len"]
    device = input_ids.device
    out = draft_model.forward(input_ids=input_ids, attention_mask=attention_mask, use_cache=True)
    root = out.logits[:, -1, :]
    scaled = root / temperature if temperature > 1e-5 else root
    vals, ids = torch.topk(F.log_softmax(scaled, dim=-1), top_k, dim=-1)
    tokens: Dict[Tuple[int, ...], int] = {(k,): int(ids[0, k]) for k in range(top_k)}
    parents = {tuple(c[:-1]) for c in sc if len(c) > 1}
    for depth in range(1, max(len(c) for c in sc)):
        for c in sc:
            path = tuple(c)
            if len(path) != depth or path not in parents or path not in tokens:
                continue
            seq = [tokens[path[:d + 1]] for d in range(depth)]
            full = torch.cat([input_ids, torch.tensor([seq], device=device, dtype=torch.long)], dim=1)
            mask = torch.ones_like(full) if attention_mask is not None else None
            lg = draft_model.forward(input_ids=full, attention_mask=mask, use_cache=False).logits[:, -1, :]
            sc_lg = lg / temperature if temperature > 1e-5 else lg
            _, cids = torch.topk(F.log_softmax(sc_lg, dim=-1), top_k, dim=-1)
            for k in range(top_k):
                tokens[path + (k,)] = int(cids[0, k])
    cand = torch.zeros(T, dtype=torch.long, device=device)
    cand[0] = input_ids[0, -1]
    for i, c in enumerate(sc):
        if tuple(c) in tokens:
            cand[i + 1] = tokens[tuple(c)]
    return cand.unsqueeze(0)


def build_tree_attention_mask(prefix_len: int, tree_attn_mask: torch.Tensor, device,
                              dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Additive mask [1,1,P+T,P+T] (tree_utils.py:501-552): causal prefix, tree
    nodes see the whole prefix and their ancestors, the prefix sees no node."""
    T = tree_attn_mask.shape[-1]
    tot = prefix_len + T
    neg = torch.finfo(dtype).min
    full = torch.zeros(1, 1, tot, tot, device=device, dtype=dtype)
    full[0, 0, :prefix_len, :prefix_len] = torch.triu(
        torch.ones(prefix_len, prefix_len, device=device, dtype=dtype) * neg, diagonal=1)
    tm = tree_attn_mask[0, 0].to(device).bool()
    full[0, 0, prefix_len:, prefix_len:] = torch.where(
        tm, torch.zeros((), device=device, dtype=dtype), torch.full((), neg, device=device, dtype=dtype))
    full[0, 0, :prefix_len, prefix_len:] = neg
    return full
