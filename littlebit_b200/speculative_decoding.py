"""Speculative decoding entry points (drop-in for the reference speculative_decoding.py).

``speculative_decode`` (speculative_decoding.py:240-398), ``autoregressive_generate``
(:401-451) and ``speculative_decode_tree`` (:454-617) keep their signatures,
return values and stats keys.  With duck-typed models they run the
reference's control flow.  With the CUDA models of cuda_models.py the greedy
loops run device-resident: the draft tokens are chained on the GPU through
captured graphs, the target verifies all of them in one batched step, and
acceptance happens on the GPU (lbx_accept_greedy_chain / _tree); the host
reads a few integers once per round.

Greedy output is token-identical to target-only greedy decoding because the
target's kernels give every token the same bits whether it is verified alone
or in a batch (integer-exact linear reductions, slot-aligned attention
chunks).

The tree path fixes two defects of the reference loop (mask rows shifted by
one after dropping the root, tree position ids computed but never passed to
the target): the root is verified with the tree, every node attends to the
prefix plus its ancestors at rotary position prefix_len - 1 + depth, and the
accepted path's KV rows are compacted in place.
"""
from __future__ import annotations

import time
from typing import Optional

import torch
import torch.nn.functional as F

from .tree_utils import (  # noqa: F401  (re-exported like the reference module)
    TREE_PRESETS, build_tree_attention_mask, evaluate_posterior, generate_draft_tree,
    generate_tree_buffers,
)


def _is_cuda_pair(draft, target) -> bool:
    from .cuda_models import CudaDraftModel, CudaTargetModel

    return isinstance(draft, CudaDraftModel) and isinstance(target, CudaTargetModel)


def _stats(gen, total_draft, total_acc, steps, elapsed, draft_length, extra=None):
    st = {
        "total_tokens_generated": len(gen),
        "total_draft_tokens": total_draft,
        "total_accepted_tokens": total_acc,
        "num_steps": steps,
        "mean_acceptance_length": total_acc / max(steps, 1),
        "acceptance_rate": total_acc / max(total_draft, 1),
        "tokens_per_second": len(gen) / max(elapsed, 1e-6),
        "elapsed_seconds": elapsed,
        "draft_length_k": draft_length,
    }
    if extra:
        st.update(extra)
    return st


def speculative_decode(draft_model, target_model, input_ids: torch.Tensor,
                       attention_mask: Optional[torch.Tensor], max_new_tokens: int = 256,
                       draft_length: int = 5, temperature: float = 1.0, greedy: bool = True,
                       eos_token_id: int = 2, verbose: bool = False):
    """Draft ``draft_length`` tokens, verify with the target, accept the longest
    matching prefix plus one target token (greedy) or rejection-sample (sampling)."""
    if _is_cuda_pair(draft_model, target_model):
        if greedy:
            return _speculative_decode_cuda(draft_model, target_model, input_ids, max_new_tokens,
                                            draft_length, eos_token_id, verbose)
        return _speculative_decode_cuda_sampling(draft_model, target_model, input_ids, max_new_tokens,
                                                 draft_length, temperature, eos_token_id, verbose)
    device = input_ids.device
    gen = []
    total_draft = total_acc = steps = 0
    cur_ids, cur_mask = input_ids, attention_mask
    t0 = time.time()
    while len(gen) < max_new_tokens:
        steps += 1
        k = min(draft_length, max_new_tokens - len(gen))
        dtoks, dprobs = draft_model.generate_draft_tokens(input_ids=cur_ids, attention_mask=cur_mask,
                                                          draft_length=k, temperature=temperature,
                                                          greedy=greedy)
        ids = torch.cat(dtoks, dim=1).to(device)
        verify_ids = torch.cat([cur_ids, ids], dim=1)
        vmask = None if cur_mask is None else torch.cat(
            [cur_mask, torch.ones(1, k, device=device, dtype=cur_mask.dtype)], dim=1)
        logits = target_model.forward(verify_ids, vmask)
        L = cur_ids.shape[1]
        acc = 0
        for i in range(k):
            tl = logits[:, L - 1 + i, :]
            d = int(dtoks[i])
            if greedy:
                t = int(torch.argmax(tl, dim=-1))
                if t == d:
                    acc += 1
                    gen.append(d)
                    if d == eos_token_id:
                        break
                else:
                    gen.append(t)
                    break
            else:
                tp = F.softmax(tl / max(temperature, 1e-8), dim=-1)
                dp = dprobs[i].to(device)
                pt, pd = tp[0, d].item(), dp[0, d].item()
                if torch.rand(1).item() < min(1.0, pt / max(pd, 1e-10)):
                    acc += 1
                    gen.append(d)
                    if d == eos_token_id:
                        break
                else:
                    resid = torch.clamp(tp - dp, min=0)
                    resid = resid / (resid.sum() + 1e-10)
                    gen.append(int(torch.multinomial(resid, num_samples=1)))
                    break
        if acc == k and len(gen) < max_new_tokens:
            bl = logits[:, L + k - 1, :]
            if greedy:
                gen.append(int(torch.argmax(bl, dim=-1)))
            else:
                gen.append(int(torch.multinomial(F.softmax(bl / max(temperature, 1e-8), dim=-1), 1)))
        total_draft += k
        total_acc += acc
        cur_ids = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=torch.long)], dim=1)
        if attention_mask is not None:
            cur_mask = torch.ones_like(cur_ids)
        if gen[-1] == eos_token_id:
            break
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    return out, _stats(gen, total_draft, total_acc, steps, el, draft_length)


def autoregressive_generate(target_model, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor],
                            max_new_tokens: int = 256, temperature: float = 1.0, greedy: bool = True,
                            eos_token_id: int = 2):
    """Target-only generation (the token-identity reference for greedy speculation)."""
    from .cuda_models import CudaTargetModel

    if greedy and isinstance(target_model, CudaTargetModel):
        return _autoregressive_cuda(target_model, input_ids, max_new_tokens, eos_token_id)
    device = input_ids.device
    gen = []
    cur_ids, cur_mask = input_ids, attention_mask
    t0 = time.time()
    for _ in range(max_new_tokens):
        lg = target_model.forward(cur_ids, cur_mask)[:, -1, :]
        if greedy:
            t = int(torch.argmax(lg, dim=-1))
        else:
            t = int(torch.multinomial(F.softmax(lg / max(temperature, 1e-8), dim=-1), 1))
        gen.append(t)
        cur_ids = torch.cat([cur_ids, torch.tensor([[t]], device=device)], dim=1)
        if cur_mask is not None:
            cur_mask = torch.cat([cur_mask, torch.ones(1, 1, device=device, dtype=cur_mask.dtype)], dim=1)
        if t == eos_token_id:
            break
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    return out, {"total_tokens_generated": len(gen), "tokens_per_second": len(gen) / max(el, 1e-6),
                 "elapsed_seconds": el}


# ---------------------------------------------------------------------------
# device-resident greedy loops
# ---------------------------------------------------------------------------
def _speculative_decode_cuda(draft, target, input_ids, max_new_tokens, draft_length, eos, verbose):
    ids = input_ids[0].tolist()
    device = input_ids.device
    dev = draft.device
    draft.reset()
    target.reset_cache()
    t0 = time.time()
    P = len(ids) - 1            # slot of the round's first (seed) token
    draft._sync_prefix(ids, P)  # both caches hold the prompt except its last token
    target.prefill_ids(ids, P)
    tok = draft.tok_buf
    tok[0:1].fill_(ids[-1])
    pending = None              # a fully accepted last draft the draft cache has not seen
    gen = []
    total_draft = total_acc = steps = 0
    acc_out = torch.empty(2, dtype=torch.int64, device=dev)
    host = torch.empty(2 + 64, dtype=torch.int64).pin_memory()
    while len(gen) < max_new_tokens:
        steps += 1
        k = min(draft_length, max_new_tokens - len(gen))
        if pending is not None:  # feed it to the draft (its KV), slot P-1
            draft.dec.step(pending, P - 1)
            pending = None
        draft.draft_on_device(P, k)
        am = target.verify_on_device(tok, P, k + 1)
        out = accept_chain(tok[1:k + 1], am, acc_out)
        host[:2].copy_(out, non_blocking=True)
        host[2:2 + k].copy_(tok[1:k + 1], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        a, nxt = int(host[0]), int(host[1])
        drafts = host[2:2 + k].tolist()
        # the reference's acceptance walk, replayed from (a, next)
        acc = 0
        for i in range(k):
            if i < a:
                acc += 1
                gen.append(drafts[i])
                if drafts[i] == eos:
                    break
            else:
                gen.append(nxt)
                break
        if acc == k and len(gen) < max_new_tokens:
            gen.append(nxt)
        total_draft += k
        total_acc += acc
        if verbose:
            print(f"step {steps}: drafted {k}, accepted {acc}, generated {len(gen)}")
        if gen[-1] == eos:
            break
        # caches: the target holds slots P..P+k (seed + drafts), valid through P+acc;
        # the draft holds slots P..P+k-1 (seed + d1..d_{k-1}), so a fully accepted
        # round leaves d_k for it to absorb before the next seed
        if acc == k:
            pending = tok[k:k + 1].clone()
        P = P + acc + 1
        tok[0:1].fill_(gen[-1])
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    return out, _stats(gen, total_draft, total_acc, steps, el, draft_length)


def _speculative_decode_cuda_sampling(draft, target, input_ids, max_new_tokens, draft_length, temperature, eos,
                                      verbose, generator: Optional[torch.Generator] = None):
    """Sampling-mode chain speculation with the drafting, the verification and
    the acceptance test on the device; the host reads the round's outcome once.

    Per round (speculative_decoding.py:331-363): the draft samples k tokens
    d_i ~ q_i = softmax(draft logits / T); the target gives p_i for the seed
    and the drafts in one batched step; draft i is accepted while
    u_i < min(1, p_i(d_i) / q_i(d_i)) (u_i uniform); at the first rejection a
    token is drawn from norm(max(p_a - q_a, 0)), and after k acceptances a
    bonus token from p_k."""
    ids = input_ids[0].tolist()
    device = input_ids.device
    dev = draft.device
    V = draft._vocab_size
    Tm = max(float(temperature), 1e-8)
    draft.reset()
    target.reset_cache()
    t0 = time.time()
    P = len(ids) - 1
    draft._sync_prefix(ids, P)
    target.prefill_ids(ids, P)
    K = draft_length
    tok = torch.empty(K + 1, dtype=torch.int64, device=dev)
    dlog = torch.empty(K, V, dtype=torch.float32, device=dev)
    tlog = torch.empty(K + 1, V, dtype=torch.float32, device=dev)
    host = torch.empty(2 + K, dtype=torch.int64).pin_memory()
    pending = None
    gen = []
    total_draft = total_acc = steps = 0
    tok[0] = ids[-1]
    while len(gen) < max_new_tokens:
        steps += 1
        k = min(K, max_new_tokens - len(gen))
        if pending is not None:
            draft.dec.step(pending, P - 1)
            pending = None
        for i in range(k):  # sample the drafts on the device
            draft.dec.step(tok[i:i + 1], P + i, logits=dlog[i:i + 1])
            q = F.softmax(dlog[i] / Tm, dim=-1)
            tok[i + 1:i + 2] = torch.multinomial(q, 1, generator=generator)
        target._step(tok[:k + 1], P, logits=tlog[:k + 1])
        pr = F.softmax(tlog[:k + 1] / Tm, dim=-1)
        qd = F.softmax(dlog[:k] / Tm, dim=-1)
        d = tok[1:k + 1]
        pt = pr[:k].gather(1, d[:, None])[:, 0]
        pq = qd.gather(1, d[:, None])[:, 0]
        u = torch.rand(k, device=dev, generator=generator)
        ok = (u < torch.clamp(pt / pq.clamp_min(1e-10), max=1.0)).to(torch.int64)
        a = torch.cumprod(ok, 0).sum()
        # the token after the accepted drafts: residual sample at a rejection,
        # bonus from p_k after k acceptances
        ai = a.clamp(max=k - 1)
        resid = torch.clamp(pr[ai] - qd[ai], min=0)
        resid = resid / (resid.sum() + 1e-10)
        dist = torch.where(a < k, resid, pr[k])
        nxt = torch.multinomial(dist, 1, generator=generator)[0]
        host[0:1].copy_(a.view(1), non_blocking=True)
        host[1:2].copy_(nxt.view(1), non_blocking=True)
        host[2:2 + k].copy_(d, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        acc_n, nx = int(host[0]), int(host[1])
        drafts = host[2:2 + k].tolist()
        acc = 0
        for i in range(k):
            if i < acc_n:
                acc += 1
                gen.append(drafts[i])
                if drafts[i] == eos:
                    break
            else:
                gen.append(nx)
                break
        if acc == k and len(gen) < max_new_tokens:
            gen.append(nx)
        total_draft += k
        total_acc += acc
        if verbose:
            print(f"step {steps}: drafted {k}, accepted {acc}, generated {len(gen)}")
        if gen[-1] == eos:
            break
        if acc == k:
            pending = tok[k:k + 1].clone()
        P = P + acc + 1
        tok[0] = gen[-1]
    for u_ in target._units:
        u_.pos = P
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    return out, _stats(gen, total_draft, total_acc, steps, el, draft_length, {"decode_mode": "sampling"})


def accept_chain(draft_toks: torch.Tensor, target_argmax: torch.Tensor, out: torch.Tensor):
    from . import _lib as L
    from .ops import _p, _stream, lib

    L.check(lib().lbx_accept_greedy_chain(_p(draft_toks), _p(target_argmax), draft_toks.numel(),
                                          _p(out), _stream(out.device)), "accept_greedy_chain")
    return out


def _autoregressive_cuda(target, input_ids, max_new_tokens, eos, sync_every: int = 16):
    ids = input_ids[0].tolist()
    device = input_ids.device
    dev = target.device
    target.reset_cache()
    t0 = time.time()
    P = len(ids) - 1
    target.prefill_ids(ids, P)
    hist = torch.zeros(max_new_tokens + 1, dtype=torch.int64, device=dev)
    hist[0] = ids[-1]
    gen = []
    done = 0
    while done < max_new_tokens:
        m = min(sync_every, max_new_tokens - done)
        for i in range(m):
            am = target.verify_on_device(hist[done + i:done + i + 1], P + done + i, 1)
            hist[done + i + 1:done + i + 2].copy_(am)
        done += m
        new = hist[done - m + 1:done + 1].tolist()
        stop = False
        for t in new:
            gen.append(t)
            if t == eos:
                stop = True
                break
        if stop:
            break
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    return out, {"total_tokens_generated": len(gen), "tokens_per_second": len(gen) / max(el, 1e-6),
                 "elapsed_seconds": el}


def speculative_decode_tree(draft_model, target_model, input_ids: torch.Tensor,
                            attention_mask: Optional[torch.Tensor], max_new_tokens: int = 256,
                            tree_buffers: dict = None, top_k: int = 10, temperature: float = 1.0,
                            greedy: bool = True, eos_token_id: int = 2, verbose: bool = False):
    """Tree speculation: draft a token tree, verify every branch in one target
    step with a tree attention mask, accept the longest matching path + bonus."""
    if not _is_cuda_pair(draft_model, target_model):
        raise NotImplementedError(
            "speculative_decode_tree verifies with the CUDA target's tree attention; pass "
            "CudaDraftModel / CudaTargetModel")
    if not greedy:
        raise NotImplementedError("tree speculation here is greedy (evaluate_posterior_greedy)")
    from .ops import accept_greedy_tree

    device = input_ids.device
    dev = target_model.device
    ids = input_ids[0].tolist()
    draft_model.reset()
    target_model.reset_cache()
    t0 = time.time()
    retrieve = tree_buffers["retrieve_indices"].to(dev)
    T = tree_buffers["tree_len"]
    Lr, D1 = retrieve.shape
    gen = []
    total_draft = total_acc = steps = 0
    P = len(ids) - 1
    target_model.prefill_ids(ids, P)
    while len(gen) < max_new_tokens:
        steps += 1
        cur = ids + gen
        cand = draft_model.expand_tree(torch.tensor([cur], device=dev), tree_buffers, top_k=top_k,
                                       temperature=temperature)[0]
        node_am = target_model.verify_tree(cand, P, tree_buffers)
        padded = torch.cat([cand, torch.full((1,), -1, dtype=torch.int64, device=dev)])
        cart = padded[retrieve]  # retrieve uses -1 for padding -> the appended -1
        res_d = accept_greedy_tree(cart.contiguous(), node_am, retrieve.contiguous())
        both = torch.cat([res_d, cand.to(torch.int64)]).tolist()  # one device read: outcome and candidates
        res, cand_h = both[:res_d.numel()], both[res_d.numel():]
        best, alen, bonus = res[0], res[1], res[2]
        nodes = [int(v) for v in res[3:3 + alen]]
        acc_toks = [cand_h[j] for j in nodes]
        stop = False
        for t in acc_toks:
            gen.append(t)
            if t == eos_token_id:
                stop = True
                break
        if not stop and len(gen) < max_new_tokens:
            gen.append(int(bonus))
        total_draft += T - 1
        total_acc += alen
        if verbose:
            print(f"step {steps}: tree {T - 1}, accepted {alen}, generated {len(gen)}")
        if gen[-1] == eos_token_id or len(gen) >= max_new_tokens:
            break
        # compact the accepted path's KV (target) to consecutive slots after the root
        if alen:
            src = torch.tensor([P + j for j in nodes], dtype=torch.int32, device=dev)
            dst = torch.tensor([P + 1 + d for d in range(alen)], dtype=torch.int32, device=dev)
            target_model.kv_move(src, dst)
        P = P + alen + 1
        for u in target_model._units:
            u.pos = P
        target_model._cached_tokens = (ids + gen)[:P]
    el = time.time() - t0
    out = torch.cat([input_ids, torch.tensor([gen], device=device, dtype=input_ids.dtype)], dim=1)
    st = _stats(gen, total_draft, total_acc, steps, el, None, {"decode_mode": "tree", "tree_size": T})
    st.pop("draft_length_k")
    return out, st
