"""Multi-sequence decoding on one GPU: many independent requests per step.

The reference decodes one sequence per process (cpu_draft_model.py,
cpu_target_model.py); batching requests is how a GPU amortises the
packed-weight read of every projection over many tokens.  ``BatchDecoder``
runs S independent sequences through one decoder step per token
(lbx_forward_multi): the linear calls see S (or S x n) tokens, attention keeps
a KV cache per sequence, and every sequence's results are bit-identical to
decoding it alone (the kernels are batch-invariant), so

  * ``greedy_generate`` gives each sequence the tokens of its own
    target-only greedy run (speculative_decoding.py:401-451), and
  * ``speculative_generate`` (chain drafting, greedy acceptance of
    speculative_decoding.py:315-330 and the bonus token of :356-363, per
    sequence, on the device) gives the same tokens again.

Sequences advance in lockstep by steps, not by tokens: after a speculative
step each sequence has accepted its own number of drafts, and its next slot
is kept on the device (start_seq).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _lib as L
from .model import LittleBitDecoder
from .ops import _p, _stream, lib


class BatchDecoder:
    """S sequences over one LittleBitDecoder's weights, with their own KV caches
    ([S, kv_heads, max_seq, head_dim] bf16 per layer)."""

    def __init__(self, dec: LittleBitDecoder, n_seq: int, max_seq: int):
        if not 1 <= n_seq <= 64:
            raise ValueError("1..64 sequences per batch decoder")
        self.dec, self.S, self.max_seq = dec, int(n_seq), int(max_seq)
        s = dec.shape
        dev = dec.device
        self.device = dev
        kvs = (self.S, s.num_key_value_heads, self.max_seq, s.head_dim)
        self.k_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dev) for _ in dec.layers]
        self.v_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dev) for _ in dec.layers]
        self.stride = s.num_key_value_heads * self.max_seq * s.head_dim
        # the decoder's descriptors with this batch's caches and length
        self._layer_arr = (L.Layer * len(dec.layers))()
        for i in range(len(dec.layers)):
            self._layer_arr[i] = dec._layer_arr[i]
            self._layer_arr[i].k_cache = _p(self.k_cache[i])
            self._layer_arr[i].v_cache = _p(self.v_cache[i])
        m = L.Model()
        ctypes.pointer(m)[0] = dec._model
        m.max_seq = self.max_seq
        m.exec_mode = L.LBX_EXEC_KERNELS
        m.layers = ctypes.cast(self._layer_arr, ctypes.POINTER(L.Layer))
        self._model = m
        self._ws = {}

    def workspace(self, n: int) -> torch.Tensor:
        if n not in self._ws:
            need = int(lib().lbx_forward_multi_workspace_size(ctypes.byref(self._model), self.S, n))
            if need == 0:
                raise RuntimeError(f"multi-sequence step of {self.S} x {n} tokens unsupported")
            self._ws[n] = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._ws[n]

    def step(self, tokens: torch.Tensor, start_seq: torch.Tensor, max_start: int, n: int, *,
             argmax: Optional[torch.Tensor] = None, logits: Optional[torch.Tensor] = None) -> None:
        """n tokens of every sequence (device int64 [S*n], sequence by sequence) at
        slots start_seq[s] .. start_seq[s]+n-1 (device int32 [S]; max_start bounds them)."""
        if max_start + n > self.max_seq:
            raise RuntimeError(f"KV cache full: {max_start}+{n} > {self.max_seq}")
        ws = self.workspace(n)
        L.check(lib().lbx_forward_multi(ctypes.byref(self._model), _p(tokens), self.S, n, int(max_start),
                                        _p(start_seq), self.stride, None, None, None, _p(logits), _p(argmax),
                                        _p(ws), ws.numel(), _stream(self.device)), "lbx_forward_multi")

    def fill_synthetic_prefix(self, n_slots: int, seed: int, scale: float = 1.0) -> None:
        """Seeded random bf16 keys and values in slots [0, n_slots) of every
        sequence (a stand-in for a prompt prefill; the attention work per new
        token depends only on the cached length)."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        for kc, vc in zip(self.k_cache, self.v_cache):
            for c in (kc, vc):
                c[:, :, :n_slots].copy_((scale * torch.randn(c[:, :, :n_slots].shape, generator=g,
                                                             device=self.device)).bfloat16())

    def copy_prefix_from(self, other: "BatchDecoder", n_slots: int) -> None:
        for a, b in zip(self.k_cache + self.v_cache, other.k_cache + other.v_cache):
            a[:, :, :n_slots].copy_(b[:, :, :n_slots])


def greedy_generate(tgt: BatchDecoder, last: torch.Tensor, start: int, max_new: int) -> torch.Tensor:
    """Target-only greedy decoding of S sequences whose caches hold slots
    [0, start) and whose next input token is last[s] (device int64 [S]).
    Returns the new tokens, device int64 [S, max_new]."""
    S, dev = tgt.S, tgt.device
    out = torch.empty(S, max_new, dtype=torch.int64, device=dev)
    tok = last.clone()
    st = torch.full((S,), start, dtype=torch.int32, device=dev)
    am = torch.empty(S, dtype=torch.int64, device=dev)
    for i in range(max_new):
        tgt.step(tok, st, start + i, 1, argmax=am)
        out[:, i] = am
        tok.copy_(am)
        st += 1
    return out


def speculative_generate(drf: BatchDecoder, tgt: BatchDecoder, prev: torch.Tensor, last: torch.Tensor,
                         start: int, max_new: int, gamma: int = 4):
    """Chain speculative decoding of S sequences in lockstep.

    Both models' caches hold slots [0, start) of every sequence; prev[s] is
    the token at slot start-1 and last[s] the next input token.  Each step:
    the draft re-feeds the previous token with the last one (a sequence whose
    drafts were all accepted has not fed its last draft; re-writing a slot
    with the same token writes the same bits) and greedy-drafts gamma tokens;
    the target verifies last + drafts (gamma + 1 tokens per sequence);
    acceptance and the bonus token are computed per sequence on the device.
    Returns (new tokens [S, max_new], stats)."""
    S, dev = tgt.S, tgt.device
    cap = max_new + gamma + 1
    out = torch.zeros(S, cap, dtype=torch.int64, device=dev)
    nacc = torch.zeros(S, dtype=torch.int64, device=dev)   # new tokens so far
    pos = torch.full((S,), start, dtype=torch.int32, device=dev)  # slot of `last`
    prev_t, last_t = prev.clone(), last.clone()
    ar = torch.arange(gamma + 1, device=dev)
    drafts = torch.empty(S, gamma + 1, dtype=torch.int64, device=dev)
    vtok = torch.empty(S, gamma + 1, dtype=torch.int64, device=dev)
    am = torch.empty(S * (gamma + 1), dtype=torch.int64, device=dev)
    two = torch.empty(S, 2, dtype=torch.int64, device=dev)
    am2 = torch.empty(S * 2, dtype=torch.int64, device=dev)
    dam = torch.empty(S, dtype=torch.int64, device=dev)
    steps, total_acc = 0, 0
    bound = start
    done = 0
    while done < max_new:
        # draft: [prev, last] at slots pos-1, pos, then gamma-1 single tokens
        two[:, 0], two[:, 1] = prev_t, last_t
        drf.step(two.reshape(-1), pos - 1, bound - 1, 2, argmax=am2)
        drafts[:, 0] = am2.view(S, 2)[:, 1]
        for i in range(1, gamma):
            drf.step(drafts[:, i - 1].contiguous(), pos + i, bound + i, 1, argmax=dam)
            drafts[:, i] = dam
        # verify: last + gamma drafts at slots pos .. pos+gamma
        vtok[:, 0] = last_t
        vtok[:, 1:] = drafts[:, :gamma]
        tgt.step(vtok.reshape(-1), pos, bound, gamma + 1, argmax=am)
        a = am.view(S, gamma + 1)
        match = (vtok[:, 1:] == a[:, :gamma]).to(torch.int64)
        m = torch.cumprod(match, dim=1).sum(dim=1)            # accepted drafts per sequence
        bonus = a.gather(1, m[:, None])[:, 0]
        # this step's tokens: the m accepted drafts, then the bonus; positions
        # past them are rewritten by later steps (or lie past max_new)
        cand = torch.cat([vtok[:, 1:], torch.zeros_like(vtok[:, :1])], dim=1)
        new = torch.where(ar[None, :] < m[:, None], cand, bonus[:, None])
        out.scatter_(1, (nacc[:, None] + ar[None, :]).clamp(max=cap - 1), new)
        # the new last token is the bonus; the token before it sits at slot pos + m
        prev_t = vtok.gather(1, m[:, None])[:, 0]
        last_t = bonus
        nacc += m + 1
        pos += (m + 1).to(torch.int32)
        steps += 1
        total_acc += int(m.sum())
        done = int(nacc.min())
        bound = start + int(nacc.max())
    stats = {"num_steps": steps, "total_accepted_tokens": total_acc,
             "acceptance_rate": total_acc / (steps * gamma * S),
             "mean_acceptance_length": total_acc / (steps * S) + 1.0}
    return out[:, :max_new], stats
