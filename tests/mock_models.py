"""Deterministic table-driven draft/target models with the duck-typed interface
the speculative loop calls (speculative_decoding.py:58-134, 137-163):
``draft.generate_draft_tokens(input_ids, attention_mask, draft_length,
temperature, greedy) -> (tokens[(1,1)], probs[(1,V)])`` and
``target.forward(input_ids, attention_mask) -> logits [1, seq, V]``.

Target logits at position t depend on the last two tokens; the draft adds a
perturbation so it agrees with the target only part of the time.  Used to
pin the loop's control flow (golden vectors from the reference, oracle
restatement, and the B200 package's host loop).
"""
from __future__ import annotations

import numpy as np


def mock_tables(vocab: int = 50, seed: int = 5):
    r = np.random.default_rng(seed)
    return {
        "A": r.standard_normal((vocab, vocab)).astype(np.float32),
        "B": r.standard_normal((vocab, vocab)).astype(np.float32),
        "N": r.standard_normal((vocab, vocab)).astype(np.float32),
        "vocab": vocab,
    }


def target_logits_np(tabs, ids):
    ids = np.asarray(ids)
    prev = np.concatenate([[ids[0]], ids[:-1]])
    return tabs["A"][ids] + 0.5 * tabs["B"][prev]


def draft_logits_np(tabs, ids):
    ids = np.asarray(ids)
    return target_logits_np(tabs, ids) + 0.9 * tabs["N"][ids]


class MockTarget:
    def __init__(self, tabs, torch):
        self.tabs, self.torch = tabs, torch

    def forward(self, input_ids, attention_mask=None):
        ids = input_ids[0].tolist()
        return self.torch.from_numpy(target_logits_np(self.tabs, ids))[None]


class MockDraft:
    def __init__(self, tabs, torch):
        self.tabs, self.torch = tabs, torch

    def generate_draft_tokens(self, input_ids, attention_mask=None, draft_length=5,
                              temperature=1.0, greedy=True):
        torch = self.torch
        ids = input_ids[0].tolist()
        toks, probs = [], []
        for _ in range(draft_length):
            lg = torch.from_numpy(draft_logits_np(self.tabs, ids)[-1:])
            t = int(torch.argmax(lg, dim=-1))
            toks.append(torch.tensor([[t]]))
            probs.append(torch.softmax(lg, dim=-1))
            ids.append(t)
        return toks, probs
