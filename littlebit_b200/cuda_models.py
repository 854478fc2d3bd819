"""CUDA draft / target models for speculative decoding on one B200.

``CudaDraftModel`` and ``CudaTargetModel`` are drop-ins for the reference's
CPU adapters (cpu_draft_model.py:141-593, cpu_target_model.py:137-556): same
constructors (runtime checkpoint paths + base model id), same methods
(``reset / prefill / generate_draft_tokens`` and ``reset_cache / forward``),
same KV-cache bookkeeping (a persistent cache per model, draft positions
rolled back after drafting, the target reusing the longest common prefix of
consecutive calls).  Underneath, every forward is one native decoder step
(lbx_forward) per model, and the greedy loops in speculative_decoding.py use
the device-resident paths below (CUDA graphs, on-device acceptance) instead
of Python-level token loops.

Target semantics (D13 of the reference): ``CudaTargetModel(draft_rt, residual_rt)``
reproduces CPUTargetModel — two full LittleBit models whose final hidden
states are summed before one lm_head (cpu_target_model.py:516-527);
``CudaTargetModel.from_decoder(m)`` wraps a single model whose projections
carry the residual branch (per-layer residual, littlebit.py:104-107), and
``CudaDraftModel.from_target(t)`` is the draft that shares that model's
packed draft factors (branch 0 of every projection, no copy).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import _lib as L
from .model import DecoderShape, LittleBitDecoder, load_runtime
from .ops import PackedLinear, _p, _stream, accept_greedy_chain, lib, lmhead_argmax

PREFILL_CHUNK = 16  # tokens per decoder step while prefilling


@dataclass
class _Out:
    logits: torch.Tensor
    past_key_values: object = None


def _embed_and_head(state, base_model_id):
    """The runtime checkpoint may carry embed/lm_head; otherwise take them from the
    base model as the CPU adapters do (cpu_draft_model.py:181-201)."""
    emb = state.get("model.embed_tokens.weight")
    head = state.get("lm_head.weight")
    if (emb is None or head is None) and base_model_id:
        from transformers import AutoModelForCausalLM

        base = AutoModelForCausalLM.from_pretrained(base_model_id, torch_dtype=torch.bfloat16,
                                                    low_cpu_mem_usage=True)
        emb = base.model.embed_tokens.weight.data if emb is None else emb
        head = base.lm_head.weight.data if head is None else head
        del base
    if emb is None or head is None:
        raise ValueError("embedding / lm_head missing: put them in the runtime checkpoint or pass base_model_id")
    return emb, head


def _branch0_view(dec: LittleBitDecoder, max_seq: int) -> LittleBitDecoder:
    """A decoder over branch 0 of every projection of ``dec`` (same device tensors,
    its own KV cache and workspace)."""
    v = LittleBitDecoder.__new__(LittleBitDecoder)
    v.shape, v.device, v.max_seq, v.use_pdl = dec.shape, dec.device, max_seq, dec.use_pdl
    v.exec_mode = getattr(dec, "exec_mode", L.LBX_EXEC_AUTO)
    v.embed, v.lm_head, v.final_norm = dec.embed, dec.lm_head, dec.final_norm
    v.layers = []
    for ly in dec.layers:
        v.layers.append({"ln1": ly["ln1"], "ln2": ly["ln2"],
                         "projs": [PackedLinear(p.in_features, p.out_features, p.branches[:1], p.bias)
                                   for p in ly["projs"]]})
    s = dec.shape
    kvs = (s.num_key_value_heads, max_seq, s.head_dim)
    v.k_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dec.device) for _ in v.layers]
    v.v_cache = [torch.zeros(kvs, dtype=torch.bfloat16, device=dec.device) for _ in v.layers]
    v._build_struct()
    v._ws = torch.zeros(0, dtype=torch.uint8, device=dec.device)
    v._ws_n = 0
    return v


class _Unit:
    """One decoder plus its cache bookkeeping and captured step graphs."""

    def __init__(self, dec: LittleBitDecoder, max_tokens: int = 32):
        self.dec = dec
        self.pos = 0  # next cache slot
        dev = dec.device
        dec.workspace(max_tokens)  # size the workspace once: graphs keep its address
        self.max_tokens = max_tokens
        self.kc_ptrs = torch.tensor([t.data_ptr() for t in dec.k_cache], dtype=torch.int64, device=dev)
        self.vc_ptrs = torch.tensor([t.data_ptr() for t in dec.v_cache], dtype=torch.int64, device=dev)

    def run(self, tokens: torch.Tensor, start: int, **kw):
        n = tokens.numel()
        for a in range(0, n, PREFILL_CHUNK if not kw else n):
            b = min(n, a + (PREFILL_CHUNK if not kw else n))
            self.dec.step(tokens[a:b], start + a, **kw)

    def kv_move(self, src: torch.Tensor, dst: torch.Tensor):
        s = self.dec.shape
        L.check(lib().lbx_kv_move(_p(self.kc_ptrs), _p(self.vc_ptrs), len(self.dec.layers),
                                  s.num_key_value_heads, self.dec.max_seq, s.head_dim, _p(src), _p(dst),
                                  src.numel(), _stream(self.dec.device)), "lbx_kv_move")


class _GraphCache:
    """CUDA graphs of fixed launch sequences, keyed by (kind, size, bound)."""

    def __init__(self):
        self.g: Dict = {}

    def get(self, key, fn, stream):
        if key not in self.g:
            # warm-up outside the capture (one-time attribute setup etc.).  It is a
            # real step with side effects (KV rows, outputs), so it must see this
            # step's inputs: order it after the copies queued on the current stream;
            # the replay that follows rewrites the same slots with the same values
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                fn()
            self.g[key] = graph
        return self.g[key]


def _bound(pos: int, extra: int, max_seq: int) -> int:
    """Upper bound of the cached-slot count a graph is captured for (it sizes the
    attention grid; chunks past the live length exit at once).  Power-of-two
    buckets from 512 keep the number of captured graphs logarithmic."""
    b = 512
    while b < pos + extra + 1:
        b *= 2
    return max(pos, min(b, max_seq - extra))


class CudaDraftModel:
    """Draft model (drop-in for CPUDraftModel) on the B200 kernels."""

    def __init__(self, runtime_path=None, base_model_id=None, torch_dtype=None, *,
                 decoder: Optional[LittleBitDecoder] = None, device="cuda", max_seq_len: int = 4096,
                 use_graphs: bool = True):
        if decoder is None:
            state, shape, _ = load_runtime(runtime_path)
            emb, head = _embed_and_head(state, base_model_id)
            decoder = LittleBitDecoder(shape, state, device=device, max_seq=max_seq_len, embed=emb,
                                       lm_head=head)
        self._init(decoder, use_graphs)

    @classmethod
    def from_decoder(cls, decoder: LittleBitDecoder, use_graphs: bool = True) -> "CudaDraftModel":
        self = cls.__new__(cls)
        self._init(decoder, use_graphs)
        return self

    @classmethod
    def from_target(cls, target: "CudaTargetModel", use_graphs: bool = True) -> "CudaDraftModel":
        """The draft sharing the packed draft factors of a per-layer-residual target."""
        if target._mode != "combined":
            raise ValueError("from_target needs a target built with CudaTargetModel.from_decoder")
        d = target._units[0].dec
        return cls.from_decoder(_branch0_view(d, d.max_seq), use_graphs)

    def _init(self, decoder: LittleBitDecoder, use_graphs: bool):
        self.dec = decoder
        self.config = decoder.shape
        self.device = decoder.device
        self.max_seq_len = decoder.max_seq
        self.use_graphs = use_graphs
        self.unit = _Unit(decoder)
        self._vocab_size = decoder.shape.vocab_size
        self._cached_ids: List[int] = []
        dev = self.device
        self.tok_buf = torch.zeros(65, dtype=torch.int64, device=dev)
        self.start_buf = torch.zeros(64, dtype=torch.int32, device=dev)
        self.iota = torch.arange(64, dtype=torch.int32, device=dev)
        self.logits_buf = torch.zeros(64, self._vocab_size, dtype=torch.float32, device=dev)
        self._graphs = _GraphCache()
        self._stream = torch.cuda.Stream(dev)

    # ---- reference API ------------------------------------------------------
    def reset(self):
        self.unit.pos = 0
        self._cached_ids = []

    @property
    def _cache_pos(self):
        return self.unit.pos

    def _sync_prefix(self, ids: List[int], upto: int):
        """Make the cache hold exactly ids[:upto] (reusing the common prefix)."""
        c = 0
        lim = min(upto, len(self._cached_ids), self.unit.pos)
        while c < lim and self._cached_ids[c] == ids[c]:
            c += 1
        if c < upto:
            t = torch.tensor(ids[c:upto], dtype=torch.int64, device=self.device)
            self.unit.run(t, c)
        self.unit.pos = upto
        self._cached_ids = list(ids[:upto])

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor):
        ids = input_ids[0].tolist()
        self._sync_prefix(ids, len(ids))

    @torch.no_grad()
    def generate_draft_tokens(self, input_ids: torch.Tensor, attention_mask=None, draft_length: int = 5,
                              temperature: float = 1.0, greedy: bool = True):
        """Draft ``draft_length`` tokens after ``input_ids``; returns ([(1,1) ids], [(1,V) probs]).
        The draft positions are rolled back afterwards (cpu_draft_model.py:589-591)."""
        ids = input_ids[0].tolist()
        P = len(ids) - 1
        self._sync_prefix(ids, P)
        toks, probs = [], []
        cur = ids[-1]
        dev = self.device
        for i in range(draft_length):
            out = self.dec.forward_tokens([cur], P + i, want_logits=True, want_argmax=True)
            lg = out["logits"]
            p = F.softmax(lg / max(temperature, 1e-8), dim=-1)
            if greedy:
                nxt = out["argmax"].view(1, 1)
            else:
                nxt = torch.multinomial(p, num_samples=1)
            toks.append(nxt)
            probs.append(p)
            cur = int(nxt)
        # the last input token stays committed; the draft positions roll back
        self.unit.pos = P + 1
        self._cached_ids = ids[:]
        return toks, probs

    @torch.no_grad()
    def forward(self, input_ids, attention_mask=None, past_key_values=None, use_cache=True):
        """Full-sequence logits (1, seq, V) over a fresh pass (reference HF-style call)."""
        ids = input_ids[0].tolist()
        self._sync_prefix(ids, 0)
        n = len(ids)
        lg = torch.empty(n, self._vocab_size, dtype=torch.float32, device=self.device)
        t = torch.tensor(ids, dtype=torch.int64, device=self.device)
        for a in range(0, n, PREFILL_CHUNK):
            b = min(n, a + PREFILL_CHUNK)
            self.dec.step(t[a:b], a, logits=lg[a:b])
        self.unit.pos = n
        self._cached_ids = ids[:]
        return _Out(lg[None])

    # ---- device-resident drafting -------------------------------------------
    def _draft_graph(self, k: int, bound: int):
        dec = self.dec

        def seq():
            for i in range(k):
                dec.step(self.tok_buf[i:i + 1], bound, start_dev=self.start_buf[i:i + 1],
                         argmax=self.tok_buf[i + 1:i + 2])
        return self._graphs.get(("draft", k, bound), seq, self._stream)

    def draft_on_device(self, P: int, k: int):
        """Greedy-draft k tokens: tok_buf[0] holds the token at slot P (already set on
        the device); tok_buf[1..k] receive the drafts.  No host synchronisation."""
        torch.add(self.iota[:k], P, out=self.start_buf[:k])
        if self.use_graphs:
            bound = _bound(P, k, self.max_seq_len)
            g = self._draft_graph(k, bound)
            self._stream.wait_stream(torch.cuda.current_stream())
            g.replay()
            torch.cuda.current_stream().wait_stream(self._stream)
        else:
            for i in range(k):
                self.dec.step(self.tok_buf[i:i + 1], P + i, argmax=self.tok_buf[i + 1:i + 2])

    def expand_tree(self, input_ids: torch.Tensor, tree_buffers: Dict, top_k: int = 10,
                    temperature: float = 1.0) -> torch.Tensor:
        """generate_draft_tree on the device: the root's top-k fill depth 1, then each
        depth level is expanded by ONE tree-masked forward over all nodes up to that
        depth (the reference runs one full-prefix forward per expanded node), one
        batched top-k over the level's parents and one indexed fill of their
        children.  Everything but the tokens depends only on the tree's shape and is
        planned once per shape (``_tree_plan``)."""
        ids = input_ids[0].tolist()
        P = len(ids) - 1
        self._sync_prefix(ids, P)
        dev = self.device
        plan = _tree_plan(tree_buffers, top_k, dev)
        root = self.dec.forward_tokens([ids[-1]], P, want_logits=True, want_argmax=False)["logits"]
        self.unit.pos = P + 1
        self._cached_ids = ids[:]
        inv_t = 1.0 / max(temperature, 1e-5)
        cand = torch.zeros(plan["T"], dtype=torch.int64, device=dev)
        cand[0] = ids[-1]
        ktop = torch.topk(root[0] * inv_t if temperature != 1.0 else root[0], top_k).indices
        cand[plan["d1_nodes"]] = ktop[plan["d1_ranks"]]
        for lv in plan["levels"]:
            out = self.dec.forward_tokens(cand[lv["nodes"]], P + 1, pos=[P + o for o in lv["depth"]],
                                          tree_mask=lv["bits"], want_logits=True, want_argmax=False)["logits"]
            if lv["kids"] is None:
                continue
            par = out[lv["parent_rows"]]
            kt = torch.topk(par * inv_t if temperature != 1.0 else par, top_k).indices
            cand[lv["kids"]] = kt[lv["kid_parent"], lv["kid_rank"]]
        return cand[None]


_TREE_PLANS: Dict = {}


def _tree_plan(tree_buffers: Dict, top_k: int, dev) -> Dict:
    """Per tree shape: for each depth level the nodes of the level's forward (all
    nodes up to that depth, in index order), their tree-mask bits over those
    nodes, their depths, the rows of the level's parents and, per child, its node
    index, its parent's row among those and its top-k rank."""
    from .tree_utils import tree_bitmasks

    sc = tree_buffers["sorted_tree_choices"]
    key = (tuple(tuple(c) for c in sc), int(tree_buffers["tree_len"]), int(top_k), str(dev))
    plan = _TREE_PLANS.get(key)
    if plan is not None:
        return plan
    T = tree_buffers["tree_len"]
    depth_of = [0] + [len(c) for c in sc]
    index = {tuple(c): i + 1 for i, c in enumerate(sc)}
    full_bits = tree_bitmasks(tree_buffers["tree_attn_mask"])  # over all T nodes (root = bit 0)
    d1 = [c for c in sc if len(c) == 1]
    t64 = lambda v: torch.tensor(v, dtype=torch.int64, device=dev)
    levels = []
    for d in range(1, max(depth_of)):
        nodes = [i for i in range(1, T) if depth_of[i] <= d]
        # nodes occupy slots P+1 .. in index order; drop the root bit (it is cached)
        remap = {j: r for r, j in enumerate(nodes)}
        bits = []
        for i in nodes:
            b = int(full_bits[i]) & ((1 << 64) - 1)
            v = 0
            for j in nodes:
                if (b >> j) & 1:
                    v |= 1 << remap[j]
            bits.append(v - (1 << 64) if v >= (1 << 63) else v)
        parent_rows, kids, kid_parent, kid_rank = [], [], [], []
        for r, i in enumerate(nodes):
            if depth_of[i] != d:
                continue
            path = tuple(sc[i - 1])
            ch = [c for c in sc if len(c) == d + 1 and tuple(c[:d]) == path]
            if not ch:
                continue
            for c in ch:
                kids.append(index[tuple(c)])
                kid_parent.append(len(parent_rows))
                kid_rank.append(c[-1])
            parent_rows.append(r)
        levels.append({"nodes": t64(nodes), "bits": bits, "depth": [depth_of[i] for i in nodes],
                       "parent_rows": t64(parent_rows) if kids else None,
                       "kids": t64(kids) if kids else None,
                       "kid_parent": t64(kid_parent) if kids else None,
                       "kid_rank": t64(kid_rank) if kids else None})
    plan = {"T": T, "levels": levels, "d1_nodes": t64([index[tuple(c)] for c in d1]),
            "d1_ranks": t64([c[0] for c in d1])}
    _TREE_PLANS[key] = plan
    return plan


class CudaTargetModel:
    """Target model (drop-in for CPUTargetModel) on the B200 kernels."""

    def __init__(self, draft_runtime_path=None, residual_runtime_path=None, base_model_id=None,
                 torch_dtype=None, *, device="cuda", max_seq_len: int = 4096, use_graphs: bool = True):
        sd, shape, _ = load_runtime(draft_runtime_path)
        sr, shape_r, _ = load_runtime(residual_runtime_path)
        emb, head = _embed_and_head({**sr, **sd}, base_model_id)
        d = LittleBitDecoder(shape, sd, device=device, max_seq=max_seq_len, embed=emb, lm_head=head)
        r = LittleBitDecoder(shape_r, sr, device=device, max_seq=max_seq_len, embed=d.embed, lm_head=d.lm_head)
        self._init([d, r], "hidden_sum", use_graphs)

    @classmethod
    def from_decoder(cls, decoder: LittleBitDecoder, use_graphs: bool = True) -> "CudaTargetModel":
        """Per-layer residual target: one model whose projections carry both branches."""
        self = cls.__new__(cls)
        self._init([decoder], "combined", use_graphs)
        return self

    @classmethod
    def from_decoders(cls, draft_unit: LittleBitDecoder, residual_unit: LittleBitDecoder,
                      use_graphs: bool = True) -> "CudaTargetModel":
        self = cls.__new__(cls)
        self._init([draft_unit, residual_unit], "hidden_sum", use_graphs)
        return self

    def _init(self, decs, mode: str, use_graphs: bool):
        self._mode = mode
        self._units = [_Unit(d) for d in decs]
        d0 = decs[0]
        self.config = d0.shape
        self.device = d0.device
        self.max_seq_len = d0.max_seq
        self._vocab_size = d0.shape.vocab_size
        self.use_graphs = use_graphs
        self._cached_tokens: Optional[List[int]] = None
        dev = self.device
        H = d0.shape.hidden_size
        self.h_buf = [torch.zeros(64, H, dtype=torch.float32, device=dev) for _ in decs]
        self.am_buf = torch.zeros(64, dtype=torch.int64, device=dev)
        self.start_buf = torch.zeros(1, dtype=torch.int32, device=dev)
        self.vtok = torch.zeros(64, dtype=torch.int64, device=dev)
        self._graphs = _GraphCache()
        self._stream = torch.cuda.Stream(dev)
        self._lm_ws = torch.zeros(int(lib().lbx_lmhead_workspace_size(64, self._vocab_size)),
                                  dtype=torch.uint8, device=dev)

    # ---- reference API ------------------------------------------------------
    def reset_cache(self):
        for u in self._units:
            u.pos = 0
        self._cached_tokens = None

    def _head(self, n: int, logits=None, argmax=None, pdl: bool = False):
        """Summed final hidden states of the units -> lm_head (hidden-sum target)."""
        hs = self.h_buf[0][:n]
        for h in self.h_buf[1:]:
            hs.add_(h[:n])
        d0 = self._units[0].dec
        L.check(lib().lbx_lmhead_argmax(_p(hs), None, 0.0, n, d0.shape.hidden_size, _p(d0.lm_head),
                                        self._vocab_size, _p(logits), _p(argmax), _p(self._lm_ws),
                                        self._lm_ws.numel(), 1 if pdl else 0, _stream(self.device)),
                "lmhead_argmax")

    def _step(self, tokens: torch.Tensor, start: int, logits=None, argmax=None, start_dev=None,
              pos=None, tree_mask=None):
        n = tokens.numel()
        if self._mode == "combined":
            self._units[0].dec.step(tokens, start, logits=logits, argmax=argmax, start_dev=start_dev,
                                    pos=pos, tree_mask=tree_mask)
        else:
            for u, h in zip(self._units, self.h_buf):
                u.dec.step(tokens, start, hidden=h[:n], start_dev=start_dev, pos=pos, tree_mask=tree_mask)
            self._head(n, logits, argmax)

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, attention_mask=None) -> torch.Tensor:
        """Logits (1, seq, V) of the combined target; positions inside the reused
        cached prefix are zero, as in cpu_target_model.py:550-556."""
        ids = input_ids[0].tolist()
        seq = len(ids)
        common = 0
        if self._cached_tokens is not None:
            m = min(seq, len(self._cached_tokens))
            while common < m and ids[common] == self._cached_tokens[common]:
                common += 1
        dev = self.device
        out = torch.zeros(1, seq, self._vocab_size, dtype=torch.float32, device=dev)
        if seq - common > 0:
            t = torch.tensor(ids[common:], dtype=torch.int64, device=dev)
            for a in range(0, t.numel(), PREFILL_CHUNK):
                b = min(t.numel(), a + PREFILL_CHUNK)
                self._step(t[a:b], common + a, logits=out[0, common + a:common + b])
        for u in self._units:
            u.pos = seq
        self._cached_tokens = ids
        return out

    # ---- device-resident verification -------------------------------------
    def prefill_ids(self, ids: List[int], upto: int):
        if upto > 0:
            t = torch.tensor(ids[:upto], dtype=torch.int64, device=self.device)
            for a in range(0, upto, PREFILL_CHUNK):
                b = min(upto, a + PREFILL_CHUNK)
                if self._mode == "combined":
                    self._units[0].dec.step(t[a:b], a)
                else:
                    for u in self._units:
                        u.dec.step(t[a:b], a)
        for u in self._units:
            u.pos = upto
        self._cached_tokens = list(ids[:upto])

    def _verify_graph(self, n: int, bound: int):
        # positions come from start_buf on the device (slots start..start+n-1)
        def seq():
            self._step(self.vtok[:n], bound, argmax=self.am_buf[:n], start_dev=self.start_buf)
        return self._graphs.get(("verify", n, bound), seq, self._stream)

    def verify_on_device(self, tokens: torch.Tensor, P: int, n: int) -> torch.Tensor:
        """Target argmax [n] for tokens[0..n) at slots P.. (no host sync)."""
        self.start_buf.fill_(P)
        if self.use_graphs:
            if tokens.data_ptr() != self.vtok.data_ptr():
                self.vtok[:n].copy_(tokens[:n])
            g = self._verify_graph(n, _bound(P, n, self.max_seq_len))
            self._stream.wait_stream(torch.cuda.current_stream())
            g.replay()
            torch.cuda.current_stream().wait_stream(self._stream)
        else:
            self._step(tokens[:n], P, argmax=self.am_buf[:n])
        return self.am_buf[:n]

    def verify_tree(self, cand: torch.Tensor, P: int, tree_buffers: Dict):
        """Argmax of every tree node: cand [T] (root = token at slot P) at slots P..P+T-1,
        rotary positions P + depth, tree attention mask."""
        from .tree_utils import tree_bitmasks

        T = cand.numel()
        key = (tuple(tuple(c) for c in tree_buffers["sorted_tree_choices"]), T, str(self.device))
        cached = self._verify_plan if getattr(self, "_verify_plan_key", None) == key else None
        if cached is None:  # per tree shape: position offsets and mask bits on the device
            cached = (tree_buffers["tree_position_ids"].to(self.device).to(torch.int32),
                      tree_bitmasks(tree_buffers["tree_attn_mask"]).to(self.device))
            self._verify_plan, self._verify_plan_key = cached, key
        pos = P + cached[0]
        bits = cached[1]
        am = torch.empty(T, dtype=torch.int64, device=self.device)
        self._step(cand, P, argmax=am, pos=pos, tree_mask=bits)
        return am

    def kv_move(self, src: torch.Tensor, dst: torch.Tensor):
        for u in self._units:
            u.kv_move(src, dst)
