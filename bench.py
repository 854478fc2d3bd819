"""Benchmark: LittleBitLinear GB/s vs HBM peak on the BASELINE config-2 layer.

Workload (per GPU): the 4096->4096 LittleBitLinear with a draft branch of
rank 208 and a residual branch of rank 1840 (independent V_R), random packed
±1 factors and |N(1,0.1)| scales, bf16 activations.  One STEP is a chain of
POOL distinct layer instances (x_{i+1} = y_i, like a deep stack), so each
step streams POOL x 2.28 MB of packed weights — 128 layers = 292 MB, more
than twice the 126 MB L2, so every step reads the weights from HBM (no L2
flush needed).  A step is one CUDA graph replay: by default the fused chain
executor (lbx_chain_fused: one launch per layer, layer i's U-stage with layer
i+1's V-stage partials, chained with programmatic dependent launch); the
two-stage grids, the cluster executor and the persistent program are timed
beside it and must give the same bits.  Scales are |N(1,0.1)| with mid and u1
divided by sqrt(in) and sqrt(rank x branches) so that every layer has unit
gain: with the raw scales the chain's activations overflow within ~11 layers
and collapse to zero, which lets the kernels skip work.

value   = algorithmic bytes of all layers of all ranks / max-over-ranks time
          (packed bits without word padding + fp32 scales + activations in/out)
e2e     = the same metric through the C-ABI call itself: every step copies
          x from pinned host memory to the device, the host calls
          lbx_chain_fused (ctypes) once for the chain, and the last layer's y
          is copied back to pinned host memory (8 KB each way per step at
          k=1).  The bench captures nothing; the library replays its own
          cached graph of a call it has seen (built during warm-up).
          e2e_per_layer_calls makes one lbx_linear_verify call per layer
          instead; e2e_graph is the default executor's step with the same
          copies, captured by the bench in a CUDA graph.
configs = the other BASELINE layer configs, each as its own chain: C1 (fp32,
          r=208), C2 verify at k=5 and k=8, the shared-factor target layer of
          config 4 (draft r=208 + residual U_R of the same rank on the draft's
          V-stage) at k=1 and k=5.
floor   = the same grids with the same PDL chaining and no arithmetic
          (lbx_linear_floor), without and with the weight copies.
roofline: the linear (V+U kernel pair) is the dominant kernel; achieved =
          bytes per layer call / mean layer time; peak = MEASURED_PEAKS.json
cpu_baseline: the reference's own C++ op (oracle/_ref, littlebit_linear from
          patches/littlebit_cpu_optimized.cpp) on the host cores, a bounded
          sample of the same layer.

    python bench.py [--gpus N --steps K --warmup W --tokens k --impl reference]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "LittleBitLinear GB/s vs HBM peak; spec-decode tokens/s, Llama-2-7B shape"
IN_F = OUT_F = 4096
RANKS = [208, 1840]


def layer_bytes(k: int, ranks=RANKS, shared: bool = False, esz: int = 2) -> tuple[int, int]:
    """(algorithmic bytes per layer call, packed-weight bytes) for k tokens of
    esz-byte activations: packed bits without word padding, fp32 scales, x read
    and y written.  A shared-factor residual (config 4) has no V or v2 of its own."""
    packed, scales = 0, 0
    for i, r in enumerate(ranks):
        own_v = not (shared and i > 0)
        packed += (OUT_F * r + 7) // 8 + ((r * IN_F + 7) // 8 if own_v else 0)
        scales += 4 * (r + OUT_F) + (4 * IN_F if own_v else 0)
    act = esz * k * IN_F + esz * k * OUT_F
    return packed + scales + act, packed


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_from_profiles(k: int, exec_name: str):
    """DRAM bytes per layer of the committed ncu capture of this executor
    (None when there is none: the persistent program has no per-layer launch)."""
    name = {"kernels": f"linear_c2_k{k}.md", "cluster": f"linear_cluster_c2_k{k}.md",
            "fused": f"chain_fused_c2_k{k}.md"}.get(exec_name)
    if name is None:
        return None
    f = ROOT / "profiles" / name
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch\s*=\s*([0-9]+)", f.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) >= 9:
                for nm, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        return dist.get_rank(), ws, local
    return 0, 1, 0


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the reference's own C++ op on host cores
# ---------------------------------------------------------------------------
def ref_chain(k: int, nlayers: int):
    """The reference's CPU op (littlebit_cpu_ops.littlebit_linear, compiled from
    the reference's own sources into oracle/_ref) over a chain of `nlayers`
    distinct C2 layers, main + residual branch summed per layer
    (littlebit.py:104-107); returns (one_pass, threads) or None when the op is
    not built."""
    from oracle import build_ref  # CPU baseline / reference arm only

    if not build_ref.load():
        return None
    from littlebit_b200 import synthetic as syn

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    layers = [syn.layer(IN_F, OUT_F, RANKS, g) for _ in range(nlayers)]
    op = torch.ops.littlebit_cpu_ops.littlebit_linear
    x0 = torch.randn(k, IN_F, generator=g).bfloat16().float()

    def one_pass():
        x = x0
        for lay in layers:
            y = None
            for b in lay:
                yb = op(x, b["v2"][None], b["v_sign"], IN_F, b["mid"][None], b["u_sign"], b["rank"],
                        b["u1"][None])
                y = yb if y is None else y + yb
            x = y.bfloat16().float()
        return x

    return one_pass, torch.get_num_threads()


def cpu_reference(k: int, budget_s: float, nlayers: int):
    """CPU baseline of our arm: passes of the reference op over the layer chain
    for about `budget_s` seconds."""
    r = ref_chain(k, nlayers)
    if r is None:
        return None
    one_pass, threads = r
    for _ in range(2):  # warm-up
        one_pass()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        one_pass()
        times.append(time.perf_counter() - t0)
    b, _ = layer_bytes(k)
    med = statistics.median(times)
    return {"gbs": b * nlayers / med / 1e9, "threads": threads,
            "sample": f"{len(times)} passes (median) of littlebit_linear x2 branches (r={RANKS}) over "
                      f"{nlayers} distinct layers, k={k}, {threads} threads"}


def cpu_decode_reference(r_d: dict, r_r: dict, prompt: int, quick: bool = False):
    """C3/C4 CPU baselines: the reference's own full_forward, generate_token and
    full_forward_batch ops (oracle/_ref, compiled from
    patches/littlebit_cpu_optimized.cpp:1522-2317) on the Llama-2-7B shape with
    random packed signs in the layout CPUDraftModel builds
    (cpu_draft_model.py:229-264: 37 tensors and 28 dims per layer, signs
    repacked by the reference's repack_signs_to_i2), timed the way
    benchmark_models_cpu.py:31-135 does: warm-up tokens, per-token
    perf_counter, tokens/s = measured tokens / summed time.

      draft_full_forward   per token dense_gemv_f32 lm_head + argmax +
                           full_forward (benchmark_draft's loop)
      draft_generate_token generate_token (Q4_0 lm_head, fused argmax)
      target_two_model     CPUTargetModel's step: full_forward_batch of the new
                           token on the draft and the residual model, hidden
                           sum, fp32 lm_head (benchmark_target's loop)
      verify_gamma4        the same step over 5 tokens (chain verify, gamma 4)

    The KV caches hold ``prompt`` zero-filled positions standing in for the
    prompt's prefill: the ops' work per token depends on the position only."""
    from oracle import build_ref  # CPU baseline only

    if not build_ref.load():
        return None
    import torch.nn.functional as F

    from littlebit_b200.model import LLAMA2_7B, PROJ_NAMES

    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    ro = torch.ops.littlebit_cpu_ops
    sh = LLAMA2_7B
    H, I, nl, V = sh.hidden_size, sh.intermediate_size, sh.num_hidden_layers, sh.vocab_size
    kvh, hd = sh.num_key_value_heads, sh.head_dim
    dims = {"q_proj": (H, H), "k_proj": (H, kvh * hd), "v_proj": (H, kvh * hd), "o_proj": (H, H),
            "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    g = torch.Generator().manual_seed(3)

    def words(rows, cols):
        w = torch.randint(-(2 ** 31), 2 ** 31, (rows, (cols + 31) // 32), generator=g, dtype=torch.int64)
        if cols % 32:
            w[:, -1] &= (1 << (cols % 32)) - 1
        return w.to(torch.int32)

    sc = lambda n: (1 + 0.1 * torch.randn(n, generator=g)).abs()
    max_seq = prompt + 32
    t_build = time.perf_counter()

    def unit(ranks):
        tens, ld = [], []
        for _ in range(nl):
            tens += [sc(H), sc(H)]
            for nm in PROJ_NAMES:
                in_f, out_f = dims[nm]
                r = ranks[nm]
                tens += [sc(in_f), ro.repack_signs_to_i2(words(r, in_f), in_f), sc(r) / in_f ** 0.5,
                         ro.repack_signs_to_i2(words(out_f, r), r), sc(out_f) / r ** 0.5]
                ld += [in_f, r, r, out_f]
        kv = [torch.zeros(kvh, max_seq, hd) for _ in range(2 * nl)]
        return tens, ld, kv

    embed = 0.02 * torch.randn(V, H, generator=g)
    head = 0.02 * torch.randn(V, H, generator=g)
    fnorm = sc(H)
    d_t, d_l, d_kv = unit(r_d)
    q4 = ro.quantize_lm_head_q4(head)
    common = (nl, H, kvh, sh.num_attention_heads // kvh, hd, max_seq)
    scale, eps = hd ** -0.5, sh.rms_norm_eps

    def per_token(fn, warm, meas):
        ts = []
        for i in range(warm + meas):
            t0 = time.perf_counter()
            fn(prompt + i)
            if i >= warm:
                ts.append(time.perf_counter() - t0)
        return {"tokens_per_s": round(len(ts) / sum(ts), 3), "ms_per_token": round(sum(ts) / len(ts) * 1e3, 2),
                "measured_tokens": len(ts), "warmup_tokens": warm}

    state = {"tok": 1, "h": torch.zeros(1, H)}

    def draft_ff(pos):
        lg = ro.dense_gemv_f32(state["h"].reshape(1, -1).contiguous(), head)
        state["tok"] = int(torch.argmax(lg, dim=-1).item())
        state["h"] = ro.full_forward(state["tok"], embed, fnorm, d_t, d_kv, d_l, *common[:5], max_seq, pos,
                                     scale, eps)

    def draft_gt(pos):
        state["tok"] = int(ro.generate_token(state["tok"] % V, embed, fnorm, d_t, d_kv, d_l, q4, V, *common[:5],
                                             max_seq, pos, scale, eps))

    out = {"threads": threads, "model": "Llama-2-7B shape, 0.1-bit draft ranks " + json.dumps(r_d),
           "start_position": prompt}
    out["draft_full_forward"] = per_token(draft_ff, 5, 8 if quick else 20)
    out["draft_generate_token"] = per_token(draft_gt, 5, 8 if quick else 20)
    r_t, r_l, r_kv = unit(r_r)
    out["build_s"] = round(time.perf_counter() - t_build, 1)

    def target_n(n):
        def fn(pos):
            ids = torch.full((n,), 1, dtype=torch.int64)
            hdd = ro.full_forward_batch(ids, embed, fnorm, d_t, d_kv, d_l, *common[:5], max_seq, pos, scale, eps)
            hr = ro.full_forward_batch(ids, embed, fnorm, r_t, r_kv, r_l, *common[:5], max_seq, pos, scale, eps)
            lg = F.linear((hdd + hr).to(torch.float32), head)
            state["tok"] = int(lg[-1].argmax().item())
        return fn

    out["target_two_model"] = per_token(target_n(1), 2, 3 if quick else 6)
    out["target_two_model"]["residual_ranks"] = r_r
    out["verify_gamma4"] = per_token(target_n(5), 1, 2 if quick else 3)
    out["verify_gamma4"]["note"] = "tokens_per_s counts verify calls of 5 tokens"
    out["timing"] = "benchmark_models_cpu.py:31-135 method (warm-up, per-token perf_counter); reference ops"
    return out


def run_reference(args):
    """The reference's CPU op on this workload: W warm-up passes, then exactly K
    timed passes over the chain of --pool distinct layers."""
    rank, ws, _ = dist_init()
    if rank != 0:
        return 0
    r = ref_chain(args.tokens, args.pool)
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference C++ op not built (oracle/_ref missing: run oracle/build_ref.py)"}))
        return 0
    one_pass, threads = r
    for _ in range(args.warmup):
        one_pass()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_pass()
    dt = time.perf_counter() - t0
    b, _ = layer_bytes(args.tokens)
    val = b * args.pool * args.steps / dt / 1e9
    sample = (f"{args.steps} passes of littlebit_linear x2 branches (r={RANKS}) over {args.pool} distinct "
              f"layers, k={args.tokens}, {threads} threads")
    out = {
        "metric": METRIC, "impl": "reference", "value": round(val, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xsign/fp32 (W1A8)", "data": "synthetic",
        "config": {"workload": f"C2 4096->4096 LittleBitLinear r={RANKS[0]}+{RANKS[1]} (independent V_R), "
                               f"k={args.tokens}, chain of {args.pool} distinct layers per step, reference "
                               "CPU op", "tokens": args.tokens, "pool_layers": args.pool},
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out))
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def build_pool(P: int, device, seed: int, ranks=RANKS, shared: bool = False):
    """P distinct layers generated on the device (random words == Bernoulli(0.5)
    signs, |N(1,0.1)| scales, mid / sqrt(in) and u1 / sqrt(rank) so that a
    layer has unit gain and a deep chain's activations stay finite);
    ``shared``: the second branch reuses the first branch's V-stage
    (littlespec_ref/littlebit_itq_spec.py:298-309)."""
    from littlebit_b200.ops import Branch, PackedLinear

    g = torch.Generator(device=device).manual_seed(seed)
    pool = []
    for _ in range(P):
        brs = []
        for i, r in enumerate(ranks):
            def words(rows, cols):
                w = torch.randint(-(2 ** 31), 2 ** 31, (rows, (cols + 31) // 32), generator=g,
                                  device=device, dtype=torch.int64)
                if cols % 32:
                    w[:, -1] &= (1 << (cols % 32)) - 1
                return w.to(torch.int32)
            sc = lambda n: (1 + 0.1 * torch.randn(n, generator=g, device=device)).abs()
            mid, u1 = sc(r) / IN_F ** 0.5, sc(OUT_F) / (r * len(ranks)) ** 0.5
            if shared and i > 0:
                brs.append(Branch(None, None, mid, words(OUT_F, r), u1, r))
            else:
                brs.append(Branch(words(r, IN_F), sc(IN_F), mid, words(OUT_F, r), u1, r))
        pool.append(PackedLinear(IN_F, OUT_F, brs))
    return pool


# ---------------------------------------------------------------------------
# decode: spec-decode tokens/s on the Llama-2-7B shape
# ---------------------------------------------------------------------------
def _ranks_at(shape, eff_bit):
    from littlebit_b200.littlebit import LittleBitLinear

    H, I = shape.hidden_size, shape.intermediate_size
    qd = shape.num_attention_heads * shape.head_dim
    kvd = shape.num_key_value_heads * shape.head_dim
    dims = {"q_proj": (H, qd), "k_proj": (H, kvd), "v_proj": (H, kvd), "o_proj": (qd, H),
            "gate_proj": (H, I), "up_proj": (H, I), "down_proj": (I, H)}
    out = {}
    for nm, (a, b) in dims.items():
        f = LittleBitLinear._estimate_split_dim(a, b, eff_bit, False)
        out[nm] = LittleBitLinear._finalize_split_dim(f, 1024, 8)
    return out


def run_decode(args, dev, rank, ws):
    """Greedy decode on the Llama-2-7B shape: 0.1-bit draft
    (ranks of littlebit.py:50-93 at eff_bit 0.1), target = draft + an independent
    0.9-bit residual branch per projection (~1.0 BPW).  128-token uniform-random
    prompt, 256 new tokens; target-only greedy, chain speculation (gamma 4) and
    depth-4 binary-tree speculation, each checked token-identical to target-only.
    Weights: |N(1,0.1)| scales times unit-gain constants (mid / sqrt(in),
    u1 / sqrt(rank)); the residual's u1 is further scaled by res_scale so that the
    draft agrees with the target often enough for speculation to matter."""
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.model import LLAMA2_7B, LittleBitDecoder, synthetic_runtime_state
    from littlebit_b200.speculative_decoding import (autoregressive_generate, speculative_decode,
                                                     speculative_decode_tree)
    from littlebit_b200.tree_utils import binary_tree_choices, generate_tree_buffers

    shape = LLAMA2_7B
    r_d, r_r = _ranks_at(shape, 0.1), _ranks_at(shape, 0.9)
    ranks = {k: [r_d[k], r_r[k]] for k in r_d}
    st = synthetic_runtime_state(shape, ranks, seed=77 + rank, device=dev, unit_gain=True)
    for k in list(st):
        if k.endswith(".u1_r"):
            st[k] = st[k] * args.res_scale
    max_seq = args.prompt + args.new_tokens + 64
    dec = LittleBitDecoder(shape, st, device=dev, max_seq=max_seq)
    del st
    tgt = CudaTargetModel.from_decoder(dec)
    drf = CudaDraftModel.from_target(tgt)
    draft_only = CudaTargetModel.from_decoder(drf.dec)
    ids = torch.randint(0, shape.vocab_size, (1, args.prompt),
                        generator=torch.Generator().manual_seed(1000 + rank)).to(dev)
    tb = generate_tree_buffers(binary_tree_choices(4, 2), device=dev)
    n = args.new_tokens

    def timed(fn):
        barrier(ws)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        return out, max_over_ranks(dt, ws)

    # warm-up: one short pass of each loop (graph capture, smem attributes)
    autoregressive_generate(draft_only, ids, None, max_new_tokens=8, eos_token_id=-1)
    autoregressive_generate(tgt, ids, None, max_new_tokens=8, eos_token_id=-1)
    speculative_decode(drf, tgt, ids, None, max_new_tokens=8, draft_length=4, eos_token_id=-1)
    speculative_decode_tree(drf, tgt, ids, None, max_new_tokens=8, tree_buffers=tb, top_k=2, eos_token_id=-1)
    (dr, _), t_draft = timed(lambda: autoregressive_generate(draft_only, ids, None, max_new_tokens=n,
                                                              eos_token_id=-1))
    (ar, _), t_ar = timed(lambda: autoregressive_generate(tgt, ids, None, max_new_tokens=n, eos_token_id=-1))
    # prompt prefill + one token: the decode-only rates exclude it
    _, t_draft1 = timed(lambda: autoregressive_generate(draft_only, ids, None, max_new_tokens=1, eos_token_id=-1))
    _, t_ar1 = timed(lambda: autoregressive_generate(tgt, ids, None, max_new_tokens=1, eos_token_id=-1))
    (sp, sst), t_sp = timed(lambda: speculative_decode(drf, tgt, ids, None, max_new_tokens=n, draft_length=4,
                                                       eos_token_id=-1))
    (tr, tst), t_tr = timed(lambda: speculative_decode_tree(drf, tgt, ids, None, max_new_tokens=n,
                                                            tree_buffers=tb, top_k=2, eos_token_id=-1))
    n_tr = tr.shape[1] - ids.shape[1]
    if n_tr > n:  # the tree loop may overshoot max_new_tokens (speculative_decoding.py:560-566)
        ar_long, _ = autoregressive_generate(tgt, ids, None, max_new_tokens=n_tr, eos_token_id=-1)
    else:
        ar_long = ar
    chain_ok = sp.tolist() == ar.tolist()
    tree_ok = tr.tolist() == ar_long[:, :tr.shape[1]].tolist()
    if not (chain_ok and tree_ok):
        raise RuntimeError(f"speculative output differs from target-only greedy (chain {chain_ok}, tree {tree_ok})")
    packed = dec.packed_bytes()

    # algorithmic bytes per generated token: packed words and fp32 scales of the
    # projections a step runs, the bf16 lm_head, and the bf16 KV read at the mean
    # sequence length of the run
    def step_bytes(d, branches):
        b = 0
        for ly in d.layers:
            for pr in ly["projs"]:
                for bi, br in enumerate(pr.branches):
                    if bi not in branches:
                        continue
                    if br.v_sign is not None:
                        b += (br.rank * pr.in_features + 7) // 8 + 4 * pr.in_features
                    b += (pr.out_features * br.rank + 7) // 8 + 4 * (br.rank + pr.out_features)
        kv_tok = 2 * shape.num_hidden_layers * shape.num_key_value_heads * shape.head_dim * 2
        return b + shape.vocab_size * shape.hidden_size * 2 + kv_tok * (args.prompt + n // 2)
    bpt_draft, bpt_target = step_bytes(dec, (0,)), step_bytes(dec, (0, 1))
    peak_gbs, _ = peaks()

    def frac(tps, bpt):
        return round(bpt * tps / ws / 1e9 / peak_gbs, 4)

    out = {
        "workload": f"Llama-2-7B shape (32 layers, hidden 4096, MLP 11008, vocab 32000), "
                    f"{args.prompt}-token random prompt, {n} greedy tokens, batch 1 per GPU",
        "unit": "tokens/s", "aggregate_over_gpus": ws,
        "draft_ranks_0p1bit": r_d, "residual_ranks_0p9bit": r_r, "residual_scale": args.res_scale,
        "target_packed_mb": round(packed / 1e6, 1),
        "draft_greedy": round(n * ws / t_draft, 2),
        "target_greedy": round(n * ws / t_ar, 2),
        "decode_only": {"draft_greedy": round((n - 1) * ws / (t_draft - t_draft1), 2),
                        "target_greedy": round((n - 1) * ws / (t_ar - t_ar1), 2),
                        "target_prefill_s": round(t_ar1, 4),
                        "method": "(n - 1) / (t(n tokens) - t(1 token)): prompt prefill excluded"},
        "spec_chain_gamma4": {"tokens_per_s": round(n * ws / t_sp, 2),
                              "acceptance_rate": round(sst["acceptance_rate"], 4),
                              "mean_acceptance_length": round(sst["mean_acceptance_length"], 3),
                              "num_steps": sst["num_steps"], "token_identical": chain_ok},
        "spec_tree_d4b2": {"tokens_per_s": round(n_tr * ws / t_tr, 2),
                           "acceptance_rate": round(tst["acceptance_rate"], 4),
                           "mean_acceptance_length": round(tst["mean_acceptance_length"], 3),
                           "num_steps": tst["num_steps"], "tokens": n_tr, "token_identical": tree_ok},
        "timing": "wall clock around each whole generate call (prompt prefill and host syncs included), "
                  "max over ranks",
    }
    out["bytes_per_token"] = {"draft": bpt_draft, "target": bpt_target,
                              "note": "packed words + fp32 scales + bf16 lm_head + bf16 KV at the mean length"}
    out["hbm_frac_per_gpu"] = {"draft_greedy": frac(out["decode_only"]["draft_greedy"], bpt_draft),
                               "target_greedy": frac(out["decode_only"]["target_greedy"], bpt_target)}
    out["weights"] = ("signs Bernoulli(0.5), scales |N(1,0.1)| times unit-gain constants (mid / sqrt(in), "
                      f"u1 / sqrt(rank)); residual u1 further x{args.res_scale}")
    del tgt, drf, draft_only, dec
    torch.cuda.empty_cache()

    # ---- BASELINE config 4 as stated: the target shares the packed draft
    # factors (littlespec_ref/littlebit_itq_spec.py:298-309): the residual of
    # every projection is a rank-matched U_R (own mid_R, u1_R) on the draft's
    # V-stage, so one V-stage feeds both U and U_R
    st = synthetic_runtime_state(shape, {k: [r_d[k], r_d[k]] for k in r_d}, seed=177 + rank,
                                 shared_residual=True, device=dev, unit_gain=True)
    for kk in list(st):
        if kk.endswith(".u1_r"):
            st[kk] = st[kk] * args.res_scale
    dec_s = LittleBitDecoder(shape, st, device=dev, max_seq=max_seq)
    del st
    tgt_s = CudaTargetModel.from_decoder(dec_s)
    drf_s = CudaDraftModel.from_target(tgt_s)
    autoregressive_generate(tgt_s, ids, None, max_new_tokens=8, eos_token_id=-1)
    speculative_decode(drf_s, tgt_s, ids, None, max_new_tokens=8, draft_length=4, eos_token_id=-1)
    speculative_decode_tree(drf_s, tgt_s, ids, None, max_new_tokens=8, tree_buffers=tb, top_k=2, eos_token_id=-1)
    (ar_s, _), t_ar_s = timed(lambda: autoregressive_generate(tgt_s, ids, None, max_new_tokens=n, eos_token_id=-1))
    _, t_ar1_s = timed(lambda: autoregressive_generate(tgt_s, ids, None, max_new_tokens=1, eos_token_id=-1))
    (sp_s, sst_s), t_sp_s = timed(lambda: speculative_decode(drf_s, tgt_s, ids, None, max_new_tokens=n,
                                                             draft_length=4, eos_token_id=-1))
    (tr_s, tst_s), t_tr_s = timed(lambda: speculative_decode_tree(drf_s, tgt_s, ids, None, max_new_tokens=n,
                                                                  tree_buffers=tb, top_k=2, eos_token_id=-1))
    n_tr_s = tr_s.shape[1] - ids.shape[1]
    ar_s_long = ar_s
    if n_tr_s > n:
        ar_s_long, _ = autoregressive_generate(tgt_s, ids, None, max_new_tokens=n_tr_s, eos_token_id=-1)
    ok_c = sp_s.tolist() == ar_s.tolist()
    ok_t = tr_s.tolist() == ar_s_long[:, :tr_s.shape[1]].tolist()
    if not (ok_c and ok_t):
        raise RuntimeError(f"shared-factor speculation differs from target-only greedy (chain {ok_c}, tree {ok_t})")
    out["c4_shared_target"] = {
        "workload": "config 4: 0.1-bit draft + rank-matched residual U_R sharing the draft's packed V "
                    "(one V-stage per projection feeds U and U_R), 7B shape, same prompt and length",
        "residual_ranks": r_d, "target_packed_mb": round(dec_s.packed_bytes() / 1e6, 1),
        "target_greedy": round(n * ws / t_ar_s, 2),
        "target_decode_only": round((n - 1) * ws / (t_ar_s - t_ar1_s), 2),
        "spec_chain_gamma4": {"tokens_per_s": round(n * ws / t_sp_s, 2),
                              "acceptance_rate": round(sst_s["acceptance_rate"], 4),
                              "mean_acceptance_length": round(sst_s["mean_acceptance_length"], 3),
                              "num_steps": sst_s["num_steps"], "token_identical": ok_c},
        "spec_tree_d4b2": {"tokens_per_s": round(n_tr_s * ws / t_tr_s, 2),
                           "acceptance_rate": round(tst_s["acceptance_rate"], 4),
                           "mean_acceptance_length": round(tst_s["mean_acceptance_length"], 3),
                           "num_steps": tst_s["num_steps"], "tokens": n_tr_s, "token_identical": ok_t},
    }
    del tgt_s, drf_s, dec_s
    torch.cuda.empty_cache()

    # ---- the reference's CPU decode ops on this box's host cores (rank 0, N=1)
    if ws == 1 and not args.no_cpu:
        out["cpu_reference"] = cpu_decode_reference(r_d, r_r, args.prompt)
    return out


def run_decode70b(args, dev, rank, ws):
    """Greedy and chain-speculative decode on the Llama-2-70B shape (BASELINE
    config 5): 0.1-bit draft + 0.9-bit residual target (~8.5 GB packed) on every
    GPU, one sequence per rank (data parallel), a 512-token random prompt."""
    from littlebit_b200.cuda_models import CudaDraftModel, CudaTargetModel
    from littlebit_b200.model import LLAMA2_70B, LittleBitDecoder, synthetic_runtime_state
    from littlebit_b200.speculative_decoding import autoregressive_generate, speculative_decode

    shape = LLAMA2_70B
    r_d, r_r = _ranks_at(shape, 0.1), _ranks_at(shape, 0.9)
    st = synthetic_runtime_state(shape, {k: [r_d[k], r_r[k]] for k in r_d}, seed=91 + rank, device=dev,
                                 unit_gain=True)
    for k in list(st):
        if k.endswith(".u1_r"):
            st[k] = st[k] * args.res_scale
    prompt, n = 512, args.new70
    dec = LittleBitDecoder(shape, st, device=dev, max_seq=prompt + n + 64)
    del st
    tgt = CudaTargetModel.from_decoder(dec)
    drf = CudaDraftModel.from_target(tgt)
    draft_only = CudaTargetModel.from_decoder(drf.dec)
    ids = torch.randint(0, shape.vocab_size, (1, prompt),
                        generator=torch.Generator().manual_seed(2000 + rank)).to(dev)

    def timed(fn):
        barrier(ws)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize()
        return out, max_over_ranks(time.perf_counter() - t0, ws)

    autoregressive_generate(draft_only, ids, None, max_new_tokens=4, eos_token_id=-1)
    autoregressive_generate(tgt, ids, None, max_new_tokens=4, eos_token_id=-1)
    speculative_decode(drf, tgt, ids, None, max_new_tokens=8, draft_length=4, eos_token_id=-1)
    (_, _), t_draft = timed(lambda: autoregressive_generate(draft_only, ids, None, max_new_tokens=n,
                                                             eos_token_id=-1))
    (ar, _), t_ar = timed(lambda: autoregressive_generate(tgt, ids, None, max_new_tokens=n, eos_token_id=-1))
    _, t_draft1 = timed(lambda: autoregressive_generate(draft_only, ids, None, max_new_tokens=1, eos_token_id=-1))
    _, t_ar1 = timed(lambda: autoregressive_generate(tgt, ids, None, max_new_tokens=1, eos_token_id=-1))
    (sp, sst), t_sp = timed(lambda: speculative_decode(drf, tgt, ids, None, max_new_tokens=n,
                                                       draft_length=4, eos_token_id=-1))
    if sp.tolist() != ar.tolist():
        raise RuntimeError("70B-shape chain speculation differs from target-only greedy")
    lm = shape.vocab_size * shape.hidden_size * 2
    kv = 2 * shape.num_hidden_layers * shape.num_key_value_heads * shape.head_dim * 2 * (prompt + n // 2)
    peak_gbs, _ = peaks()
    out = {"workload": f"Llama-2-70B shape (80 layers, hidden 8192, MLP 28672, 64/8 heads), "
                       f"{prompt}-token random prompt, {n} greedy tokens, one sequence per GPU",
           "unit": "tokens/s", "aggregate_over_gpus": ws,
           "target_packed_gb": round(dec.packed_bytes() / 1e9, 2),
           "draft_greedy": round(n * ws / t_draft, 2), "target_greedy": round(n * ws / t_ar, 2),
           "decode_only": {"draft_greedy": round((n - 1) * ws / (t_draft - t_draft1), 2),
                           "target_greedy": round((n - 1) * ws / (t_ar - t_ar1), 2),
                           "target_prefill_s": round(t_ar1, 4),
                           "method": "(n - 1) / (t(n tokens) - t(1 token)): prompt prefill excluded"},
           "timing": "wall clock around each whole generate call (prompt prefill included), max over ranks",
           "spec_chain_gamma4": {"tokens_per_s": round(n * ws / t_sp, 2),
                                 "acceptance_rate": round(sst["acceptance_rate"], 4),
                                 "mean_acceptance_length": round(sst["mean_acceptance_length"], 3),
                                 "token_identical": True},
           "lm_head_and_kv_bytes_per_token": lm + kv}
    out["target_hbm_frac_per_gpu"] = round((dec.packed_bytes() + dec.scale_bytes() + lm + kv)
                                           * out["decode_only"]["target_greedy"] / ws / 1e9
                                           / peak_gbs, 4)
    return out


def run_c5(args, dev, rank, ws):
    """BASELINE config 5 on the Llama-2-70B shape: 64 independent sequences split
    data-parallel over the ranks (64/N per GPU, the first 64 % N ranks one
    more when N does not divide 64), each GPU decoding its share as
    one batch (lbx_forward_multi: every packed-weight read serves all of its
    sequences).  0.1-bit draft + 0.9-bit residual target (per-layer residual),
    chain speculation with gamma 4 against batched target-only greedy decoding;
    every sequence's tokens must be identical between the two.  The 512-token
    prompt prefill is replaced by a seeded random bf16 KV prefix of 511 slots
    per sequence (the decode work per token depends only on the cached length;
    the draft's caches hold the same prefix)."""
    from littlebit_b200.batch_decode import BatchDecoder, greedy_generate, speculative_generate
    from littlebit_b200.cuda_models import _branch0_view
    from littlebit_b200.model import LLAMA2_70B, LittleBitDecoder, synthetic_runtime_state

    shape = LLAMA2_70B
    r_d, r_r = _ranks_at(shape, 0.1), _ranks_at(shape, 0.9)
    st = synthetic_runtime_state(shape, {k: [r_d[k], r_r[k]] for k in r_d}, seed=91, device=dev,
                                 unit_gain=True)
    for k in list(st):
        if k.endswith(".u1_r"):
            st[k] = st[k] * args.res_scale
    from littlebit_b200 import sharded

    S_total, gamma, P, G = 64, 4, 512, args.c5_new
    S = len(sharded.split_requests(S_total, ws, rank))  # (rank 0 holds the largest share)
    max_seq = P + (gamma + 1) * G + 16
    dec = LittleBitDecoder(shape, st, device=dev, max_seq=16)  # weights only (the batches own the caches)
    del st
    tgt = BatchDecoder(dec, S, max_seq)
    drf = BatchDecoder(_branch0_view(dec, 16), S, max_seq)
    tgt.fill_synthetic_prefix(P - 1, seed=3000 + rank)
    drf.copy_prefix_from(tgt, P - 1)
    g = torch.Generator().manual_seed(4000 + rank)
    last = torch.randint(0, shape.vocab_size, (S,), generator=g).to(dev)
    prev = torch.randint(0, shape.vocab_size, (S,), generator=g).to(dev)

    def timed(fn):
        barrier(ws)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = fn()
        torch.cuda.synchronize()
        return out, max_over_ranks(time.perf_counter() - t0, ws)

    # warm-up (kernel attributes, workspaces), then the timed runs
    greedy_generate(tgt, last, P - 1, 2)
    speculative_generate(drf, tgt, prev, last, P - 1, 2, gamma)
    greedy_generate(drf, last, P - 1, 2)
    greedy, t_g = timed(lambda: greedy_generate(tgt, last, P - 1, G))
    _, t_d = timed(lambda: greedy_generate(drf, last, P - 1, G))
    (spec, sst), t_s = timed(lambda: speculative_generate(drf, tgt, prev, last, P - 1, G, gamma))
    same = bool(torch.equal(spec, greedy))
    if not same:
        raise RuntimeError("C5 batched speculation differs from batched target-only greedy")
    lm = shape.vocab_size * shape.hidden_size * 2
    kv_tok = 2 * shape.num_hidden_layers * shape.num_key_value_heads * shape.head_dim * 2
    step_bytes = dec.packed_bytes() + dec.scale_bytes() + lm + S * kv_tok * (P + G // 2)
    peak_gbs, _ = peaks()
    tps_g = S_total * G / t_g
    return {"workload": f"Llama-2-70B shape, {S_total} independent sequences ({S} per GPU, one batch), "
                        f"{P}-token context (random bf16 KV prefix standing in for the prefill), {G} new "
                        f"tokens each, greedy",
            "unit": "tokens/s (all sequences, all GPUs)", "sequences_per_gpu": S,
            "target_packed_gb": round(dec.packed_bytes() / 1e9, 2),
            "target_greedy": round(tps_g, 2), "draft_greedy": round(S_total * G / t_d, 2),
            "spec_chain_gamma4": {"tokens_per_s": round(S_total * G / t_s, 2),
                                  "acceptance_rate": round(sst["acceptance_rate"], 4),
                                  "mean_acceptance_length": round(sst["mean_acceptance_length"], 3),
                                  "num_steps": sst["num_steps"], "token_identical": same},
            "target_step_ms": round(t_g / G * 1e3, 2),
            "target_hbm_frac_per_gpu": round(step_bytes * (G / t_g) / 1e9 / peak_gbs, 4),
            "bytes_per_target_step": step_bytes,
            "timing": "wall clock around each generate call, max over ranks; residual u1 x"
                      f"{args.res_scale}, unit-gain scales"}


# ---------------------------------------------------------------------------
# row-sharded 8192 -> 28672 LittleBitLinear (N > 1)
# ---------------------------------------------------------------------------
def run_row_shard(args, dev, rank, ws, reps: int = 200):
    """The 70B-MLP-shaped LittleBitLinear at this world size: U rows split over
    the ranks, V replicated, the y slices all-gathered, timed two ways — the
    local layer followed by an NCCL all-gather, and the all-gather fused into
    the U-stage (tagged NVLink stores + an unpack kernel; ``us_per_call``) —
    beside the whole layer on one GPU, at one token (the top-level keys) and
    at a 16-token verify batch (``k16``).  GB/s counts the whole layer's
    algorithmic bytes once per call."""
    import torch.distributed as dist
    from littlebit_b200 import synthetic
    from littlebit_b200 import ops
    from littlebit_b200.sharded import FusedRowShardedLinear, RowShardedLinear

    K, N, r = 8192, 28672, 616
    g = torch.Generator().manual_seed(4242)
    full = synthetic.to_packed_linear(K, N, synthetic.layer(K, N, [r], g), dev)
    sh = RowShardedLinear(full, ws, rank)
    fsh = FusedRowShardedLinear(full, ws, rank, max_tokens=16)
    stream = torch.cuda.current_stream(dev)
    per = 20  # calls per CUDA graph

    def timed(fn):
        """Device time per call: ``per`` calls captured in one CUDA graph (the
        Python launch cost of a call exceeds its GPU time), replayed."""
        for _ in range(4):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(per):
                fn()
        for _ in range(3):
            graph.replay()
        barrier(ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps // per):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        t = max_over_ranks(e0.elapsed_time(e1) / (reps // per * per) * 1e3, ws)
        del graph  # a graph holding NCCL calls goes before the process group
        return t

    def measure(k):
        x = torch.randn(k, K, generator=g).to(dev)
        part = sh.local_forward(x)
        gat = torch.empty(ws, k, N // ws, device=dev)
        t_local = timed(lambda: sh.local_forward(x, part))
        t_ag = timed(lambda: dist.all_gather_into_tensor(gat, part))
        t_all = timed(lambda: (sh.local_forward(x, part), dist.all_gather_into_tensor(gat, part)))
        # the all-gather fused into the U-stage; must agree with the NCCL path bitwise
        yf = torch.empty(k, N, device=dev)
        t_fused = timed(lambda: fsh.forward(x, yf))
        ref = gat.permute(1, 0, 2).reshape(k, N)
        same = bool(torch.equal(fsh.forward(x, yf), ref))
        # the whole layer on this GPU alone: the sharded result must be its bits
        yfull = torch.empty(k, N, device=dev)
        t_unsharded = timed(lambda: ops.linear_group([full], x, [yfull]))
        same_full = bool(torch.equal(yf, yfull))
        dev_err = ops.device_error(dev)
        if not same or not same_full or dev_err:
            raise RuntimeError(f"fused all-gather disagrees at k={k} (equal to NCCL {same}, to the unsharded "
                               f"layer {same_full}, device error {dev_err:#x})")
        alg = (r * K + 7) // 8 + (N * r + 7) // 8 + 4 * (K + r + N) + 4 * K * k + 4 * N * k
        return {"us_per_call": round(t_fused, 3), "local_kernel_us": round(t_local, 3),
                "nccl_us_per_call": round(t_all, 3), "nccl_allgather_us": round(t_ag, 3),
                "fused_us_per_call": round(t_fused, 3), "fused_equals_nccl": same,
                "fused_equals_unsharded": same_full, "unsharded_us_per_call": round(t_unsharded, 3),
                "exchange_us": round(t_fused - t_local, 3),
                "allgather_bytes_per_rank": 4 * N * k // ws,
                "gbs_whole_layer": round(alg / (t_fused * 1e-6) / 1e9, 2), "algorithmic_bytes": alg}

    k1 = measure(1)
    k16 = measure(16)
    fsh.close()
    return {"workload": f"LittleBitLinear {K}->{N} r={r}, fp32, U rows split over {ws} GPUs, "
                        f"V replicated, y all-gathered; k=1 (top level) and k=16 (k16)",
            **k1,
            "limiter": "the replicated V-stage and the stage launches: at one token the layer is latency-bound "
                       "(2.8 MB in ~10 us), so splitting its rows shortens only the U-stage body; at 16 tokens "
                       "the U-stage body is the larger part and shrinks with the rows",
            "k16": k16,
            "timing": f"CUDA events over {reps} calls ({per} per CUDA graph), max over ranks"}


def run_dense_ref(args, dev, rank, ws, P: int = 64):
    """The reference's own GPU path for the same layer, as its module computes it
    (littlebit.py:114-121 with the residual branch of 104-107): bf16 ±1 U and V
    unpacked to dense tensors, two cuBLAS GEMMs per branch.  A reported
    baseline: same chain-of-distinct-layers workload, CUDA-graph timed."""
    k = args.tokens
    g = torch.Generator(device=dev).manual_seed(7)
    sgn = lambda r, c: (torch.randint(0, 2, (r, c), generator=g, device=dev, dtype=torch.int8) * 2 - 1).bfloat16()
    sc = lambda n: (1 + 0.1 * torch.randn(n, generator=g, device=dev)).abs().bfloat16()
    layers = [[(sgn(r, IN_F), sc(IN_F), sc(r), sgn(OUT_F, r), sc(OUT_F)) for r in RANKS] for _ in range(P)]
    acts = [torch.randn(k, IN_F, generator=g, device=dev).bfloat16()] + \
           [torch.empty(k, OUT_F, device=dev, dtype=torch.bfloat16) for _ in range(P)]

    def step():
        for i in range(P):
            x = acts[i]
            y = None
            for V, v2, mid, U, u1 in layers[i]:
                yb = ((x * v2) @ V.t() * mid) @ U.t() * u1
                y = yb if y is None else y + yb
            acts[i + 1].copy_(y)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps / P * 1e3
    b, _ = layer_bytes(k)
    dense_bytes = sum(2 * r * (IN_F + OUT_F) for r in RANKS)
    del graph
    return {"workload": f"C2 layer as the reference's module runs it on GPU: bf16 dense ±1 U/V, "
                        f"two cuBLAS GEMMs per branch, k={k}, chain of {P} distinct layers",
            "us_per_layer": round(us, 3), "gbs_algorithmic": round(b / (us * 1e-6) / 1e9, 2),
            "dense_weight_bytes_per_layer": dense_bytes,
            "speedup_of_packed_kernels": None}


class Chain:
    """A chain of distinct layers, x_{i+1} = y_i, with its activation buffers and
    the prebuilt C-ABI arguments of every layer call."""

    def __init__(self, pool, k: int, dtype, dev, seed: int = 5):
        from littlebit_b200 import ops

        self.pool, self.k, self.dev = pool, k, dev
        g = torch.Generator(device=dev).manual_seed(seed)
        self.acts = [torch.randn(k, IN_F, device=dev, generator=g).to(dtype)] + \
                    [torch.empty(k, OUT_F, device=dev, dtype=dtype) for _ in pool]
        self.arrs = [ops.projs_array([p]) for p in pool]
        self.args = [ops.linear_args([pool[i]], self.acts[i], [self.acts[i + 1]]) for i in range(len(pool))]
        self.ws = torch.zeros(ops.linear_workspace_bytes([pool[0]], k), dtype=torch.uint8, device=dev)
        self.lib = ops.lib()

    def run(self, exec_mode: int, stream, use_pdl: int = 1):
        """Every layer through lbx_linear_verify (the C-ABI call), on ``stream``."""
        from littlebit_b200 import _lib as L

        fn, ws, n, st = self.lib.lbx_linear_verify, self.ws.data_ptr(), self.ws.numel(), stream.cuda_stream
        for arr, a in zip(self.arrs, self.args):
            a.exec = exec_mode
            a.use_pdl = use_pdl
            rc = fn(arr, ctypes.byref(a), ws, n, st)
            if rc:
                L.check(rc, "lbx_linear_verify")

    def floor(self, mode: int, stream):
        from littlebit_b200 import _lib as L

        for arr, a in zip(self.arrs, self.args):
            a.use_pdl = 1
            L.check(self.lib.lbx_linear_floor(arr, ctypes.byref(a), mode, self.ws.data_ptr(), self.ws.numel(),
                                              stream.cuda_stream), "lbx_linear_floor")


def timed_graph(fn, stream, warmup: int, steps: int, ws: int):
    """Device ms of ``steps`` replays of fn captured in one CUDA graph, after
    ``warmup`` replays, bracketed by barrier + synchronize; max over ranks."""
    from littlebit_b200 import ops

    with torch.cuda.stream(stream):
        fn()  # eager warm-up (kernel attributes, programs)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    ops.clear_device_error()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    out = max_over_ranks(e0.elapsed_time(e1), ws)
    del graph
    return out


def roofline_entry(b_layer: int, us: float, peak: float, peak_kind: str, traffic=None) -> dict:
    gbs = b_layer / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
            "frac": round(gbs / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": b_layer, "launch": "one LittleBit layer",
            "mean_launch_us": round(us, 3)}


def cpu_layer_gbs(k: int, ranks, shared: bool, esz: int, budget_s: float = 2.0, nlayers: int = 8):
    """The reference's CPU op (oracle/_ref littlebit_linear) on a config's layer:
    GB/s over a few distinct layers for about budget_s seconds (None when the
    op is not built or a branch shares its V, which the op cannot express)."""
    from oracle import build_ref  # CPU baseline only

    if shared or not build_ref.load():
        return None
    from littlebit_b200 import synthetic as syn

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(9)
    layers = [syn.layer(IN_F, OUT_F, list(ranks), g) for _ in range(nlayers)]
    op = torch.ops.littlebit_cpu_ops.littlebit_linear
    x = torch.randn(k, IN_F, generator=g)

    def one_pass():
        for lay in layers:
            for b in lay:
                op(x, b["v2"][None], b["v_sign"], IN_F, b["mid"][None], b["u_sign"], b["rank"], b["u1"][None])

    one_pass()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        one_pass()
        times.append(time.perf_counter() - t0)
    b, _ = layer_bytes(k, ranks, shared, esz)
    return {"value": round(b * nlayers / statistics.median(times) / 1e9, 3), "unit": "GB/s",
            "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"{len(times)} passes (median) over {nlayers} distinct layers, k={k}"}


def run_configs(args, dev, stream, ws, main_pool, peak, peak_kind):
    """The other BASELINE layer configs, each a chain of distinct layers timed
    like the headline (CUDA graph of the C-ABI calls, weights streamed from HBM),
    with the reference's CPU op on the same layer beside each (rank 0, N=1)."""
    from littlebit_b200 import _lib as L

    out = {}
    steps, warm = max(5, args.steps // 2), args.warmup

    def one(name, pool, k, dtype, ranks, shared, desc):
        from littlebit_b200 import ops

        ch = Chain(pool, k, dtype, dev)
        t_k = timed_graph(lambda: ch.run(L.LBX_EXEC_KERNELS, stream), stream, warm, steps, ws)
        y_k = ch.acts[-1].clone()
        t, exe = t_k, "two stage grids per layer"
        if k <= 8:  # the fused chain executor (same bits) when the call fits it
            fc = ops.FusedChain(pool)
            ptrs = (ctypes.c_void_p * (len(pool) + 1))(*[a.data_ptr() for a in ch.acts])
            t_f = timed_graph(lambda: fc.run(ch.acts, ptrs=ptrs, stream=stream), stream, warm, steps, ws)
            if not torch.equal(ch.acts[-1], y_k):
                raise RuntimeError(f"{name}: fused chain and stage grids disagree")
            if t_f < t_k:
                t, exe = t_f, ("fused chain (one launch per layer)" if k == 1 else
                               f"fused chain as two concurrent sub-chains of {(k + 1) // 2} and {k // 2} tokens "
                               f"(one launch per layer each)")
            del fc
        us = t * 1e3 / (steps * len(pool))
        b, packed = layer_bytes(k, ranks, shared, 4 if dtype == torch.float32 else 2)
        e = roofline_entry(b, us, peak, peak_kind)
        e.update({"exec": exe, "stage_grids_us": round(t_k * 1e3 / (steps * len(pool)), 3)})
        e.update({"workload": desc, "tokens": k, "pool_layers": len(pool),
                  "pool_mb": round(len(pool) * (b - (4 if dtype == torch.float32 else 2) * k * (IN_F + OUT_F)) / 1e6, 1),
                  "gbs_aggregate": round(b * len(pool) * steps * ws / (t * 1e-3) / 1e9, 2),
                  "finite": bool(torch.isfinite(ch.acts[-1].float()).all())})
        if ws == 1 and not args.no_cpu:
            e["cpu_baseline"] = cpu_layer_gbs(k, ranks, shared, 4 if dtype == torch.float32 else 2)
        out[name] = e
        del ch

    c1 = build_pool(1024, dev, seed=4321, ranks=[208])
    one("c1_k1", c1, 1, torch.float32, [208], False,
        "C1 4096->4096 r=208 (~0.1 BPW), fp32 x/y, k=1, chain of 1024 distinct layers (> 2x L2)")
    del c1
    for k in (5, 8):
        one(f"c2_k{k}", main_pool, k, torch.bfloat16, RANKS, False,
            f"C2 verify batch k={k}: r=208+1840 (independent V_R), bf16, chain of {len(main_pool)} layers")
    c4 = build_pool(768, dev, seed=8765, ranks=[208, 208], shared=True)
    for k in (1, 5):
        one(f"c4_shared_k{k}", c4, k, torch.bfloat16, [208, 208], True,
            f"config-4 shared-factor target layer: draft r=208 + rank-matched residual U_R on the draft's "
            f"V-stage (one V-stage feeds U and U_R), bf16, k={k}, chain of 768 layers")
    del c4
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    from littlebit_b200 import _lib as L
    from littlebit_b200 import ops

    rank, ws, lrank = dist_init()
    torch.cuda.set_device(lrank)
    dev = torch.device("cuda", lrank)
    k, P = args.tokens, args.pool
    pool = build_pool(P, dev, seed=1234 + rank)
    ch = Chain(pool, k, torch.bfloat16, dev)
    acts = ch.acts
    arr_all = ops.projs_array(pool)
    ptrs = (ctypes.c_void_p * (P + 1))(*[t.data_ptr() for t in acts])
    wsc = torch.zeros(int(ops.lib().lbx_linear_chain_workspace_size(arr_all, P, k)), dtype=torch.uint8,
                      device=dev)
    stream = torch.cuda.Stream(dev)

    def step_kernels():  # one V-stage + one U-stage grid per layer, chained with PDL
        ch.run(L.LBX_EXEC_KERNELS, stream, args.pdl)

    def step_cluster():  # one split-rank cluster launch per layer, chained with PDL
        ch.run(L.LBX_EXEC_CLUSTER, stream, args.pdl)

    def step_program():  # the whole chain as one persistent program
        ops.linear_chain(pool, acts, ws=wsc, arr=arr_all, ptrs=ptrs)

    fchain = ops.FusedChain(pool) if k <= 8 else None  # sign words copied once into its layout

    def step_fused():  # n + 1 launches: layer i's U-stage with layer i+1's V partials
        fchain.run(acts, ptrs=ptrs, stream=stream)

    execs = {"cluster": step_cluster, "kernels": step_kernels, "program": step_program}
    if fchain is not None:
        execs["fused"] = step_fused
    main_fn = execs[args.exec]
    sampler = ClockSampler(lrank)
    sampler.start()
    time.sleep(0.3)
    t_ms = timed_graph(main_fn, stream, args.warmup, args.steps, ws)
    clocks = sampler.stop()
    assert ops.device_error() == 0, "device error word set during the bench"
    if not torch.isfinite(acts[-1].float()).all():
        raise RuntimeError("non-finite output in the layer chain")
    if not float(acts[-1].float().abs().mean()) > 1e-3 * float(acts[0].float().abs().mean()):
        raise RuntimeError("the layer chain's activations collapsed to zero (the timing would skip work)")
    y_main = acts[-1].clone()
    # the other executors: timed the same way, and they must give the same bits
    exec_t = {}
    for name, fn in execs.items():
        if name == args.exec:
            continue
        if (name == "cluster" and k > 4) or (name == "fused" and k > 8):
            continue  # the cluster executor takes k <= 4, the fused chain k <= 8
        exec_t[name] = timed_graph(fn, stream, args.warmup, args.steps, ws)
        if not torch.equal(acts[-1], y_main):
            raise RuntimeError(f"{name} and {args.exec} executors disagree")

    b_layer, packed = layer_bytes(k)
    total_bytes = b_layer * P * args.steps * ws
    value = total_bytes / (t_ms * 1e-3) / 1e9
    exec_gbs = {n: round(total_bytes / (t_o * 1e-3) / 1e9, 2) for n, t_o in exec_t.items()}
    exec_gbs[args.exec] = round(value, 2)
    per_launch_s = t_ms * 1e-3 / (P * args.steps)
    peak, peak_kind = peaks()

    # ---- launch floor: the same grids and PDL chaining without arithmetic
    floor = {}
    for mode, nm in ((0, "launch_only_us"), (1, "with_weight_copies_us")):
        tf = timed_graph(lambda: ch.floor(mode, stream), stream, args.warmup, args.steps, ws)
        floor[nm] = round(tf * 1e3 / (P * args.steps), 3)
    floor["kernel_us"] = round(per_launch_s * 1e6, 3)
    floor["what"] = ("per-layer time of the same V/U grids (launch shapes, shared memory, PDL chaining) "
                     "doing no arithmetic (lbx_linear_floor): launches only, and with each unit's weight "
                     "bulk copies and their wait")

    # ---- e2e through the C ABI with host buffers, no graph captured here: every step
    # copies x from pinned host memory, makes the library call(s) of the
    # chain from the host (ctypes), and copies the last y back to pinned host
    # memory.  Two forms: the chain entry point (lbx_chain_fused, one call
    # per step, the default executor), and one lbx_linear_verify call per
    # layer (the reference's one-op-per-layer usage).
    hx = torch.empty(k, IN_F, dtype=torch.bfloat16).pin_memory()
    hx.copy_(acts[0].cpu())
    hy = torch.empty(k, OUT_F, dtype=torch.bfloat16).pin_memory()

    def e2e_time(run_chain):
        def e2e_step():
            with torch.cuda.stream(stream):
                acts[0].copy_(hx, non_blocking=True)
                run_chain()
                hy.copy_(acts[-1], non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier(ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_wall0 = time.perf_counter()
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        t_wall = time.perf_counter() - t_wall0
        t_dev = max_over_ranks(e0.elapsed_time(e1), ws)
        barrier(ws)
        return t_dev, t_wall

    if fchain is not None:
        t2, t_wall = e2e_time(step_fused)
        e2e_path = (f"pinned host x -> device; the host calls lbx_chain_fused (C ABI, ctypes) once for the "
                    f"{P}-layer chain (the library replays its cached graph of the call, built on the first "
                    f"call during warm-up); last y -> pinned host; every step")
    else:
        t2, t_wall = e2e_time(lambda: ch.run(L.LBX_EXEC_KERNELS, stream, args.pdl))
        e2e_path = (f"pinned host x -> device; the host calls lbx_linear_verify (C ABI, ctypes) for each of "
                    f"the {P} layers, no CUDA graph; last y -> pinned host; every step")
    e2e_val = b_layer * P * args.steps * ws / (t2 * 1e-3) / 1e9
    t3, t3_wall = e2e_time(lambda: ch.run(L.LBX_EXEC_KERNELS, stream, args.pdl))
    e2e_layer_val = b_layer * P * args.steps * ws / (t3 * 1e-3) / 1e9

    def e2e_graph_step():
        acts[0].copy_(hx, non_blocking=True)
        main_fn()
        hy.copy_(acts[-1], non_blocking=True)

    tg = timed_graph(e2e_graph_step, stream, args.warmup, args.steps, ws)
    e2e_graph_val = b_layer * P * args.steps * ws / (tg * 1e-3) / 1e9

    # ---- the other layer configs
    configs = run_configs(args, dev, stream, ws, pool, peak, peak_kind) if args.configs else None

    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    if ws == 1 and not args.no_cpu:
        r = cpu_reference(k, budget_s=args.cpu_seconds, nlayers=P)
        if r is not None:
            cpu = {"value": round(r["gbs"], 4), "unit": "GB/s", "cores": r["threads"],
                   "kind": "reference", "sample": r["sample"]}
        else:
            cpu = {"value": None, "unavailable": "the reference's C++ op is not built (oracle/_ref is missing: "
                                                 "run __graft_entry__.build() where the reference sources are)"}

    dense = run_dense_ref(args, dev, rank, ws) if args.dense_ref and ws == 1 else None
    if dense:
        dense["speedup_of_packed_kernels"] = round(dense["us_per_layer"] / (per_launch_s * 1e6), 2)
    decode = run_decode(args, dev, rank, ws) if args.decode else None
    decode70 = run_decode70b(args, dev, rank, ws) if args.decode70b else None
    c5 = run_c5(args, dev, rank, ws) if args.c5 else None
    row_shard = run_row_shard(args, dev, rank, ws) if ws > 1 else None

    if rank == 0:
        traffic = traffic_from_profiles(k, args.exec)
        roof = roofline_entry(b_layer, per_launch_s * 1e6, peak, peak_kind, traffic)
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "s8 digits x packed sign bits, int32 acc (bf16 in/out)", "data": "synthetic",
            "config": {"workload": f"C2 4096->4096 LittleBitLinear r={RANKS[0]}+{RANKS[1]} (independent "
                                   f"V_R), k={k} bf16 tokens, chain of {P} distinct layers per step",
                       "tokens": k, "pool_layers": P,
                       "pool_mb": round(P * (packed + sum(4 * (IN_F + r + OUT_F) for r in RANKS)) / 1e6, 1),
                       "l2": "weight pool > 2x L2 (126 MB): no flush needed",
                       "scales": "|N(1,0.1)|; mid / sqrt(in), u1 / sqrt(rank x branches) (unit gain: the "
                                 "128-layer chain's activations stay finite, so the executors' outputs are "
                                 "compared bit for bit)",
                       "parallelism": f"dp{ws} (independent replicas)",
                       "exec": {"program": "one persistent cooperative program per step (lbx_linear_chain)",
                                "kernels": "two kernels per layer (V-stage, U-stage grids), PDL-chained",
                                "cluster": "one split-rank cluster launch per layer (16-CTA clusters), "
                                           "PDL-chained",
                                "fused": "one launch per layer (8-CTA clusters per 256 rows): layer i's "
                                         "U-stage with layer i+1's V-stage partials, PDL-chained "
                                         "(lbx_chain_fused)"}[args.exec]},
            "roofline": roof,
            "exec_gbs": exec_gbs,
            "floor": floor,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": 2 * k * IN_F, "d2h_bytes_per_step": 2 * k * OUT_F,
                    "ms_per_step": round(t2 / args.steps, 4),
                    "host_wall_ms_per_step": round(t_wall * 1e3 / args.steps, 4), "path": e2e_path},
            "e2e_per_layer_calls": {
                "value": round(e2e_layer_val, 2), "unit": "GB/s", "ms_per_step": round(t3 / args.steps, 4),
                "host_wall_ms_per_step": round(t3_wall * 1e3 / args.steps, 4),
                "path": f"the same copies; the host calls lbx_linear_verify (C ABI, ctypes) for each of the {P} "
                        f"layers (two stage grids per call), no CUDA graph"},
            "e2e_graph": {"value": round(e2e_graph_val, 2), "unit": "GB/s",
                          "ms_per_step": round(tg / args.steps, 4),
                          "path": "the same step (copies + chain) captured in one CUDA graph"},
            "configs": configs,
            "cpu_baseline": cpu,
            "dense_bf16_ref": dense,
            "decode": decode,
            "decode_70b": decode70,
            "c5_70b_dp": c5,
            "row_shard": row_shard,
            "gpu_launches": {"program": 1, "kernels": 2 * P, "cluster": P, "fused": P + 1}[args.exec] * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(out))
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--pool", type=int, default=128)
    ap.add_argument("--pdl", type=int, default=1)
    ap.add_argument("--exec", default="fused", choices=["kernels", "cluster", "program", "fused"],
                    help="cluster: one split-rank cluster launch per layer; kernels: one grid per stage; "
                         "program: each step is one persistent launch")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--configs", type=int, default=1, help="also time C1, C2 k=5/8 and the config-4 layer")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--decode", type=int, default=1, help="also run the 7B-shape decode section")
    ap.add_argument("--decode70b", type=int, default=0,
                    help="also run the 70B-shape decode section (about a minute more)")
    ap.add_argument("--new70", type=int, default=32, help="tokens generated in the 70B section")
    ap.add_argument("--c5", type=int, default=1, help="BASELINE config 5: 64 sequences of the 70B shape, "
                                                      "data-parallel over the ranks, batched per GPU")
    ap.add_argument("--c5-new", type=int, default=32, help="tokens generated per sequence in config 5")
    ap.add_argument("--dense-ref", type=int, default=1,
                    help="also time the reference's GPU path (bf16 dense GEMMs) on the same layer")
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--res-scale", type=float, default=0.02)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
