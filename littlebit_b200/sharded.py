"""Multi-GPU pieces of the path: rank plumbing for data-parallel replicas and a
row-sharded LittleBitLinear.

Data parallel (the path's natural partition): every rank holds a full model
replica and decodes its own requests; no collective touches the data path.
Ranks meet only at the timing barriers and the max-over-ranks reduction.

Row sharding (the demonstration for one wide layer, e.g. 8192 -> 28672 at rank
616): rank g holds rows [g*N/G, (g+1)*N/G) of U (and of g, the u1 scale) and a
full copy of V, h and l.  Each rank runs the V-stage on the whole rank-r
latent (identical on every rank), its U-stage on its rows, then one all-gather
of the y slices.  The V-stage is replicated instead of split so that the only
exchange is that all-gather of k*N/G values per rank.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional, Sequence, Tuple

import torch

from .ops import Branch, PackedLinear, linear_group


# ---------------------------------------------------------------------------
# rank plumbing
# ---------------------------------------------------------------------------
def init_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment; initialises
    the process group (short timeout) when world_size > 1."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import torch.distributed as dist

        if not dist.is_initialized():
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
        return dist.get_rank(), ws, int(os.environ.get("LOCAL_RANK", "0"))
    return 0, 1, 0


def barrier(world_size: int) -> None:
    if world_size > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world_size: int, device="cpu") -> float:
    """The slowest rank's value (device timings are reported as the max)."""
    if world_size == 1:
        return float(v)
    import torch.distributed as dist

    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v: float, world_size: int, device="cpu") -> float:
    if world_size == 1:
        return float(v)
    import torch.distributed as dist

    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def split_requests(n_requests: int, world_size: int, rank: int) -> range:
    """Contiguous share of n independent requests for this rank (data parallel);
    the first n % G ranks take one more."""
    base, extra = divmod(n_requests, world_size)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


# ---------------------------------------------------------------------------
# row sharding
# ---------------------------------------------------------------------------
def shard_rows(out_features: int, world_size: int, rank: int, align: int = 16) -> Tuple[int, int]:
    """[lo, hi) output rows of this rank: equal shares, each a multiple of
    ``align`` (the U-stage tile height)."""
    if out_features % (world_size * align):
        raise ValueError(f"out_features {out_features} must split into {world_size} shares of a multiple "
                         f"of {align}")
    per = out_features // world_size
    return rank * per, (rank + 1) * per


def shard_branch(br: Branch, lo: int, hi: int) -> Branch:
    """This rank's view of a branch: U rows and u1 entries [lo, hi), V/h/l whole."""
    return Branch(br.v_sign, br.v2, br.mid, br.u_sign[lo:hi].contiguous(), br.u1[lo:hi].contiguous(), br.rank)


def assemble_rows(parts: Sequence[torch.Tensor]) -> torch.Tensor:
    """[k, N/G] slices of ranks 0..G-1 -> [k, N]."""
    return torch.cat(list(parts), dim=-1)


class RowShardedLinear:
    """LittleBitLinear with U's rows split over the ranks of a process group."""

    def __init__(self, full: PackedLinear, world_size: int, rank: int, group=None):
        self.world_size, self.rank, self.group = world_size, rank, group
        self.in_features, self.out_features = full.in_features, full.out_features
        self.lo, self.hi = shard_rows(full.out_features, world_size, rank)
        bias = None if full.bias is None else full.bias[self.lo:self.hi].contiguous()
        self.local = PackedLinear(full.in_features, self.hi - self.lo,
                                  [shard_branch(b, self.lo, self.hi) for b in full.branches], bias)
        self._gather: Optional[torch.Tensor] = None

    def local_forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        k = x.shape[0]
        if out is None:
            out = torch.empty(k, self.hi - self.lo, dtype=torch.float32, device=x.device)
        linear_group([self.local], x, [out])
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """y [k, N] on every rank: local U rows, then an NCCL all-gather."""
        import torch.distributed as dist

        k = x.shape[0]
        part = self.local_forward(x)
        if self.world_size == 1:
            return part
        if self._gather is None or self._gather.shape != (self.world_size, k, self.hi - self.lo):
            self._gather = torch.empty(self.world_size, k, self.hi - self.lo, dtype=part.dtype,
                                       device=part.device)
        dist.all_gather_into_tensor(self._gather, part, group=self.group)
        return self._gather.permute(1, 0, 2).reshape(k, self.out_features)


class FusedRowShardedLinear(RowShardedLinear):
    """Row-sharded LittleBitLinear with the all-gather fused into the U-stage
    (lbx_linear_allgather + lbx_allgather_unpack).

    Each rank's U-stage stores every result straight into every rank's
    exchange buffer over NVLink, as an 8-byte word tagged with the call
    number; the unpack kernel polls its own buffer until every word of the
    call has arrived and writes the plain fp32 y.  No fence, signal or
    collective launch sits between the layer and its consumer.

    The exchange buffers are torch symmetric memory (CUDA backend): two
    halves of [max_tokens, N] words per rank, used by alternate calls.  A
    rank rewrites half h two calls later, after its own unpack of the call in
    between, which needs every peer's U-stage of that call, which each peer's
    stream runs after its unpack of the call that used h — so the ordering is
    automatic as long as every rank makes the same sequence of calls on one
    stream."""

    def __init__(self, full: PackedLinear, world_size: int, rank: int, group=None,
                 max_tokens: int = 16):
        super().__init__(full, world_size, rank, group)
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        from . import _lib as L
        from .ops import lib, projs_array

        if not 1 <= max_tokens <= L.LBX_MAX_TOKENS:
            raise ValueError(f"max_tokens must be in [1, {L.LBX_MAX_TOKENS}]")
        if world_size > 8:
            raise ValueError("at most 8 ranks")
        self._L, self._lib, self._ct = L, lib(), ctypes
        dev = self.local.device
        pg = group if group is not None else dist.group.WORLD
        self.max_tokens = max_tokens
        self.half = max_tokens * self.out_features  # words per half
        if symm.get_backend(dev) is None:
            symm.set_backend("CUDA")
        self.xbuf = symm.empty(2 * self.half, dtype=torch.int64, device=dev)
        self.xbuf.zero_()
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        self.hdl = symm.rendezvous(self.xbuf, pg)
        self._peers = (ctypes.c_void_p * world_size)(*[int(p) for p in self.hdl.buffer_ptrs])
        self._arr = projs_array([self.local])
        self._ws = torch.zeros(int(self._lib.lbx_linear_workspace_size(self._arr, 1, max_tokens)),
                               dtype=torch.uint8, device=dev)
        # every rank's buffer is zero before any peer writes into it
        dist.barrier(group=pg)
        torch.cuda.synchronize(dev)

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y [k, N] fp32 on every rank (``out`` if given)."""
        from .ops import _cuda, _dt, _stream

        L, ct = self._L, self._ct
        _cuda("x", x)
        k = x.shape[0]
        if k > self.max_tokens or x.shape[1] != self.in_features:
            raise RuntimeError(f"x {tuple(x.shape)}: at most {self.max_tokens} rows of {self.in_features}")
        N = self.out_features
        if out is None:
            out = torch.empty(k, N, dtype=torch.float32, device=x.device)
        elif out.dtype != torch.float32 or out.shape != (k, N) or out.stride(1) != 1:
            raise RuntimeError(f"out must be float32 [{k}, {N}] with unit column stride")
        a = L.LinearArgs()
        a.n_proj = 1
        a.n_tokens = k
        a.x_dtype = _dt(x)
        a.y_dtype = L.LBX_F32
        a.prologue = L.LBX_PRO_NONE
        a.epilogue = L.LBX_EPI_STORE
        a.use_pdl = 1
        a.x = x.data_ptr()
        st = _stream(x.device)
        L.check(self._lib.lbx_linear_allgather(
            self._arr, ct.byref(a), self.world_size, self._peers, self.half, self.lo, N,
            self.state.data_ptr(), self._ws.data_ptr(), self._ws.numel(), st), "linear_allgather")
        L.check(self._lib.lbx_allgather_unpack(self.xbuf.data_ptr(), self.half, k, N, N, out.data_ptr(),
                                               out.stride(0), self.state.data_ptr(), 1, st),
                "allgather_unpack")
        return out

    def close(self) -> None:
        """Release the symmetric-memory handle (call on every rank)."""
        torch.cuda.synchronize(self.local.device)
        self.hdl = None
        self.xbuf = None
