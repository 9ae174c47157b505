"""Expert parallelism over torch.distributed, one process per GPU.

Rank g of G holds experts [g*E/G, (g+1)*E/G) of every layer (a MoeLayer created with
ep_rank=g, ep_world=G).  The input rows are on every rank (the router is replicated, so every
rank knows every job's expert); each rank runs the jobs of its own experts
(umsx_moe_forward_jobs), then one all-to-all moves every job's output row to the rank that owns
the token (contiguous token blocks), and that rank combines its tokens in rank order
(umsx_combine).  Every output row is computed by the same kernels from the same inputs as on one
GPU, so the result has the single-GPU layer's bits.  The exchange plan needs no count exchange:
it follows from the routing, which all ranks share.

The reference (appatalks/unified-memory-scheduler) runs a layer on one GPU (plus the host); this
module is the multi-GPU extension of its layer call (`ExpertPlan::execute`,
tools/engine/expert_dispatch.cpp:22-89, whose combine loop :77-87 is the per-token rank-order sum
done here on the token's rank).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def token_range(tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Tokens [t0, t1) that `rank` combines: contiguous blocks, the first tokens % world ranks one longer."""
    base, extra = divmod(tokens, world)
    t0 = rank * base + min(rank, extra)
    return t0, t0 + base + (1 if rank < extra else 0)


def token_ranks(tokens: int, world: int) -> torch.Tensor:
    """Rank that combines each token (the inverse of token_range)."""
    owner = torch.empty(tokens, dtype=torch.int64)
    for r in range(world):
        t0, t1 = token_range(tokens, world, r)
        owner[t0:t1] = r
    return owner


def plan_exchange(ids: torch.Tensor, experts: int, world: int, rank: int):
    """The all-to-all of one layer for `rank`, from the routing ids [T, k] shared by all ranks.

    Returns (send_jobs, send_sizes, recv_jobs, recv_sizes): send_jobs are the job indices t*k + r
    whose expert is on this rank, grouped by destination rank (the token's rank), ascending within
    a group; recv_jobs are the job indices of this rank's tokens grouped by source rank (the
    expert's rank), ascending within a group, which is the order the rows arrive in."""
    T, K = ids.shape
    per = experts // world
    owner = ids.to("cpu", torch.int64).reshape(-1) // per
    dest = token_ranks(T, world).repeat_interleave(K)
    jobs = torch.arange(T * K)
    mine = owner == rank
    send = [jobs[mine & (dest == d)] for d in range(world)]
    recv = [jobs[(dest == rank) & (owner == s)] for s in range(world)]
    return (torch.cat(send), [int(a.numel()) for a in send], torch.cat(recv), [int(a.numel()) for a in recv])


def exchange(y: torch.Tensor, ids: torch.Tensor, experts: int, group=None) -> tuple[torch.Tensor, tuple[int, int]]:
    """y [T, k, H]: this rank's job outputs (rows of its experts' jobs valid).  Returns the
    complete job outputs of this rank's tokens, [t1 - t0, k, H], and (t0, t1)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    T, K, H = y.shape
    send_jobs, send_sizes, recv_jobs, recv_sizes = plan_exchange(ids, experts, world, rank)
    dev = y.device
    send = y.reshape(T * K, H).index_select(0, send_jobs.to(dev))
    recv = torch.empty((sum(recv_sizes), H), dtype=y.dtype, device=dev)
    dist.all_to_all_single(recv, send, recv_sizes, send_sizes, group=group)
    t0, t1 = token_range(T, world, rank)
    mine = torch.empty(((t1 - t0) * K, H), dtype=y.dtype, device=dev)
    mine.index_copy_(0, (recv_jobs - t0 * K).to(dev), recv)
    return mine.reshape(t1 - t0, K, H), (t0, t1)


class ExpertParallelLayer:
    """One MoE layer split over the ranks of `group` by expert (see the module docstring)."""

    def __init__(self, layer, group=None):
        self.layer = layer
        self.group = group
        d = layer.desc
        if d.ep_world != dist.get_world_size(group) or d.ep_rank != dist.get_rank(group):
            raise ValueError("the layer's ep_rank / ep_world must match the process group")

    def forward(self, x: torch.Tensor, y: torch.Tensor | None = None, stream=None):
        """x [T, H] on this rank's GPU, the same rows on every rank; y: optional [T, k, H] f32
        scratch for the job outputs (reused across calls: only this rank's rows are read).
        stream: a torch.cuda.Stream (or None for the current stream); every step of the layer --
        the expert kernels, the host read of the routing, the torch index copies, the all-to-all
        and the combine -- is ordered on it, so x must be ready on it and the result is ready on it.
        Returns (out [t1 - t0, H] f32 for this rank's tokens, (t0, t1))."""
        from .umsx import combine
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        with torch.cuda.stream(s):
            y, ids, w = self.layer.forward_jobs(x, y=y, stream=s)
            mine, (t0, t1) = exchange(y, ids, self.layer.desc.experts, self.group)
            if t1 == t0:  # fewer tokens than ranks: nothing to combine here
                return torch.empty((0, self.layer.desc.hidden), dtype=torch.float32, device=x.device), (t0, t1)
            out = combine(mine, w[t0:t1].contiguous(), stream=s)
        return out, (t0, t1)


# ---- decode over NVLink: the exchange inside the kernels ----------------------------------------

IPC_HANDLE_BYTES = 64


class EpGroup:
    """This rank's exchange buffer, mapped into every other rank's process (umsx_ep_*).  The IPC
    handles travel once, at set-up, over the process group (all_gather_object); after that the
    decode steps exchange rows by P2P stores from inside the kernels, with no collective call."""

    def __init__(self, hidden: int, top_k: int, device: int, group=None, wait_limit_cycles: int | None = None):
        import ctypes as C

        from .umsx import check, lib
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self._h = C.c_void_p()
        L = lib()
        check(L.umsx_ep_create(self.rank, self.world, device, hidden, top_k, C.byref(self._h)))
        mine = (C.c_uint8 * IPC_HANDLE_BYTES)()
        check(L.umsx_ep_handle(self._h, mine, IPC_HANDLE_BYTES))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(mine), group=group)
        buf = (C.c_uint8 * (IPC_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        check(L.umsx_ep_connect(self._h, buf, IPC_HANDLE_BYTES * self.world))
        if wait_limit_cycles:
            check(L.umsx_ep_set_wait(self._h, int(wait_limit_cycles)))
        dist.barrier(group=group)  # every rank is mapped before any step stores into a peer

    def close(self):
        from .umsx import lib
        if self._h:
            lib().umsx_ep_destroy(self._h)
            self._h = None


class EpStack:
    """A decode stack split over the group by expert: h <- h + MoE_l(RMSNorm(h)) for one token per
    rank (token g on rank g), each layer a handle created with ep_rank / ep_world of the group.
    With up to four ranks and MXFP4 layers with fused gate_up a step is one kernel launch per rank
    (the exchanges happen inside it); otherwise the per-stage kernels run between two exchange
    kernels per layer.  Every rank must step in turn."""

    def __init__(self, group: EpGroup, layers: list, rms_eps: float = 1e-5):
        import ctypes as C

        from .umsx import check, lib
        self.group, self.layers = group, list(layers)
        self.hidden = self.layers[0].desc.hidden
        arr = (C.c_void_p * len(self.layers))(*[l._h for l in self.layers])
        self._h = C.c_void_p()
        check(lib().umsx_ep_stack_create(group._h, arr, len(self.layers), rms_eps, C.byref(self._h)))

    def forward(self, x, out=None, stream=None):
        """x: this rank's token [1, H] (CUDA, f32 or bf16) -> out [1, H] f32."""
        from .umsx import _dtype_code, _ptr, _stream, check, lib
        out = out if out is not None else torch.empty((1, self.hidden), dtype=torch.float32, device=x.device)
        check(lib().umsx_ep_stack_forward(self._h, _ptr(x), _dtype_code(x), _ptr(out), _stream(stream)))
        return out

    def forward_host(self, x_host, out_host, stream=None):
        from .umsx import _dtype_code, _ptr, _stream, check, lib
        check(lib().umsx_ep_stack_forward_host(self._h, _ptr(x_host), _dtype_code(x_host), _ptr(out_host),
                                               _stream(stream)))
        return out_host

    def status(self, stream=None):
        from .umsx import _stream, check, lib
        check(lib().umsx_ep_stack_status(self._h, _stream(stream)))

    def close(self):
        from .umsx import lib
        if self._h:
            lib().umsx_ep_stack_destroy(self._h)
            self._h = None


# ---- prefill over NVLink: tokens sharded over the ranks, rows exchanged inside the kernels -------

class EpPrefill:
    """A prefill stack split over the group by expert, every rank with its own tokens (umsx_ep_prefill_*):
    per layer the token rows travel to the ranks that hold their experts and the outputs come back,
    both as P2P stores from inside the exchange kernels.  The receive buffers' IPC handles travel
    once, at set-up, over the process group."""

    def __init__(self, group: EpGroup, layers: list, max_tokens: int, rms_eps: float = 1e-5, pg=None):
        import ctypes as C

        from .umsx import check, lib
        self.group, self.layers = group, list(layers)
        self.hidden = self.layers[0].desc.hidden
        L = lib()
        arr = (C.c_void_p * len(self.layers))(*[l._h for l in self.layers])
        self._h = C.c_void_p()
        check(L.umsx_ep_prefill_create(group._h, arr, len(self.layers), int(max_tokens), rms_eps, C.byref(self._h)))
        mine = (C.c_uint8 * IPC_HANDLE_BYTES)()
        check(L.umsx_ep_prefill_handle(self._h, mine, IPC_HANDLE_BYTES))
        handles = [None] * group.world
        dist.all_gather_object(handles, bytes(mine), group=pg)
        buf = (C.c_uint8 * (IPC_HANDLE_BYTES * group.world)).from_buffer_copy(b"".join(handles))
        check(L.umsx_ep_prefill_connect(self._h, buf, IPC_HANDLE_BYTES * group.world))
        dist.barrier(group=pg)  # every rank is mapped before any layer stores into a peer

    def forward(self, x, out=None, stream=None):
        """x: this rank's tokens [T, H] (CUDA, f32 or bf16) -> out [T, H] f32."""
        from .umsx import _dtype_code, _ptr, _stream, check, lib
        T = x.shape[0]
        out = out if out is not None else torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        check(lib().umsx_ep_prefill_forward(self._h, _ptr(x), _dtype_code(x), T, _ptr(out), _stream(stream)))
        return out

    def forward_host(self, x_host, out_host, stream=None):
        from .umsx import _dtype_code, _ptr, _stream, check, lib
        check(lib().umsx_ep_prefill_forward_host(self._h, _ptr(x_host), _dtype_code(x_host), x_host.shape[0],
                                                 _ptr(out_host), _stream(stream)))
        return out_host

    def loads(self):
        """Per layer of the last call: (rows received, expert jobs run) on this rank, int32 [layers, 2]."""
        import ctypes as C

        import numpy as np

        from .umsx import check, lib
        a = np.zeros((len(self.layers), 2), dtype=np.int32)
        check(lib().umsx_ep_prefill_loads(self._h, C.c_void_p(a.ctypes.data), a.size))
        return a

    def status(self, stream=None):
        from .umsx import _stream, check, lib
        check(lib().umsx_ep_prefill_status(self._h, _stream(stream)))

    def close(self):
        from .umsx import lib
        if self._h:
            lib().umsx_ep_prefill_destroy(self._h)
            self._h = None
