"""Expert parallelism for the MoE block, one process per GPU.

Mirrors the reference's EP module (engine/runtime/ep.py):

* ``init_ep(world_size, rank, local_rank)`` -- NCCL process group
  (ep.py:43-75), MASTER_ADDR defaulting to 127.0.0.1;
* ``expert_range(num_experts, rank, world_size)`` -- the same contiguous
  ``rank * n // world_size`` split (ep.py:78-86);
* ``patch_moe_for_ep(model, rank, world_size)`` -- installs the EP forward on
  every ``Qwen3_5MoeSparseMoeBlock`` of a model (ep.py:148-178; the reference
  looks for ``Qwen3NextSparseMoeBlock``, which the Qwen3.5 block does not
  subclass, so its patch never applied).

Semantics follow ``ep_forward`` (ep.py:97-143): tokens are replicated, every
rank routes all of them, computes only its experts, and the partial outputs
are summed.  Two ways to sum:

* ``fused`` (decode batches, T <= 64): the down-projection epilogue stores
  each weighted expert row straight into every rank's exchange buffer over
  NVLink (CUDA IPC-mapped), raises per-rank completion flags, and the
  combine waits on them (bounded) and sums locally -- every rank ends with the
  full output and no collective kernel runs;
  Prefill-sized batches use the row split: the down GEMM stores each row at
  the rank owning its token over NVLink, that rank combines its token slice
  and pushes it to every rank (``pmoe_block_forward_rows_fused``).  Both
  exchanges are registered with a native communicator (``pmoe_comm_create``),
  which picks the path by T and keeps the row exchange's epoch; its handle is
  the ``comm_handle`` of ``torch.ops.paris_moe.moe_block``, the call the
  patched HF module makes (``EPGroup.op_forward``);
* ``nccl`` (the comparator): each rank returns its partial (its experts plus
  its share of the shared expert's tokens) and ``torch.distributed.all_reduce``
  sums them, as ep.py:140 does; ``a2a``: token dispatch with all_to_all_single.

A peer that never arrives makes the kernels' bounded waits give up (about a
second) and set a sticky status word in this rank's exchange buffer instead
of hanging; ``EPGroup`` reads it asynchronously after every exchange call and
raises ``PmoeError(PMOE_ERR_PEER_TIMEOUT)`` at the next call, at ``check()``
and at ``close()`` (the reference's ep_forward relies on NCCL's error path).
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib

_BF16 = torch.bfloat16
FUSED_MAX_T = 64


def init_ep(world_size: int, rank: int, local_rank: int | None = None):
    """NCCL process group for EP (idempotent); returns (rank, world_size)."""
    if world_size <= 1:
        return 0, 1
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    if local_rank is None:
        local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        dist.init_process_group("nccl", world_size=world_size, rank=rank)
    return rank, world_size


def expert_range(num_experts: int, rank: int, world_size: int):
    """Contiguous experts [lo, hi) owned by ``rank`` (ep.py:78-86)."""
    return rank * num_experts // world_size, (rank + 1) * num_experts // world_size


def token_range(num_tokens: int, rank: int, world_size: int):
    """Tokens [lo, hi) whose shared-expert rows ``rank`` computes."""
    return rank * num_tokens // world_size, (rank + 1) * num_tokens // world_size


def expert_owner(idx: torch.Tensor, num_experts: int, world_size: int) -> torch.Tensor:
    """Rank owning each expert id under the contiguous ranges of expert_range."""
    bounds = torch.tensor([r * num_experts // world_size for r in range(world_size)],
                          dtype=torch.long, device=idx.device)
    return torch.searchsorted(bounds, idx.long(), right=True) - 1


def a2a_plan(idx: torch.Tensor, num_experts: int, world_size: int):
    """Token-dispatch send plan for local tokens routed as ``idx`` [Tl, K]: each
    token goes once to every rank owning at least one of its experts.  Returns
    (send_tok [S] local token ids grouped by destination rank ascending,
    counts [world] tokens per destination rank)."""
    owners = expert_owner(idx, num_experts, world_size)            # [Tl, K]
    hit = torch.zeros((idx.shape[0], world_size), dtype=torch.bool, device=idx.device)
    hit.scatter_(1, owners, True)
    toks = [torch.nonzero(hit[:, r], as_tuple=False).flatten() for r in range(world_size)]
    counts = torch.tensor([t.numel() for t in toks], dtype=torch.long)
    send = torch.cat(toks) if toks else torch.empty(0, dtype=torch.long, device=idx.device)
    return send, counts


def exchange_handles(local: bytes, group=None) -> list[bytes]:
    """All ranks' 64-byte IPC handles, indexed by rank (host collective)."""
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, local, group=group)
    return out


class EPGroup:
    """One rank's state for expert-parallel MoE calls.

    ``mode`` is "fused" (T <= t_max: NVLink exchange inside the kernels;
    beyond: row-split expert GEMMs + NVLink all-reduce) or
    "nccl" (contiguous expert ranges, replicated routing, partials summed with
    all_reduce: the reference's ep_forward, the comparator) or "a2a" (token
    dispatch with all_to_all_single: the second comparator)."""

    def __init__(self, num_experts: int, hidden: int, top_k: int, mode: str = "fused",
                 t_max: int = FUSED_MAX_T, group=None):
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        self._init_state(num_experts, hidden, top_k, mode, rank, world, group)
        if mode == "fused" and self.world > 1:
            nbytes = ctypes.c_size_t(0)
            _lib.check("pmoe_ep_buffer_bytes",
                       self.lib.pmoe_ep_buffer_bytes(t_max, hidden, top_k, ctypes.byref(nbytes)))
            self.buf_bytes = int(nbytes.value)
            ptr = ctypes.c_void_p()
            _lib.check("pmoe_ipc_alloc", self.lib.pmoe_ipc_alloc(self.buf_bytes, ctypes.byref(ptr)))
            self.local_buf = ptr.value
            h = ctypes.create_string_buffer(64)
            _lib.check("pmoe_ipc_handle", self.lib.pmoe_ipc_handle(self.local_buf, h))
            handles = exchange_handles(h.raw, group)
            ptrs = []
            for r, hr in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.local_buf)
                    continue
                p = ctypes.c_void_p()
                _lib.check("pmoe_ipc_open", self.lib.pmoe_ipc_open(hr, ctypes.byref(p)))
                ptrs.append(p.value)
            self.peer_ptrs = ptrs
            self.peer_arr = (ctypes.c_void_p * self.world)(*ptrs)
            self.t_max = t_max
            _lib.check("pmoe_comm_set_ep", self.lib.pmoe_comm_set_ep(
                self.comm, self.peer_arr, self.buf_bytes, min(t_max, FUSED_MAX_T)))
            torch.cuda.synchronize()
            dist.barrier(group)

    def _init_state(self, num_experts, hidden, top_k, mode, rank, world, group):
        self.group = group
        self.rank, self.world = rank, world
        self.E, self.H, self.K = num_experts, hidden, top_k
        self.lo, self.hi = expert_range(num_experts, self.rank, self.world)
        self.mode = mode
        self.epoch = 0
        self.lib = _lib.load()
        self.local_buf = None
        self.peer_ptrs = None
        self.owns_buffers = True
        self.rx_local = None    # row-split exchange buffers (prefill), allocated on first use
        self.rx_tmax = 0
        # the native communicator (pmoe_comm_create): the exchange buffers'
        # peer pointers and the row exchange's epoch; the comm_handle of
        # torch.ops.paris_moe.moe_block
        c = ctypes.c_void_p()
        _lib.check("pmoe_comm_create", self.lib.pmoe_comm_create(rank, world, ctypes.byref(c)))
        self.comm = c.value
        # prefill exchange: "rows" (the down GEMM stores rows at their token
        # owner, pmoe_block_forward_rows_fused), "slice" (the same with each
        # rank routing only its token slice and the routing exchanged over
        # NVLink: token-dispatch routing, PMOE_F_ROUTE_SLICE) or "partial"
        # (per-rank partial outputs summed by pmoe_rows_allreduce).  Measured (tokens/s, T=8192
        # Zipf): 2 ranks rows 14.7M / partial 13.9M, 4 ranks 17.4M / 17.1M,
        # 8 ranks 5.9M / 18.6M -- back-to-back row-exchange calls stalled at 8
        # ranks (a synchronised call took 0.39 ms, a pipelined one 1.39 ms), so
        # from 8 ranks on the partial-sum exchange is the default.
        self.prefill = "rows" if world < 8 else "partial"
        # sticky status words of this rank's exchange buffers ([0] decode, [1]
        # row split), copied here asynchronously after every exchange call
        self._st_host = torch.zeros(2, dtype=torch.int32,
                                    pin_memory=torch.cuda.is_available())
        self._st_event = None

    @classmethod
    def emulated(cls, num_experts: int, hidden: int, top_k: int, rank: int, world: int,
                 peer_bufs=None, rows_bufs=None, rows_t_max: int = 0, t_max: int = FUSED_MAX_T):
        """A rank of a peer group whose exchange buffers the caller provides
        (device pointers, one per rank; no process group, no IPC): for running
        the exchange paths in one process, e.g. with ranks that never arrive.
        ``peer_bufs``: pmoe_ep_buffer_bytes(t_max) each; ``rows_bufs``:
        pmoe_rows_fused_buffer_bytes(rows_t_max) each.  The caller frees them."""
        g = cls.__new__(cls)
        g._init_state(num_experts, hidden, top_k, "fused", rank, world, None)
        g.owns_buffers = False
        if peer_bufs is not None:
            nb = ctypes.c_size_t(0)
            _lib.check("pmoe_ep_buffer_bytes",
                       g.lib.pmoe_ep_buffer_bytes(t_max, hidden, top_k, ctypes.byref(nb)))
            g.buf_bytes, g.t_max = int(nb.value), t_max
            g.peer_ptrs = list(peer_bufs)
            g.local_buf = g.peer_ptrs[rank]
            g.peer_arr = (ctypes.c_void_p * world)(*g.peer_ptrs)
            _lib.check("pmoe_comm_set_ep", g.lib.pmoe_comm_set_ep(
                g.comm, g.peer_arr, g.buf_bytes, min(t_max, FUSED_MAX_T)))
        if rows_bufs is not None:
            g.rx_ptrs = list(rows_bufs)
            g.rx_local = g.rx_ptrs[rank]
            g.rx_tmax = rows_t_max
            g.rx_arr = (ctypes.c_void_p * world)(*g.rx_ptrs)
            _lib.check("pmoe_comm_set_rows", g.lib.pmoe_comm_set_rows(g.comm, g.rx_arr,
                                                                      rows_t_max))
        return g

    # ---- peer-loss detection ---------------------------------------------------

    def _status_enqueue(self, stream):
        """Copy the sticky status words to pinned host memory in stream order
        (not while the stream is being captured into a graph)."""
        if torch.cuda.is_current_stream_capturing():
            return
        hp = self._st_host.data_ptr()
        if self.local_buf is not None:
            _lib.check("pmoe_ep_status_async",
                       self.lib.pmoe_ep_status_async(self.local_buf, hp, stream))
        if self.rx_local is not None:
            _lib.check("pmoe_rows_status_async",
                       self.lib.pmoe_rows_status_async(self.rx_local, hp + 4, stream))
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        self._st_event = ev

    def _status_check(self, block: bool):
        ev = self._st_event
        if ev is None:
            return
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            # no event query while a graph is being captured: the sticky word
            # is read at the next call outside the capture
            return
        if block:
            ev.synchronize()
        elif not ev.query():
            return
        codes = self._st_host.tolist()
        if any(codes):
            raise _lib.PmoeError(
                "EPGroup", _lib.PMOE_ERR_PEER_TIMEOUT,
                f"rank {self.rank}: a peer GPU did not arrive within the bounded wait "
                f"(status words {codes}); the exchange results since then are invalid")

    def check(self):
        """Wait for the last exchange call's status and raise PmoeError
        (PMOE_ERR_PEER_TIMEOUT) if any wait on a peer has given up."""
        self._status_check(block=True)

    def uses_exchange(self, T: int) -> bool:
        return self.peer_ptrs is not None and T <= min(self.t_max, FUSED_MAX_T)

    def forward(self, x: torch.Tensor, weights, flags: int = 3,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                events=None):
        """y[T,H] (full output on every rank) for replicated x[T,H].  `events`
        (5 CUDA event handles, as pmoe_block_forward_profiled takes) are recorded
        between the phases of a fused prefill call and ignored otherwise."""
        self._status_check(block=False)
        T, H = x.shape
        w = list(weights)
        I, Is = w[1].shape[1] // 2, w[4].shape[0]
        y = out if out is not None else torch.empty((T, H), dtype=_BF16, device=x.device)
        if T == 0:
            return y
        nbytes = _lib.workspace_size(T, H, self.E, self.K, I, Is)
        ws = workspace if workspace is not None else torch.empty(nbytes, dtype=torch.uint8,
                                                                 device=x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        wp = [t.data_ptr() for t in w]
        slo, shi = token_range(T, self.rank, self.world)
        if self.mode == "fused" and self.world > 1:
            if not self.uses_exchange(T):
                if self.prefill == "partial" or (flags & 3) != 3:
                    return self._forward_rows_partial(x, wp, I, Is, flags, y, ws, nbytes, st)
                self._rows_buffers(T)
            # the communicator picks the exchange: T <= t_max the decode one
            # (device-side epoch, so the call can be captured in a CUDA graph),
            # else the row-split one with its next host epoch
            ev, nev = (events, 5) if events is not None else (None, 0)
            fl = flags
            if self.prefill == "slice" and not self.uses_exchange(T):
                fl |= _lib.PMOE_F_ROUTE_SLICE
            _lib.check("pmoe_block_forward_comm", self.lib.pmoe_block_forward_comm(
                self.comm, x.data_ptr(), T, H, self.E, self.K, I, Is, *wp, fl, y.data_ptr(),
                ws.data_ptr(), nbytes, st, ev, nev))
            self._status_enqueue(st)
            return y
        if self.mode == "a2a" and self.world > 1:
            return self._forward_a2a(x, w, I, Is, y)
        s = self.lib.pmoe_block_forward_ep(
            x.data_ptr(), T, H, self.E, self.K, I, Is, *wp, self.lo, self.hi, slo, shi, flags,
            None, 0, self.rank, self.world, 0, y.data_ptr(), ws.data_ptr(), nbytes, st)
        _lib.check("pmoe_block_forward_ep", s)
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y

    def reserve(self, T: int) -> None:
        """Make the exchanges take batches of T tokens (collective: every rank
        calls it with the same T).  Needed before torch.ops.paris_moe.moe_block
        is called with this group's comm_handle at a T above t_max, since the
        operator cannot allocate the IPC-mapped row buffers itself."""
        if self.mode == "fused" and self.world > 1 and not self.uses_exchange(T):
            self._rows_buffers(T)

    @property
    def comm_handle(self) -> int:
        """The pmoe_comm_create handle, for torch.ops.paris_moe.moe_block(...,
        ep_rank=rank, ep_size=world, comm_handle=...)."""
        return int(self.comm or 0)

    def op_forward(self, x: torch.Tensor, weights, flags: int = 3) -> torch.Tensor:
        """forward() through the registered operator, as the patched HF module
        calls it: torch.ops.paris_moe.moe_block with this group's comm_handle
        (mode "fused"; the other modes are comparators and use forward())."""
        if self.mode != "fused" or self.world == 1 or (
                self.prefill == "partial" and not self.uses_exchange(x.shape[0])):
            return self.forward(x, weights, flags)
        from . import ops
        self._status_check(block=False)
        self.reserve(x.shape[0])
        y = ops.moe_block(x, *weights, self.K, 0, -1, flags, ep_rank=self.rank,
                          ep_size=self.world, comm_handle=self.comm_handle)
        self._status_enqueue(torch.cuda.current_stream(x.device).cuda_stream)
        return y

    def _forward_rows_partial(self, x, wp, I, Is, flags, y, ws, nbytes, st):
        """Prefill "partial" (the comparator of the fused row exchange): every
        rank routes all tokens (identically), computes its row-balanced share of
        the dispatched rows into its partial output in its exchange buffer
        (pmoe_block_forward_rows), and pmoe_rows_allreduce sums the partials
        (deterministic, fp32) into y.  The epoch comes from the communicator,
        which shares the row buffers with the fused path."""
        T, H = x.shape
        self._rows_buffers(T)
        ep = ctypes.c_int(0)
        _lib.check("pmoe_comm_next_rows_epoch",
                   self.lib.pmoe_comm_next_rows_epoch(self.comm, ctypes.byref(ep)))
        part = ctypes.c_void_p()
        _lib.check("pmoe_rows_partial", self.lib.pmoe_rows_partial(
            self.rx_local, self.rx_tmax, H, ep.value, ctypes.byref(part)))
        _lib.check("pmoe_block_forward_rows", self.lib.pmoe_block_forward_rows(
            x.data_ptr(), T, H, self.E, self.K, I, Is, *wp, None, None, None, 0, self.E,
            self.rank, self.world, flags, part.value, ws.data_ptr(), nbytes, st))
        _lib.check("pmoe_rows_allreduce", self.lib.pmoe_rows_allreduce(
            self.rx_arr, self.rx_tmax, T, H, self.rank, self.world, ep.value, y.data_ptr(),
            st))
        self._status_enqueue(st)
        return y

    def _forward_a2a(self, x, w, I, Is, y):
        """Token-dispatch comparator (all_to_all_single, the variant ep.py does not
        have): each rank routes its own tokens, sends every token once to each
        rank owning one of its experts, receivers compute their expert range on
        the received tokens with the sender's routing (pmoe_block_forward_rows,
        world 1), partial rows come back through a second all-to-all and are
        added to the shared expert's output at home; an all_gather replicates y."""
        from . import ops
        T, H = x.shape
        K, world, rank = self.K, self.world, self.rank
        dev = x.device
        t0, t1 = token_range(T, rank, world)
        xl = x[t0:t1]
        idx, wts, *_ = ops.moe_route(xl, w[0], w[6], K)
        send, counts = a2a_plan(idx, self.E, world)
        rc = torch.empty(world, dtype=torch.long, device=dev)
        dist.all_to_all_single(rc, counts.to(dev), group=self.group)
        sc, rc = counts.tolist(), rc.cpu().tolist()
        M = sum(rc)
        rx = torch.empty((M, H), dtype=_BF16, device=dev)
        ri = torch.empty((M, K), dtype=torch.int32, device=dev)
        rw = torch.empty((M, K), dtype=torch.float32, device=dev)
        dist.all_to_all_single(rx, xl[send].contiguous(), rc, sc, group=self.group)
        dist.all_to_all_single(ri, idx[send].contiguous(), rc, sc, group=self.group)
        dist.all_to_all_single(rw, wts[send].contiguous(), rc, sc, group=self.group)
        yr = torch.zeros((M, H), dtype=_BF16, device=dev)
        if M > 0:
            nb = _lib.workspace_size(M, H, self.E, K, I, Is)
            ws = torch.empty(nb, dtype=torch.uint8, device=dev)
            gate = torch.zeros(M, dtype=torch.float32, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            _lib.check("pmoe_block_forward_rows", self.lib.pmoe_block_forward_rows(
                rx.data_ptr(), M, H, self.E, K, I, Is, *[t.data_ptr() for t in w],
                ri.data_ptr(), rw.data_ptr(), gate.data_ptr(), self.lo, self.hi, 0, 1, 2,
                yr.data_ptr(), ws.data_ptr(), nb, st))
        back = torch.empty((sum(sc), H), dtype=_BF16, device=dev)
        dist.all_to_all_single(back, yr, sc, rc, group=self.group)
        yl = ops.moe_block(xl, *w, K, 0, 0, 1).float()          # shared expert only
        yl.index_add_(0, send, back.float())
        chunk = (T + world - 1) // world
        slab = torch.zeros((world * chunk, H), dtype=_BF16, device=dev)
        slab[rank * chunk:rank * chunk + (t1 - t0)] = yl.to(_BF16)
        dist.all_gather_into_tensor(slab, slab[rank * chunk:(rank + 1) * chunk].clone(),
                                    group=self.group)
        for r in range(world):
            a, b = token_range(T, r, world)
            y[a:b] = slab[r * chunk:r * chunk + (b - a)]
        return y

    def _rows_buffers(self, T: int):
        """(Re)allocate the IPC-mapped partial buffers for batches of T tokens
        (collective: every rank calls forward with the same T)."""
        if self.rx_local is not None and T <= self.rx_tmax:
            return
        if not self.owns_buffers:
            raise ValueError(f"emulated group: row buffers for {self.rx_tmax} tokens, got {T}")
        self._close_rows()
        nb = ctypes.c_size_t(0)
        _lib.check("pmoe_rows_fused_buffer_bytes",
                   self.lib.pmoe_rows_fused_buffer_bytes(T, self.H, self.K, ctypes.byref(nb)))
        ptr = ctypes.c_void_p()
        _lib.check("pmoe_ipc_alloc", self.lib.pmoe_ipc_alloc(nb.value, ctypes.byref(ptr)))
        self.rx_local, self.rx_tmax = ptr.value, T
        h = ctypes.create_string_buffer(64)
        _lib.check("pmoe_ipc_handle", self.lib.pmoe_ipc_handle(self.rx_local, h))
        ptrs = []
        for r, hr in enumerate(exchange_handles(h.raw, self.group)):
            if r == self.rank:
                ptrs.append(self.rx_local)
                continue
            p = ctypes.c_void_p()
            _lib.check("pmoe_ipc_open", self.lib.pmoe_ipc_open(hr, ctypes.byref(p)))
            ptrs.append(p.value)
        self.rx_ptrs = ptrs
        self.rx_arr = (ctypes.c_void_p * self.world)(*ptrs)
        _lib.check("pmoe_comm_set_rows", self.lib.pmoe_comm_set_rows(self.comm, self.rx_arr, T))
        torch.cuda.synchronize()
        dist.barrier(self.group)

    def _close_rows(self):
        if self.rx_local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        _lib.check("pmoe_comm_set_rows", self.lib.pmoe_comm_set_rows(self.comm, None, 0))
        for r, p in enumerate(self.rx_ptrs):
            if r != self.rank:
                self.lib.pmoe_ipc_close(p)
        self.lib.pmoe_ipc_free(self.rx_local)
        self.rx_local = None

    def layer_forward(self, x: torch.Tensor, w_norm: torch.Tensor, eps: float, weights,
                      flags: int = 3, out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None):
        """One MoE-only decoder layer, x + block(RMSNorm(x)), full output on every
        rank (pmoe_layer_forward over the NVLink exchange; T <= t_max).  ``out``
        may be ``x`` (in-place residual update)."""
        self._status_check(block=False)
        T, H = x.shape
        if not self.uses_exchange(T) and self.world > 1:
            raise ValueError("layer_forward across ranks needs the fused exchange (T <= t_max)")
        w = list(weights)
        I, Is = w[1].shape[1] // 2, w[4].shape[0]
        y = out if out is not None else torch.empty((T, H), dtype=_BF16, device=x.device)
        if T == 0:
            return y
        nbytes = _lib.workspace_size(T, H, self.E, self.K, I, Is)
        ws = workspace if workspace is not None else torch.empty(nbytes, dtype=torch.uint8,
                                                                 device=x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        wp = [t.data_ptr() for t in w]
        slo, shi = token_range(T, self.rank, self.world)
        peers = self.peer_arr if self.world > 1 else None
        s = self.lib.pmoe_layer_forward(
            x.data_ptr(), T, H, self.E, self.K, I, Is, w_norm.data_ptr(), float(eps), *wp,
            self.lo, self.hi, slo, shi, flags, peers, self.buf_bytes if peers else 0, self.rank,
            self.world, 0, y.data_ptr(), ws.data_ptr(), nbytes, st)
        _lib.check("pmoe_layer_forward", s)
        if peers is not None:
            self._status_enqueue(st)
        return y

    def close(self):
        """Release the exchange buffers; raises PmoeError afterwards if a wait
        on a peer gave up in any call since the last check."""
        err = None
        try:
            self._status_check(block=True)
        except _lib.PmoeError as e:
            err = e
        if self.owns_buffers:
            self._close_rows()
            if self.peer_ptrs is not None:
                torch.cuda.synchronize()
                for r, p in enumerate(self.peer_ptrs):
                    if r != self.rank:
                        self.lib.pmoe_ipc_close(p)
                self.lib.pmoe_ipc_free(self.local_buf)
        if self.comm:
            self.lib.pmoe_comm_destroy(self.comm)
            self.comm = None
        self.peer_ptrs = None
        self.local_buf = None
        self.rx_local = None
        self._st_event = None
        if err is not None:
            raise err


def patch_moe_for_ep(model, rank: int, world_size: int, mode: str = "fused") -> int:
    """Install the EP forward on every Qwen3_5MoeSparseMoeBlock of ``model``
    (after ``moe.patch_qwen3_5_moe()``).  Returns the number of blocks."""
    if world_size <= 1:
        return 0
    from transformers.models.qwen3_5_moe.modeling_qwen3_5_moe import Qwen3_5MoeSparseMoeBlock
    from .moe import block_weights
    count = 0
    group = None
    for m in model.modules():
        if isinstance(m, Qwen3_5MoeSparseMoeBlock):
            if group is None:
                group = EPGroup(m.gate.weight.shape[0], m.gate.weight.shape[1],
                                int(m.gate.top_k), mode=mode)
            m._pmoe_expert_range = (group.lo, group.hi)
            m._pmoe_post = (lambda blk, x, g=group: g.op_forward(x, block_weights(blk)))
            count += 1
    return count
