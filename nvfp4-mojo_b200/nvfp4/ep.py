"""Expert-parallel NVFP4 MoE layer over NCCL (torch.distributed).

One process per GPU; rank r of a world of G owns experts
[r * E/G, (r+1) * E/G) (their stacked NVFP4 weights) and a replica of the
fp32 router.  Per layer, on every rank:

  1. route its own tokens (softmax top-k over all E experts);
  2. plan the dispatch on the device: slots grouped by destination rank;
  3. exchange per-rank slot counts (all-to-all, 4 bytes per peer);
  4. gather the token rows in send order and exchange them with the local
     expert ids (all-to-all over NVLink);
  5. run the local experts on the received rows (grouped NVFP4 GEMMs);
  6. return the fp32 expert outputs (reverse all-to-all);
  7. combine them in slot order with the routing weights (+ residual).

Steps 1, 2, 4 (gather), 5 and 7 are libnvfp4 CUDA kernels; steps 3, 4 and 6
are NCCL collectives.  With exchange="p2p" the kernels move the rows
themselves: the dispatch kernel stores each routed row straight into the
owning rank's window (peer memory over NVLink / NVSwitch) and the combine
kernel loads the expert outputs back from the peers' windows, ordered by
cross-GPU flags with bounded waits (include/nvfp4_ep.h) -- no NCCL call and
no host synchronisation in the step.  For small batches the exchange uses fixed capacities
instead (EPMoELayer.forward_static): no step 3, no host synchronisation.  The kernel calls go through a backend object so the
exchange logic can be exercised with CPU ranks (gloo) in tests.
"""
from __future__ import annotations

from typing import Optional

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .moe import MoEWeights, make_desc, moe_combine, moe_experts, moe_route, _ptr
from .nvfp4_gemm_gpu import _stream


class CudaBackend:
    """The libnvfp4 kernels (the product path)."""

    def __init__(self, local: MoEWeights, router: torch.Tensor, top_k: int, renormalize=True):
        self.local = local
        self.router_w = MoEWeights(router, local.gate_up, local.gate_up_scale,
                                   local.gate_up_scale_2, local.down, local.down_scale,
                                   local.down_scale_2)
        self.E_total = router.shape[1]
        self.top_k = top_k
        self.renormalize = renormalize
        self._ws = None

    def route(self, x):
        desc = _lib.MoEDesc(self.E_total, self.top_k, self.local.hidden, self.local.intermediate,
                            int(self.renormalize))
        T = x.shape[0]
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        tw = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        logits = torch.empty((T, self.E_total), dtype=torch.float32, device=x.device)
        import ctypes
        rc = _lib.load().nvfp4_moe_route(ctypes.byref(desc), _ptr(self.router_w.router), _ptr(x),
                                         T, _ptr(ids), _ptr(tw), _ptr(logits), _stream(None))
        _lib.check(rc)
        return ids, tw

    def plan(self, ids, epr, world):
        T, k = ids.shape
        R = T * k
        dev = ids.device
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        send_token = torch.empty(R, dtype=torch.int32, device=dev)
        send_expert = torch.empty(R, dtype=torch.int32, device=dev)
        slot_pos = torch.empty(R, dtype=torch.int32, device=dev)
        rc = _lib.load().nvfp4_ep_dispatch_plan(_ptr(ids), T, k, epr, world, _ptr(counts),
                                                _ptr(send_token), _ptr(send_expert),
                                                _ptr(slot_pos), _stream(None))
        _lib.check(rc)
        return counts, send_token, send_expert, slot_pos

    def pad(self, x, counts, send_token, send_expert, slot_pos, cap, world):
        """Fixed-capacity send layout: rows [world * cap, H], expert ids
        [world * cap] (-1 = padding) and the padded position of each slot."""
        T, H = x.shape
        k = slot_pos.numel() // max(T, 1)
        rows = torch.empty((world * cap, H), dtype=x.dtype, device=x.device)
        rows_e = torch.empty(world * cap, dtype=torch.int32, device=x.device)
        slot_pad = torch.empty(slot_pos.numel(), dtype=torch.int32, device=x.device)
        rc = _lib.load().nvfp4_ep_dispatch_padded(
            _ptr(counts), _ptr(send_token), _ptr(send_expert), _ptr(slot_pos), T, k, world, cap,
            _ptr(x), H * x.element_size(), _ptr(rows), _ptr(rows_e), _ptr(slot_pad),
            _stream(None))
        _lib.check(rc)
        return rows, rows_e, slot_pad

    def gather(self, x, idx):
        out = torch.empty((idx.numel(), x.shape[1]), dtype=x.dtype, device=x.device)
        rc = _lib.load().nvfp4_gather_rows(_ptr(x), _ptr(idx), idx.numel(),
                                           x.shape[1] * x.element_size(), _ptr(out), _stream(None))
        _lib.check(rc)
        return out

    def experts(self, rows, local_ids):
        return moe_experts(self.local, rows, local_ids, top_k=self.top_k, out_dtype=torch.float32)

    def combine(self, y_send, tw, slot_pos, residual):
        return moe_combine(y_send, tw, residual=residual, slot_pos=slot_pos)


def exchange_handles(handle: bytes, group=None) -> list:
    """All-gathers one fixed-size byte string per rank (the windows' IPC
    handles): element p of the result is rank p's."""
    world = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
    every = torch.empty(world * len(handle), dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(every, mine, group=group)
    raw = every.cpu().numpy().tobytes()
    return [raw[p * len(handle):(p + 1) * len(handle)] for p in range(world)]


class PeerWindows:
    """This rank's exchange window and the other ranks' windows as mapped in
    this process (nvfp4_ep_window_create / _open).  `rendezvous` builds them
    across the processes of a group (IPC handles all-gathered once);
    `emulated` builds the windows of `world` ranks in one process on one
    device, for running the ranks' steps one after another in one stream."""

    def __init__(self, rank, world, max_rows, hidden, windows, owned, opened, timeout_ms=0,
                 group=None, collective=False):
        self.rank, self.world = rank, world
        self.group, self._collective = group, collective
        self.max_rows, self.hidden = max_rows, hidden
        self.windows = list(windows)
        self._owned = list(owned)    # windows this object frees
        self._opened = list(opened)  # peer mappings this object closes
        self.timeout_ms = timeout_ms

    @staticmethod
    def _create(world, max_rows, hidden):
        L = _lib.load()
        size = L.nvfp4_ep_window_size(world, max_rows, hidden)
        if size == 0:
            raise ValueError(f"bad window shape: world {world}, max_rows {max_rows}, "
                             f"hidden {hidden}")
        win = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES)()
        _lib.check(L.nvfp4_ep_window_create(size, ctypes.byref(win), handle))
        return win.value, bytes(handle)

    @classmethod
    def rendezvous(cls, max_rows: int, hidden: int, group=None, timeout_ms: int = 0):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        if world > _lib.EP_MAX_WORLD:
            raise ValueError(f"peer exchange supports up to {_lib.EP_MAX_WORLD} ranks")
        own, handle = cls._create(world, max_rows, hidden)
        windows, opened = [None] * world, []
        windows[rank] = own
        L = _lib.load()
        try:
            if world > 1:
                every = exchange_handles(handle, group)
                for p in range(world):
                    if p == rank:
                        continue
                    h = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES).from_buffer_copy(every[p])
                    w = ctypes.c_void_p()
                    _lib.check(L.nvfp4_ep_window_open(h, ctypes.byref(w)))
                    windows[p] = w.value
                    opened.append(w.value)
                dist.barrier(group)  # every window zeroed and mapped before any step
        except BaseException:
            for w in opened:
                L.nvfp4_ep_window_close(w)
            L.nvfp4_ep_window_destroy(own)
            raise
        return cls(rank, world, max_rows, hidden, windows, [own], opened, timeout_ms, group,
                   collective=world > 1)

    @classmethod
    def emulated(cls, world: int, max_rows: int, hidden: int, timeout_ms: int = 0):
        wins = [cls._create(world, max_rows, hidden)[0] for _ in range(world)]
        return [cls(r, world, max_rows, hidden, wins, wins if r == 0 else [], [], timeout_ms)
                for r in range(world)]

    def peers(self) -> _lib.EpPeers:
        p = _lib.EpPeers()
        p.rank, p.world, p.max_rows = self.rank, self.world, self.max_rows
        p.hidden, p.timeout_ms = self.hidden, self.timeout_ms
        for i, w in enumerate(self.windows):
            p.windows[i] = w
        return p

    def rows(self, T: int, k: int):
        """Device pointers of this rank's received rows, expert ids and
        expert output rows for a step of T tokens."""
        x, e, o = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.load().nvfp4_ep_p2p_rows(ctypes.byref(self.peers()), T, k,
                                                 ctypes.byref(x), ctypes.byref(e),
                                                 ctypes.byref(o)))
        return x.value, e.value, o.value

    def error(self, clear: bool = True, stream=None) -> int:
        v = ctypes.c_uint32()
        _lib.check(_lib.load().nvfp4_ep_p2p_error(ctypes.byref(self.peers()), ctypes.byref(v),
                                                  int(clear), _stream(stream)))
        return v.value

    def close(self):
        """Unmaps the peers' windows and frees this rank's.  For windows made
        by `rendezvous` this is collective: every rank unmaps first, then a
        barrier, then each frees its own, so no window is freed while another
        process still maps it."""
        L = _lib.load()
        for w in self._opened:
            L.nvfp4_ep_window_close(w)
        self._opened = []
        if self._collective and self._owned and dist.is_initialized():
            dist.barrier(self.group)
        for w in self._owned:
            L.nvfp4_ep_window_destroy(w)
        self._owned = []


def p2p_dispatch(pw: PeerWindows, topk_ids, x, experts_per_rank: int, stream=None):
    T, k = topk_ids.shape
    _lib.check(_lib.load().nvfp4_ep_p2p_dispatch(ctypes.byref(pw.peers()), _ptr(topk_ids),
                                                 _ptr(x), T, k, experts_per_rank,
                                                 _stream(stream)))


def p2p_wait_dispatch(pw: PeerWindows, stream=None):
    _lib.check(_lib.load().nvfp4_ep_p2p_wait_dispatch(ctypes.byref(pw.peers()), _stream(stream)))


def p2p_experts(pw: PeerWindows, local: MoEWeights, T: int, k: int, workspace=None,
                stream=None):
    """The local experts on the world*T*k received rows, into the window."""
    rx, re, out = pw.rows(T, k)
    R = pw.world * T * k
    desc = make_desc(local, 1)
    L = _lib.load()
    need = L.nvfp4_moe_experts_workspace_size(ctypes.byref(desc), R)
    ws = workspace if workspace is not None and workspace.numel() >= need else \
        torch.empty(max(need, 256), dtype=torch.uint8, device=local.gate_up.device)
    _lib.check(L.nvfp4_moe_experts(ctypes.byref(desc), ctypes.byref(local.ptrs()), rx, None, re,
                                   R, out, _lib.DTYPE_F32, _ptr(ws), ws.numel(),
                                   _stream(stream)))


def p2p_signal_done(pw: PeerWindows, stream=None):
    _lib.check(_lib.load().nvfp4_ep_p2p_signal_done(ctypes.byref(pw.peers()), _stream(stream)))


def p2p_combine(pw: PeerWindows, topk_ids, topk_w, experts_per_rank: int, residual=None,
                out=None, stream=None):
    T, k = topk_ids.shape
    y = out if out is not None else torch.empty((T, pw.hidden), dtype=torch.bfloat16,
                                                device=topk_ids.device)
    ydt = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}[y.dtype]
    _lib.check(_lib.load().nvfp4_ep_p2p_combine(ctypes.byref(pw.peers()), _ptr(topk_ids),
                                                _ptr(topk_w), T, k, experts_per_rank,
                                                _ptr(residual), _ptr(y), ydt, _stream(stream)))
    return y


class EPMoELayer:
    """Expert-parallel MoE layer; `backend` defaults to the CUDA kernels.

    Two exchange modes.  Variable (the default for large batches): per-peer
    slot counts are exchanged and read on the host, and only the routed rows
    cross NVLink.  Fixed capacity (`static=True`; chosen automatically when
    world * T * k <= static_rows): every peer gets T * k rows (the most any
    peer can receive from one rank), padded, so no count is read on the host
    and a step can be captured in a CUDA graph with its NCCL calls; the
    padding costs NVLink bytes, not expert compute (padded rows carry expert
    id -1 and are skipped)."""

    def __init__(self, local: Optional[MoEWeights], router: torch.Tensor, top_k: int = 8,
                 num_experts: Optional[int] = None, group=None, backend=None,
                 renormalize: bool = True, static: Optional[bool] = None,
                 static_rows: int = 8192, exchange: str = "nccl",
                 max_tokens: Optional[int] = None, timeout_ms: int = 0,
                 windows: Optional["PeerWindows"] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.E = num_experts if num_experts is not None else router.shape[1]
        if self.E % self.world:
            raise ValueError("num_experts must be divisible by the world size")
        self.epr = self.E // self.world
        self.top_k = top_k
        self.backend = backend or CudaBackend(local, router, top_k, renormalize)
        self.static = static
        self.static_rows = static_rows
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.exchange = exchange
        self.windows = None
        self._own_windows = False
        self.renormalize = renormalize
        self._ws = {}
        if exchange == "p2p":
            if max_tokens is None:
                raise ValueError("the peer exchange needs max_tokens (rows per rank are "
                                 "max_tokens * top_k)")
            self.max_tokens = max_tokens
            if windows is not None:
                # Layers that run one after another in one stream may share
                # windows: each step's flags carry the step counter, and the
                # received rows of one layer are dead once its combine ran.
                if (windows.world != self.world or windows.hidden != router.shape[0] or
                        windows.max_rows < max_tokens * top_k):
                    raise ValueError("shared windows do not fit this layer")
                self.windows = windows
            else:
                self.windows = PeerWindows.rendezvous(max_tokens * top_k, router.shape[0],
                                                      group, timeout_ms)
                self._own_windows = True

    def uses_static(self, T: int) -> bool:
        if self.static is not None:
            return bool(self.static)
        return self.world * T * self.top_k <= self.static_rows

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward_static(self, x: torch.Tensor,
                       residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Fixed-capacity exchange: equal splits of T * k rows per peer."""
        be = self.backend
        cap = x.shape[0] * self.top_k
        ids, tw = be.route(x)
        counts, send_token, send_expert, slot_pos = be.plan(ids, self.epr, self.world)
        send_x, send_e, slot_pad = be.pad(x, counts, send_token, send_expert, slot_pos, cap,
                                          self.world)
        recv_x = torch.empty_like(send_x)
        recv_e = torch.empty_like(send_e)
        self._a2a(recv_x, send_x, None, None)
        self._a2a(recv_e, send_e, None, None)
        y_recv = be.experts(recv_x, recv_e)
        y_send = torch.empty_like(y_recv)
        self._a2a(y_send, y_recv, None, None)
        return be.combine(y_send, tw, slot_pad, residual)

    def forward_p2p(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One step through peer memory (nvfp4_ep_p2p_forward): every rank
        calls it with the same token count."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the windows' {self.max_tokens}")
        be = self.backend
        w = be.router_w
        desc = _lib.MoEDesc(self.E, self.top_k, w.hidden, w.intermediate, int(self.renormalize))
        peers = self.windows.peers()
        L = _lib.load()
        ws = self._ws.get(T)
        if ws is None:
            need = L.nvfp4_ep_p2p_workspace_size(ctypes.byref(desc), ctypes.byref(peers), T)
            if need == 0:
                raise ValueError("bad expert-parallel layer shape")
            ws = self._ws[T] = torch.empty(need, dtype=torch.uint8, device=x.device)
        y = out if out is not None else torch.empty_like(x)
        ydt = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}[y.dtype]
        _lib.check(L.nvfp4_ep_p2p_forward(ctypes.byref(desc), ctypes.byref(w.ptrs()),
                                          ctypes.byref(peers), _ptr(x), _ptr(residual), _ptr(y),
                                          ydt, T, _ptr(ws), ws.numel(), _stream(None)))
        return y

    def close(self):
        if self.windows is not None and self._own_windows:
            self.windows.close()
        self.windows = None

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.exchange == "p2p":
            return self.forward_p2p(x, residual)
        if self.uses_static(x.shape[0]):
            return self.forward_static(x, residual)
        be = self.backend
        ids, tw = be.route(x)
        counts, send_token, send_expert, slot_pos = be.plan(ids, self.epr, self.world)
        recv_counts = torch.empty_like(counts)
        self._a2a(recv_counts, counts, None, None)
        send_sizes = counts.tolist()
        recv_sizes = recv_counts.tolist()
        n_recv = sum(recv_sizes)
        n_send = sum(send_sizes)  # slots with a valid expert id
        send_token, send_expert = send_token[:n_send], send_expert[:n_send]
        send_x = be.gather(x, send_token)
        recv_x = torch.empty((n_recv, x.shape[1]), dtype=x.dtype, device=x.device)
        recv_e = torch.empty(n_recv, dtype=torch.int32, device=x.device)
        self._a2a(recv_x, send_x, recv_sizes, send_sizes)
        self._a2a(recv_e, send_expert, recv_sizes, send_sizes)
        y_recv = be.experts(recv_x, recv_e)
        y_send = torch.empty((send_x.shape[0], x.shape[1]), dtype=y_recv.dtype, device=x.device)
        self._a2a(y_send, y_recv, send_sizes, recv_sizes)
        return be.combine(y_send, tw, slot_pos, residual)

    __call__ = forward
