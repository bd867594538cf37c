"""Expert parallelism over the GPUs of one node: one process per GPU,
experts of every layer split in contiguous blocks of E/N, the routers replicated.

Each decode layer is one `moe_ep_decode_layer` call per rank (include/moe_b200.h): the router
and top-k run on every rank with identical results, every rank runs its own experts on the
(token, k) slots routed to them, and one kernel moves the expert outputs over NVLink straight
into every rank's exchange buffer and combines them in MLX order, so every rank ends the
layer with the same hidden states, bit for bit equal to the single-GPU decode layer.

torch.distributed is plumbing here: it only carries the CUDA IPC handles of the exchange
buffers between the ranks once at set-up and the barriers around teardown; the data path
uses no library collective.

Batches with several tokens per GPU run token-sharded (`ep_a2a_layer`, `EPA2AStack`): every
rank owns a block of the batch's tokens; one kernel dispatches each token's row only to the
ranks holding its routed experts and another returns each expert output row only to the
token's owner, which combines (a routed all-to-all over peer stores).

The reference runs the MoE block on one device (mlx-qwen38/loader.py:903-922 per layer); this
module is the multi-GPU form of that block the expert-parallel configuration asks for.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import call
from .ops import QMatrix, _need, _ptr, _stream
from .synthetic import ExpertLayer

HANDLE_BYTES = 64


def expert_shard(E: int, rank: int, world: int) -> tuple[int, int]:
    """(first expert, count) of rank's contiguous block: E/world each, the first E % world
    ranks one more."""
    if world <= 0 or not 0 <= rank < world or E < world:
        raise ValueError(f"cannot split {E} experts over {world} ranks (rank {rank})")
    base, extra = divmod(E, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def shard_qmatrix(q: QMatrix, first: int, count: int) -> QMatrix:
    """The experts [first, first + count) of an [E, ...] QMatrix (contiguous copies)."""
    return QMatrix(q.w[first:first + count].contiguous(), q.s[first:first + count].contiguous(),
                   q.b[first:first + count].contiguous(), q.bits, q.group_size)


def shard_layer(layer: ExpertLayer, first: int, count: int) -> ExpertLayer:
    """A rank's part of one layer: the whole router, its block of the experts."""
    return ExpertLayer(layer.router, shard_qmatrix(layer.gate, first, count), shard_qmatrix(layer.up, first, count),
                       shard_qmatrix(layer.down, first, count))


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's IPC handle, in rank order (one all_gather_object over the process group;
    a single process gets its own)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return [bytes(handle)]
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return [bytes(h) for h in out]


class ExchangeBuffers:
    """This rank's exchange buffer and the mapped buffers of the other ranks; `peers` is the
    device array the kernels take. Sized for up to T tokens: the replicated layer's flags + two
    receive buffers (moe_ep_buffer_bytes), or with a2a=True the token-sharded layer's flags,
    receive rows, routing table and returned rows (moe_ep_a2a_buffer_bytes)."""

    def __init__(self, T: int, K: int, H: int, device, group=None, a2a: bool = False):
        import torch.distributed as dist

        self.dist = dist.is_available() and dist.is_initialized()
        self.group = group
        self.world = dist.get_world_size(group) if self.dist else 1
        self.rank = dist.get_rank(group) if self.dist else 0
        self.T, self.K, self.H = T, K, H
        self.a2a = a2a
        self.device = torch.device(device)
        nbytes = int(call("moe_ep_a2a_buffer_bytes", T, K, H, self.world) if a2a else
                     call("moe_ep_buffer_bytes", T, K, H))
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            call("moe_ep_buffer_alloc", nbytes, ctypes.byref(own), handle)
        self.own = own.value
        self.opened: list[int] = []
        ptrs = []
        for q, h in enumerate(gather_handles(bytes(handle), group)):
            if q == self.rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * HANDLE_BYTES).from_buffer_copy(h)
            with torch.cuda.device(self.device):
                call("moe_ep_buffer_open", hb, ctypes.byref(p))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=self.device)

    def close(self) -> None:
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.dist and self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self.opened:
                call("moe_ep_buffer_close", p)
        if self.dist and self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            call("moe_ep_buffer_free", self.own)
        self.own = None
        self.opened = []


def ep_decode_layer(x: torch.Tensor, layer: ExpertLayer, E: int, first: int, K: int, xbuf: ExchangeBuffers, *,
                    norm: bool = True, resid=None, out: dict | None = None, workspace: torch.Tensor | None = None,
                    stream=None) -> dict:
    """One expert-parallel decode layer on this rank; every rank must make the same calls in
    the same order. layer holds the whole router and this rank's expert block, which starts
    at expert `first`. Returns dict(y, inds, scores), identical on every rank."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    T, H = x.shape
    if T > xbuf.T or K != xbuf.K or H != xbuf.H:
        raise ValueError(f"exchange buffers sized for T<={xbuf.T}, K={xbuf.K}, H={xbuf.H}; got {T}, {K}, {H}")
    _need(layer.router, "router", (torch.bfloat16,), dev)
    if layer.router.shape[0] != E:
        raise ValueError("the router must hold all E experts")
    n = layer.gate.w.shape[0]
    I = layer.gate.w.shape[1]
    for nm, q in (("gate", layer.gate), ("up", layer.up), ("down", layer.down)):
        q.check(nm, dev)
    o = out if out is not None else {}
    o.setdefault("y", torch.empty((T, H), dtype=torch.bfloat16, device=dev))
    o.setdefault("inds", torch.empty((T, K), dtype=torch.int32, device=dev))
    o.setdefault("scores", torch.empty((T, K), dtype=torch.bfloat16, device=dev))
    if workspace is None:
        workspace = torch.zeros(int(call("moe_ep_workspace_bytes", T, H, I, E, K)), dtype=torch.uint8, device=dev)
    g, u, d = layer.gate, layer.up, layer.down
    call("moe_ep_decode_layer", x.data_ptr(), T, H, I, E, K, first, n, layer.router.data_ptr(), g.w.data_ptr(),
         g.s.data_ptr(), g.b.data_ptr(), u.w.data_ptr(), u.s.data_ptr(), u.b.data_ptr(), d.w.data_ptr(),
         d.s.data_ptr(), d.b.data_ptr(), g.sb_fp16, int(norm), _ptr(resid), xbuf.peers.data_ptr(), xbuf.rank,
         xbuf.world, o["inds"].data_ptr(), o["scores"].data_ptr(), o["y"].data_ptr(), workspace.data_ptr(),
         workspace.numel(), _stream(stream))
    return o


class EPDecodeStack:
    """Decode of a batch of T tokens through L layers with the experts split across the
    ranks: h_{l+1} = h_l + MoE_l(norm(h_l)), every layer an ep_decode_layer, the whole token
    step captured in one CUDA graph per rank (the exchange kernel keeps its epoch in device
    memory, so graph replays stay in step across ranks)."""

    def __init__(self, layers: list[ExpertLayer], E: int, first: int, K: int, T: int, device, group=None,
                 use_graph: bool = True, norm: bool = True):
        self.layers, self.E, self.first, self.K, self.T = layers, E, first, K, T
        self.device = torch.device(device)
        self.norm = norm
        H = layers[0].router.shape[1]
        I = layers[0].gate.w.shape[1]
        self.H = H
        self.xbuf = ExchangeBuffers(T, K, H, self.device, group)
        self.ws = torch.zeros(int(call("moe_ep_workspace_bytes", T, H, I, E, K)), dtype=torch.uint8,
                              device=self.device)
        self.x = torch.zeros((T, H), dtype=torch.bfloat16, device=self.device)
        self.hs = [torch.zeros((T, H), dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        self.inds = torch.zeros((len(layers), T, K), dtype=torch.int32, device=self.device)
        self.scores = torch.zeros((len(layers), T, K), dtype=torch.bfloat16, device=self.device)
        self.launches_per_step = 4 * len(layers)     # router, gate/up, down, exchange + combine
        self.graph = None
        self.stream = torch.cuda.Stream(self.device)
        if use_graph:
            self._capture()

    def _layers_once(self) -> torch.Tensor:
        h = self.x
        for li, ly in enumerate(self.layers):
            o = dict(y=self.hs[li & 1], inds=self.inds[li], scores=self.scores[li])
            ep_decode_layer(h, ly, self.E, self.first, self.K, self.xbuf, norm=self.norm, resid=h, out=o,
                            workspace=self.ws, stream=torch.cuda.current_stream(self.device))
            h = o["y"]
        return h

    def _capture(self) -> None:
        # one eager step first (every rank does the same), then the capture
        self._layers_once()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.out = self._layers_once()
        self.graph = g

    def step_device(self, x: torch.Tensor) -> torch.Tensor:
        """One decode step of the batch x [T, H] (device); returns the last layer's output."""
        self.x.copy_(x)
        if self.graph is not None:
            self.graph.replay()
            return self.out
        return self._layers_once()

    def decode(self, h_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """End to end: the batch's hidden states from (pinned) host memory in, the final ones
        back to host memory, synchronised."""
        self.x.copy_(h_host, non_blocking=True)
        y = self.step_device(self.x)
        out_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_host

    def close(self) -> None:
        self.graph = None
        self.xbuf.close()


# batches with at least this many tokens per rank run token-sharded (routed all-to-all)
A2A_MIN_TOKENS_PER_RANK = 4


def expert_bounds(E: int, world: int) -> list[int]:
    """e_first: rank q holds experts [e_first[q], e_first[q + 1]) (expert_shard's blocks)."""
    out = [expert_shard(E, q, world)[0] for q in range(world)]
    return out + [E]


def local_tokens(T: int, world: int, rank: int) -> tuple[int, int]:
    """(first token, count) this rank owns in a token-sharded batch of T."""
    first = ctypes.c_int(0)
    n = int(call("moe_ep_a2a_local_tokens", T, world, rank, ctypes.byref(first)))
    return first.value, n


def ep_a2a_layer(x: torch.Tensor, layer: ExpertLayer, E: int, e_first: list[int], K: int, T: int,
                 xbuf: ExchangeBuffers, *, norm: bool = True, resid=None, out: dict | None = None,
                 workspace: torch.Tensor | None = None, stream=None) -> dict:
    """One token-sharded expert-parallel layer on this rank (moe_ep_a2a_layer): x [n, H] holds
    this rank's n tokens of the batch of T; layer holds the whole router and this rank's expert
    block [e_first[rank], e_first[rank + 1]). Every rank makes the same calls in the same order.
    Returns dict(y, inds, scores) for this rank's tokens."""
    _need(x, "x", (torch.bfloat16,))
    dev = x.device
    n, H = x.shape
    if not xbuf.a2a or T > xbuf.T or K != xbuf.K or H != xbuf.H:
        raise ValueError("exchange buffers must be a2a buffers sized for the batch")
    first, cnt = local_tokens(T, xbuf.world, xbuf.rank)
    if n != cnt:
        raise ValueError(f"rank {xbuf.rank} owns {cnt} of the {T} tokens, got {n} rows")
    I = layer.gate.w.shape[1]
    o = out if out is not None else {}
    o.setdefault("y", torch.empty((n, H), dtype=torch.bfloat16, device=dev))
    o.setdefault("inds", torch.empty((n, K), dtype=torch.int32, device=dev))
    o.setdefault("scores", torch.empty((n, K), dtype=torch.bfloat16, device=dev))
    if workspace is None:
        workspace = torch.zeros(int(call("moe_ep_a2a_workspace_bytes", T, H, I, E, K, xbuf.world)),
                                dtype=torch.uint8, device=dev)
    ef = (ctypes.c_int * len(e_first))(*e_first)
    g, u, d = layer.gate, layer.up, layer.down
    call("moe_ep_a2a_layer", x.data_ptr(), T, H, I, E, K, ef, layer.router.data_ptr(), g.w.data_ptr(),
         g.s.data_ptr(), g.b.data_ptr(), u.w.data_ptr(), u.s.data_ptr(), u.b.data_ptr(), d.w.data_ptr(),
         d.s.data_ptr(), d.b.data_ptr(), g.sb_fp16, int(norm), _ptr(resid), xbuf.peers.data_ptr(), xbuf.own,
         xbuf.rank, xbuf.world, o["inds"].data_ptr(), o["scores"].data_ptr(), o["y"].data_ptr(),
         workspace.data_ptr(), workspace.numel(), _stream(stream))
    return o


class EPA2AStack:
    """Decode (or prefill) of a batch of T tokens through L layers, token-sharded: this rank
    holds the hidden states of its own tokens (local_tokens) and its expert block of every
    layer; every layer is one ep_a2a_layer (routed all-to-all), the whole step one CUDA graph
    per rank (the kernels keep their epoch in device memory)."""

    def __init__(self, layers: list[ExpertLayer], E: int, e_first: list[int], K: int, T: int, device, group=None,
                 use_graph: bool = True, norm: bool = True):
        self.layers, self.E, self.e_first, self.K, self.T = layers, E, list(e_first), K, T
        self.device = torch.device(device)
        self.norm = norm
        H = layers[0].router.shape[1]
        I = layers[0].gate.w.shape[1]
        self.H = H
        self.xbuf = ExchangeBuffers(T, K, H, self.device, group, a2a=True)
        self.first, self.n = local_tokens(T, self.xbuf.world, self.xbuf.rank)
        self.ws = torch.zeros(int(call("moe_ep_a2a_workspace_bytes", T, H, I, E, K, self.xbuf.world)),
                              dtype=torch.uint8, device=self.device)
        n = max(self.n, 1)
        self.x = torch.zeros((n, H), dtype=torch.bfloat16, device=self.device)
        self.hs = [torch.zeros((n, H), dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        self.inds = torch.zeros((len(layers), n, K), dtype=torch.int32, device=self.device)
        self.scores = torch.zeros((len(layers), n, K), dtype=torch.bfloat16, device=self.device)
        # per layer: row normalisation, router, dispatch, gate/up + down (or the grouped GEMMs'
        # bucketing, gather, gate/up, down), combine
        self.launches_per_step = (9 if T >= 32 else 6) * len(layers)
        self.graph = None
        self.stream = torch.cuda.Stream(self.device)
        if use_graph:
            self._capture()

    def _layers_once(self) -> torch.Tensor:
        h = self.x[:self.n]
        for li, ly in enumerate(self.layers):
            o = dict(y=self.hs[li & 1][:self.n], inds=self.inds[li][:self.n], scores=self.scores[li][:self.n])
            ep_a2a_layer(h, ly, self.E, self.e_first, self.K, self.T, self.xbuf, norm=self.norm, resid=h, out=o,
                         workspace=self.ws, stream=torch.cuda.current_stream(self.device))
            h = o["y"]
        return h

    def _capture(self) -> None:
        self._layers_once()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.out = self._layers_once()
        self.graph = g

    def step_device(self, x_local: torch.Tensor) -> torch.Tensor:
        """One step of this rank's tokens x_local [n, H] (device); returns their outputs."""
        self.x[:self.n].copy_(x_local)
        if self.graph is not None:
            self.graph.replay()
            return self.out
        return self._layers_once()

    def decode(self, h_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """End to end for this rank's tokens: (pinned) host rows in, host rows out, synchronised."""
        self.x[:self.n].copy_(h_host, non_blocking=True)
        y = self.step_device(self.x[:self.n])
        out_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_host

    def close(self) -> None:
        self.graph = None
        self.xbuf.close()
