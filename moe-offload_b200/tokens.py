"""Token loop around the MoE stack: embedding lookup, LM head, next-token choice and the
decode loop that drives them (the step after the routed block in the reference:
mlx-qwen38/server.py:93-110 `_sample_next_token`, server.py:113-199 `_generate_stream_impl`,
loader.py:1125-1244 `generate_greedy`).

The reference runs a Qwen3.8 checkpoint's embedding, attention layers and LM head in MLX; none
of them exist here, so `TokenHead.synthetic` builds seeded bf16 tables of the model's shape
(vocabulary V, hidden H) and the loop runs token ids -> embedding rows -> the routed-expert
stack -> LM head -> next id, every step on the GPU through libmoe_b200 (moe_embed_tokens,
moe_lm_head_argmax for greedy steps, moe_lm_head_logits + moe_sample_tokens for sampled ones). `ByteTokenizer` stands in for the tokenizer: ids
0..255 are UTF-8 bytes, `eos_id` ends a generation.
"""
from __future__ import annotations

import time
from typing import Any, Iterable, Iterator

import torch

from ._lib import call
from .ops import _need, _stream


class ByteTokenizer:
    """ids 0..255 <-> bytes; eos_id (default V - 1) is the stop token."""

    def __init__(self, vocab_size: int, eos_id: int | None = None):
        if vocab_size < 257:
            raise ValueError("the byte tokenizer needs a vocabulary of at least 257 ids")
        self.vocab_size = vocab_size
        self.eos_token_id = vocab_size - 1 if eos_id is None else int(eos_id)

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: Iterable[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")


class TokenHead:
    """Embedding table and LM head, bf16 [V, H] on the device (head None: tied to the embedding)."""

    def __init__(self, embed: torch.Tensor, head: torch.Tensor | None = None):
        _need(embed, "embed", (torch.bfloat16,))
        self.embed_w = embed
        self.head_w = embed if head is None else head
        _need(self.head_w, "head", (torch.bfloat16,), embed.device)
        self.V, self.H = embed.shape
        if tuple(self.head_w.shape) != (self.V, self.H):
            raise ValueError("embedding and head shapes differ")
        self.device = embed.device
        self._ws = None
        self._best = None

    @classmethod
    def synthetic(cls, vocab_size: int, hidden: int, device, seed: int = 7, embed_std: float = 1.0,
                  head_std: float = 0.02) -> "TokenHead":
        """Seeded N(0, embed_std) embedding rows and N(0, head_std) head rows, bf16."""
        dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        emb = (torch.randn((vocab_size, hidden), generator=g, device=dev) * embed_std).to(torch.bfloat16)
        head = (torch.randn((vocab_size, hidden), generator=g, device=dev) * head_std).to(torch.bfloat16)
        return cls(emb, head)

    @property
    def head_bytes(self) -> int:
        return self.V * self.H * 2

    def embed(self, ids: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """ids int32 [T] (device) -> bf16 [T, H]."""
        _need(ids, "ids", (torch.int32,), self.device)
        T = ids.numel()
        if out is None:
            out = torch.empty((T, self.H), dtype=torch.bfloat16, device=self.device)
        call("moe_embed_tokens", self.embed_w.data_ptr(), self.V, self.H, ids.data_ptr(), T, out.data_ptr(),
             _stream(stream))
        return out

    def logits(self, h: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """h bf16 [T, H] (T <= 4) -> fp32 [T, V]."""
        _need(h, "h", (torch.bfloat16,), self.device)
        T = h.shape[0]
        if out is None:
            out = torch.empty((T, self.V), dtype=torch.float32, device=self.device)
        call("moe_lm_head_logits", self.head_w.data_ptr(), self.V, self.H, h.data_ptr(), T, out.data_ptr(),
             _stream(stream))
        return out

    def argmax(self, h: torch.Tensor, out: torch.Tensor | None = None, logits: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
        """h bf16 [T, H] -> int32 [T] greedy next ids, the LM head and the argmax in one pass
        (logits, when given, also receives the fp32 logits)."""
        _need(h, "h", (torch.bfloat16,), self.device)
        T = h.shape[0]
        if out is None:
            out = torch.empty((T,), dtype=torch.int32, device=self.device)
        need = int(call("moe_lm_head_argmax_workspace_bytes", T))
        if self._best is None or self._best.numel() * 8 < need:
            self._best = torch.zeros(max(4, T), dtype=torch.int64, device=self.device)
        call("moe_lm_head_argmax", self.head_w.data_ptr(), self.V, self.H, h.data_ptr(), T,
             None if logits is None else logits.data_ptr(), out.data_ptr(), self._best.data_ptr(),
             self._best.numel() * 8, _stream(stream))
        return out

    def sample(self, logits: torch.Tensor, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0,
               counter: int = 0, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """fp32 [T, V] -> int32 [T] next ids (argmax when temperature <= 0)."""
        _need(logits, "logits", (torch.float32,), self.device)
        T, V = logits.shape
        if out is None:
            out = torch.empty((T,), dtype=torch.int32, device=self.device)
        need = int(call("moe_sample_workspace_bytes", T, V))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        call("moe_sample_tokens", logits.data_ptr(), T, V, float(temperature), float(top_p),
             int(seed) & 0xFFFFFFFFFFFFFFFF, int(counter) & 0xFFFFFFFFFFFFFFFF, out.data_ptr(), self._ws.data_ptr(),
             self._ws.numel(), _stream(stream))
        return out


def generate_stream(stack, head: TokenHead, prompt_ids: list[int], max_tokens: int, temperature: float = 0.0,
                    top_p: float = 1.0, stop_ids: Iterable[int] | None = None, seed: int = 0,
                    timings: dict[str, Any] | None = None) -> Iterator[int]:
    """server.py:113-199 as a token-id generator over `stack` (anything with prefill(rows [T, H])
    -> [T, H] and decode_token(h [1, H]) -> [1, H], e.g. offload.OffloadStack): prefill of the
    prompt's embedding rows, the next id from the last row's logits, then one decode step per
    yielded id until max_tokens, a stop id, or the caller stops iterating. `timings` receives
    prefill_s, decode_s, decode_tok_per_s, stopped_by_token (the reference's keys). Each step
    reads its id back to the host (the stop test), as the reference does."""
    stop_set = set(int(x) for x in stop_ids) if stop_ids is not None else set()
    tm = timings if timings is not None else {}
    tm.update({"prefill_s": 0.0, "decode_s": 0.0, "decode_tok_per_s": 0.0, "stopped_by_token": False})
    if max_tokens <= 0:
        return
    if not prompt_ids:
        raise ValueError("empty prompt")
    dev = head.device
    t0 = time.perf_counter()
    ids = torch.tensor(list(prompt_ids), dtype=torch.int32).to(dev, non_blocking=True)
    rows = head.embed(ids)
    out = stack.prefill(rows)
    greedy = not temperature > 0.0
    logits = head.logits(out[-1:].contiguous())
    cur = head.sample(logits, temperature, top_p, seed, 0)
    tok = int(cur.item())
    tm["prefill_s"] = round(time.perf_counter() - t0, 4)
    n = 0
    t_dec0 = time.perf_counter()
    try:
        for d in range(max_tokens):
            if tok in stop_set:
                tm["stopped_by_token"] = True
                break
            n += 1
            yield tok
            if d + 1 >= max_tokens:
                break
            y = stack.decode_token(head.embed(cur))
            if greedy:
                head.argmax(y, out=cur)
            else:
                head.logits(y, out=logits)
                head.sample(logits, temperature, top_p, seed, d + 1, out=cur)
            tok = int(cur.item())
    finally:
        dec = max(1e-6, time.perf_counter() - t_dec0)
        tm["decode_s"] = round(dec, 4)
        tm["decode_tok_per_s"] = round(n / dec, 3)


class ResidentTokenLoop:
    """Greedy / sampled decode over a resident stack.PersistentStack, one CUDA graph per token:
    embedding row -> the persistent stack launch -> LM head -> next id, with the id copied to a
    pinned host word (the only per-token transfer). `step()` returns that id."""

    def __init__(self, stack, head: TokenHead, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0):
        self.stack, self.head = stack, head
        self.temperature, self.top_p, self.seed = float(temperature), float(top_p), int(seed)
        dev = head.device
        self.cur = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.logits = torch.empty((1, head.V), dtype=torch.float32, device=dev)
        self.host_id = torch.zeros((1,), dtype=torch.int32, pin_memory=True)
        self.counter = 0
        self.graph = None
        self._graph_failed = False
        # embed, stack, head (+ the argmax's id kernel when greedy) / head + sample
        self.launches_per_step = 4

    def _body(self) -> None:
        self.head.embed(self.cur, out=self.stack.x_in)
        self.stack.step_device()
        if self.temperature <= 0.0:
            self.head.argmax(self.stack.y, out=self.cur)
        else:
            # the counter of a captured step would be fixed at capture: a sampled loop runs uncaptured
            self.head.logits(self.stack.y, out=self.logits)
            self.head.sample(self.logits, self.temperature, self.top_p, self.seed, self.counter, out=self.cur)
        self.host_id.copy_(self.cur, non_blocking=True)

    def start(self, token_id: int) -> None:
        self.cur.fill_(int(token_id))
        self.counter = 0

    def _capture(self) -> None:
        cur = torch.cuda.current_stream(self.head.device)
        s = torch.cuda.Stream(device=self.head.device)
        s.wait_stream(cur)
        try:
            with torch.cuda.stream(s):
                save = self.cur.clone()
                self._body()                                      # warm-up outside the graph
                self.cur.copy_(save)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._body()
            self.graph = g
        except RuntimeError:
            # a driver that cannot capture the cooperative stack launch: run the step directly
            self._graph_failed = True
            torch.cuda.synchronize(self.head.device)
        cur.wait_stream(s)

    def step(self) -> int:
        self.counter += 1
        if self.temperature <= 0.0 and self.graph is None and not self._graph_failed:
            self._capture()
        if self.temperature <= 0.0 and self.graph is not None:
            self.graph.replay()
        else:
            self._body()
        torch.cuda.current_stream(self.head.device).synchronize()
        return int(self.host_id.item())
