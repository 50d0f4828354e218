"""Continuous-batching scheduler on the B200 paged-KV path.

Keeps the reference scheduler's contract (scheduler.py:477-1009): requests
are admitted head-of-line while a batch slot and the prompt's pages are free
(:624-637), prefilled, decoded one token per step with a page allocated when
a request crosses a page boundary (:842-847), and retired -- their pages
zeroed in every layer and returned to the free list in order (:984-1003).
A request finishes on EOS, on ``max_new_tokens`` (the prefill token counts)
or when ``current_position`` reaches ``max_seq_len`` (:970-978). Tokens go
back through each request's asyncio queue (:1005-1009).

What differs is where the work runs:

* the page pool, page tables and CSR metadata live on the GPU
  (``PagedKVCache`` slot API); a decode step's page growth and CSR building
  are one kernel inside the step's CUDA graph, so the host only uploads each
  lane's (slot, position, last token) -- one small copy -- and replays;
* prefill is batched: every request admitted in a step is prefilled in one
  ragged forward (``qo_indptr``), computing logits only for each request's
  last token;
* decode graphs are captured per batch bucket {1,2,4,8,16,32,48,64}
  (:350); padding lanes carry slot -1, so their append lands on the scratch
  page and their attention is empty.
"""
from __future__ import annotations

import asyncio
import enum
import logging
import math
import threading
import time
from collections import deque
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .decode import BatchDecodeWithPagedKVCacheWrapper
from .kv_cache import PagedKVCache
from .prefill import BatchPrefillWithPagedKVCacheWrapper

logger = logging.getLogger(__name__)

EOS_TOKEN_IDS: set[int] = {151645, 151643}
GRAPH_BATCH_SIZES = [1, 2, 4, 8, 16, 32, 48, 64]


class RequestStatus(enum.Enum):
    WAITING = "waiting"
    PREFILLING = "prefilling"
    DECODING = "decoding"
    FINISHED = "finished"


@dataclass
class Request:
    request_id: str
    input_ids: list[int]
    max_new_tokens: int
    temperature: float
    status: RequestStatus = RequestStatus.WAITING
    generated_tokens: list[int] = field(default_factory=list)
    current_position: int = 0
    batch_slot: int = -1
    pages: list[int] = field(default_factory=list)  # filled on demand (debug/tests)
    finish_reason: str | None = None
    prefill_done_time: float = 0.0
    last_token_time: float = 0.0
    token_queue: asyncio.Queue = field(default_factory=asyncio.Queue)
    loop: asyncio.AbstractEventLoop | None = None


class AttentionBackend:
    """What the model's attention layers need for one forward (scheduler.py:229-259).

    Holds the paged cache, the planned wrapper, the CSR page table, the
    append token map and per-forward scratch buffers; ``next_layer()``
    walks the layers.
    """

    def __init__(self, paged_kv_cache, wrapper, mode, kv_page_indptr, kv_page_indices,
                 kv_last_page_len, append_indptr, batch_indices, positions, status=None,
                 q_buf=None, out_buf=None):
        self.paged_kv_cache = paged_kv_cache
        self.wrapper = wrapper
        self.mode = mode
        self.kv_page_indptr = kv_page_indptr
        self.kv_page_indices = kv_page_indices
        self.kv_last_page_len = kv_last_page_len
        self.append_indptr = append_indptr
        self.batch_indices = batch_indices
        self.positions = positions
        self.status = status if status is not None else paged_kv_cache.status
        self.rope_cos = self.rope_sin = None
        self._q_buf, self._out_buf = q_buf, out_buf
        self._layer_idx = 0

    def next_layer(self) -> int:
        idx = self._layer_idx
        self._layer_idx += 1
        return idx

    def q_buffer(self, n, hq, d, dtype):
        if self._q_buf is None or self._q_buf.shape[0] < n:
            self._q_buf = torch.empty(n, hq, d, dtype=dtype, device=self.positions.device)
        return self._q_buf[:n]

    def out_buffer(self, n, hq, d, dtype):
        if self._out_buf is None or self._out_buf.shape[0] < n:
            self._out_buf = torch.empty(n, hq, d, dtype=dtype, device=self.positions.device)
        return self._out_buf[:n]


def build_csr_metadata(page_lists, seq_lens, page_size, device):
    """CSR page table from host lists (scheduler.py:267-302)."""
    indptr, flat, last = [0], [], []
    for pages, seq_len in zip(page_lists, seq_lens):
        flat.extend(pages)
        indptr.append(len(flat))
        ll = seq_len % page_size
        if ll == 0 and seq_len > 0:
            ll = page_size
        last.append(ll)
    mk = lambda x: torch.tensor(x, dtype=torch.int32, device=device)  # noqa: E731
    return mk(indptr), mk(flat), mk(last)


def sample(logits: torch.Tensor, temperature: float) -> int:
    """Sample from ``logits[1, S, V]`` (scheduler.py:310-316)."""
    if temperature <= 0:
        return int(logits[0, -1].argmax(dim=-1).item())
    probs = F.softmax(logits[0, -1] / temperature, dim=-1)
    return int(torch.multinomial(probs, num_samples=1).item())


def sample_rows(last_logits: torch.Tensor, temperatures: list[float]) -> torch.Tensor:
    """Batched sampling of ``[B, V]`` rows on the device (scheduler.py:319-343)."""
    temps = torch.tensor(temperatures, dtype=torch.float32, device=last_logits.device)
    greedy = temps <= 0
    if bool(greedy.all()):
        return last_logits.argmax(dim=-1)
    scaled = last_logits.float() / temps.clamp(min=1e-6).unsqueeze(1)
    sampled = torch.multinomial(F.softmax(scaled, dim=-1), num_samples=1).squeeze(1)
    return torch.where(greedy, last_logits.argmax(dim=-1), sampled)


def sample_batch(logits: torch.Tensor, temperatures: list[float]) -> list[int]:
    return sample_rows(logits[:, -1, :], temperatures).tolist()


class CUDAGraphRunner:
    """One captured decode step for a fixed batch bucket.

    The graph holds the whole step: page growth + CSR (``mi_step_prepare``),
    the model forward with fused append and paged decode per layer, and the
    logits. Inputs are one int32 tensor ``[3, bs]`` (slot, position, last
    token per lane; slot -1 = padding), copied in before each replay.
    """

    def __init__(self, batch_size, kv_cache: PagedKVCache, num_heads, head_dim, dtype, device):
        self.batch_size = bs = batch_size
        i32 = dict(dtype=torch.int32, device=device)
        self.inputs = torch.zeros(3, bs, **i32)
        self.inputs[0].fill_(-1)
        self.host_inputs = torch.zeros(3, bs, dtype=torch.int32).pin_memory()
        self.kv_page_indptr = torch.zeros(bs + 1, **i32)
        self.kv_page_indices = torch.zeros(bs * kv_cache.max_pages_per_seq, **i32)
        self.kv_last_page_len = torch.ones(bs, **i32)
        self.append_positions = torch.zeros(bs, **i32)
        self.batch_indices = torch.arange(bs, **i32)
        self.append_indptr = torch.arange(bs + 1, **i32)
        self.q_buf = torch.empty(bs, num_heads, head_dim, dtype=dtype, device=device)
        self.out_buf = torch.empty(bs, num_heads, head_dim, dtype=dtype, device=device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.logits: torch.Tensor | None = None
        self.kv_cache = kv_cache

    def _step(self, model, backend):
        self.kv_cache.step_prepare(self.inputs[0], self.inputs[1], self.kv_page_indptr,
                                   self.kv_page_indices, self.kv_last_page_len,
                                   self.append_positions, grow=True)
        backend._layer_idx = 0
        ids = self.inputs[2].long().unsqueeze(1)
        return model(ids, position_ids=None, attn_backend=backend)[:, -1, :]

    def capture(self, model, decode_wrapper, config, page_size, dtype):
        backend = AttentionBackend(self.kv_cache, decode_wrapper, "decode", self.kv_page_indptr,
                                   self.kv_page_indices, self.kv_last_page_len,
                                   self.append_indptr, self.batch_indices,
                                   self.append_positions, q_buf=self.q_buf,
                                   out_buf=self.out_buf)
        decode_wrapper.plan(self.kv_page_indptr, self.kv_page_indices, self.kv_last_page_len,
                            model.layers[0].self_attn.num_heads,
                            model.layers[0].self_attn.num_kv_heads, config.head_dim, page_size,
                            q_data_type=dtype)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step(model, backend)
        s.synchronize()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._step(model, backend)
        self._backend = backend

    def replay(self, slots, positions, tokens) -> torch.Tensor:
        n = len(slots)
        h = self.host_inputs
        h[0].fill_(-1)
        h[1].zero_()
        h[2].zero_()
        h[0, :n] = torch.tensor(slots, dtype=torch.int32)
        h[1, :n] = torch.tensor(positions, dtype=torch.int32)
        h[2, :n] = torch.tensor(tokens, dtype=torch.int32)
        self.inputs.copy_(h, non_blocking=True)
        self.graph.replay()
        return self.logits


class Scheduler:
    def __init__(self, model, config, device, dtype, max_batch_size: int = 8,
                 max_seq_len: int = 4096, page_size: int = 16,
                 eos_token_ids: set[int] | None = None, use_flashinfer: bool = True,
                 use_cuda_graph: bool = True, teacher_tokens: dict | None = None,
                 num_kv_heads: int | None = None, num_heads: int | None = None,
                 max_prefill_tokens: int = 32768):
        global EOS_TOKEN_IDS
        if eos_token_ids is not None:
            EOS_TOKEN_IDS = eos_token_ids
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("mi_b200.Scheduler runs on a CUDA device (no CPU fallback)")
        # a model built the way server.py builds it (Model(cfg), load_weights,
        # .to(...).eval()) still has trainable parameters and unfused GEMM
        # weights: this is an inference engine, and the graphs below must
        # capture the fused weights
        model.requires_grad_(False)
        if getattr(model.layers[0].self_attn, "_qkv_wt", None) is None:
            model.prepare()
        self.model, self.config = model, config
        self.device, self.dtype = device, dtype
        self.max_batch_size, self.max_seq_len, self.page_size = max_batch_size, max_seq_len, page_size
        attn0 = model.layers[0].self_attn   # this rank's heads under tensor parallelism
        self.num_heads = num_heads or attn0.num_heads
        self.num_kv_heads = num_kv_heads or attn0.num_kv_heads
        self.max_prefill_tokens = max_prefill_tokens
        self.kv_cache = PagedKVCache(config, max_batch_size, max_seq_len, page_size, device, dtype,
                                     num_kv_heads=self.num_kv_heads)
        ws = 256 * 1024 * 1024
        self._prefill_workspace = torch.empty(ws, dtype=torch.uint8, device=device)
        self._decode_workspace = torch.zeros(ws, dtype=torch.uint8, device=device)
        self._prefill_wrapper = BatchPrefillWithPagedKVCacheWrapper(self._prefill_workspace)
        self._decode_wrapper = BatchDecodeWithPagedKVCacheWrapper(self._decode_workspace)
        self.free_slots = list(range(max_batch_size))
        self.teacher_tokens = teacher_tokens  # request_id -> forced token list (tests)
        self.step_logits: list = []           # (kind, [request ids], logits rows) when recording
        self.record_logits = False
        self._graph_runners: dict[int, CUDAGraphRunner] = {}
        if use_cuda_graph:
            for bs in GRAPH_BATCH_SIZES:
                if bs > max_batch_size:
                    break
                r = CUDAGraphRunner(bs, self.kv_cache, self.num_heads, config.head_dim, dtype,
                                    device)
                r.capture(model, self._decode_wrapper, config, page_size, dtype)
                self._graph_runners[bs] = r
            torch.cuda.synchronize()
            self.kv_cache.check_status()
        self.waiting_queue: deque[Request] = deque()
        self.active_requests: list[Request] = []
        self.lock = threading.Lock()
        self.new_request_event = threading.Event()
        self._running = False
        self._thread: threading.Thread | None = None

    # ---- thread plumbing (scheduler.py:569-600) -----------------------------
    def start(self) -> None:
        self._running = True
        self._thread = threading.Thread(target=self._run_loop, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._running = False
        self.new_request_event.set()
        if self._thread:
            self._thread.join()

    def close(self) -> None:
        """Release the decode CUDA graphs (they hold NCCL work under tensor
        parallelism and must go before the process group is destroyed)."""
        torch.cuda.synchronize(self.device)
        for r in self._graph_runners.values():
            r.graph = None
            r.logits = None
        self._graph_runners.clear()

    def submit_request(self, request: Request) -> None:
        with self.lock:
            self.waiting_queue.append(request)
        self.new_request_event.set()

    def _run_loop(self) -> None:
        while self._running:
            if not self.active_requests and not self.waiting_queue:
                self.new_request_event.wait(timeout=0.1)
                self.new_request_event.clear()
                continue
            self.step()

    def step(self) -> None:
        """One scheduler iteration: admit -> prefill -> decode -> retire."""
        self._admit_new_requests()
        self._prefill_new_requests()
        if any(r.status == RequestStatus.DECODING for r in self.active_requests):
            self._decode_step()
        self._retire_finished_requests()

    # ---- admit (scheduler.py:624-637) -----------------------------------------
    def _admit_new_requests(self) -> None:
        admitted = []
        with self.lock:
            while self.waiting_queue and len(self.active_requests) < self.max_batch_size:
                req = self.waiting_queue[0]
                need = math.ceil(len(req.input_ids) / self.page_size)
                if len(self.kv_cache.free_pages) < need or not self.free_slots:
                    break
                self.waiting_queue.popleft()
                req.batch_slot = self.free_slots.pop(0)
                req.status = RequestStatus.PREFILLING
                self.active_requests.append(req)
                admitted.append((req, need))
        if admitted:
            slots = torch.tensor([r.batch_slot for r, _ in admitted], dtype=torch.int32,
                                 device=self.device)
            counts = torch.tensor([n for _, n in admitted], dtype=torch.int32, device=self.device)
            self.kv_cache.slot_alloc(slots, counts, sum(n for _, n in admitted))

    # ---- prefill (scheduler.py:643-752), batched -----------------------------
    def _prefill_new_requests(self) -> None:
        reqs = [r for r in self.active_requests if r.status == RequestStatus.PREFILLING]
        # one ragged forward per group of at most max_prefill_tokens prompt
        # tokens (a longer prompt goes alone), in admission order
        group, n = [], 0
        for r in reqs:
            if group and n + len(r.input_ids) > self.max_prefill_tokens:
                self._prefill_batch(group)
                group, n = [], 0
            group.append(r)
            n += len(r.input_ids)
        if group:
            self._prefill_batch(group)

    @torch.inference_mode()
    def _prefill_batch(self, reqs: list) -> None:
        dev = self.device
        lens = [len(r.input_ids) for r in reqs]
        total = sum(lens)
        qo = [0]
        for n in lens:
            qo.append(qo[-1] + n)
        i32 = dict(dtype=torch.int32, device=dev)
        ids = torch.tensor([t for r in reqs for t in r.input_ids], dtype=torch.long, device=dev)
        lane_slots = torch.tensor([r.batch_slot for r in reqs], **i32)
        lane_last = torch.tensor([n - 1 for n in lens], **i32)
        b = len(reqs)
        indptr = torch.empty(b + 1, **i32)
        indices = torch.empty(sum(math.ceil(n / self.page_size) for n in lens), **i32)
        last = torch.empty(b, **i32)
        apos_unused = torch.empty(b, **i32)
        self.kv_cache.step_prepare(lane_slots, lane_last, indptr, indices, last, apos_unused,
                                   grow=False)
        qo_t = torch.tensor(qo, **i32)
        batch_indices = torch.repeat_interleave(torch.arange(b, **i32),
                                                torch.tensor(lens, device=dev))
        positions = torch.cat([torch.arange(n, **i32) for n in lens])
        self._prefill_wrapper.plan(qo_t, indptr, indices, last, self.num_heads,
                                   self.num_kv_heads, self.config.head_dim, self.page_size,
                                   causal=True, q_data_type=self.dtype)
        backend = AttentionBackend(self.kv_cache, self._prefill_wrapper, "prefill", indptr,
                                   indices, last, qo_t, batch_indices, positions)
        last_rows = qo_t[1:].long() - 1                  # each request's last token
        rows = self.model(ids.unsqueeze(0), position_ids=None, attn_backend=backend,
                          logits_rows=last_rows)[0]
        if self.record_logits:
            self.step_logits.append(("prefill", [r.request_id for r in reqs], rows.float().cpu()))
        next_tokens = sample_rows(rows, [r.temperature for r in reqs]).tolist()
        now = time.perf_counter()
        for req, n, tok in zip(reqs, lens, next_tokens):
            tok = self._forced(req, tok)
            req.generated_tokens.append(tok)
            req.current_position = n
            req.status = RequestStatus.DECODING
            req.prefill_done_time = req.last_token_time = now
            self._push_token(req, tok)
            if tok in EOS_TOKEN_IDS or len(req.generated_tokens) >= req.max_new_tokens:
                req.status = RequestStatus.FINISHED
                req.finish_reason = "stop" if tok in EOS_TOKEN_IDS else "length"

    def _forced(self, req, tok: int) -> int:
        if self.teacher_tokens and req.request_id in self.teacher_tokens:
            seq = self.teacher_tokens[req.request_id]
            k = len(req.generated_tokens)
            if k < len(seq):
                return int(seq[k])
        return tok

    # ---- decode (scheduler.py:835-978) ---------------------------------------
    @torch.inference_mode()
    def _decode_step(self) -> None:
        decoding = [r for r in self.active_requests if r.status == RequestStatus.DECODING]
        if not decoding:
            return
        b = len(decoding)
        # pages this step grows (host mirror of the device allocator)
        grow = sum(1 for r in decoding
                   if math.ceil((r.current_position + 1) / self.page_size)
                   > math.ceil(r.current_position / self.page_size))
        if grow > self.kv_cache.num_free_pages:
            raise RuntimeError(
                f"Cannot allocate {grow} pages, only {self.kv_cache.num_free_pages} free")
        self.kv_cache.num_free_pages -= grow
        slots = [r.batch_slot for r in decoding]
        positions = [r.current_position for r in decoding]
        tokens = [r.generated_tokens[-1] for r in decoding]
        bucket = next((bs for bs in GRAPH_BATCH_SIZES if bs >= b), 0)
        runner = self._graph_runners.get(bucket) if bucket else None
        if runner is not None:
            logits = runner.replay(slots, positions, tokens)[:b]
        else:
            logits = self._decode_eager(slots, positions, tokens)
        if self.record_logits:
            self.step_logits.append(("decode", [r.request_id for r in decoding],
                                     logits.float().cpu()))
        next_tokens = sample_rows(logits, [r.temperature for r in decoding]).tolist()
        now = time.perf_counter()
        for req, tok in zip(decoding, next_tokens):
            tok = self._forced(req, tok)
            req.generated_tokens.append(tok)
            req.current_position += 1
            req.last_token_time = now
            self._push_token(req, tok)
            if (tok in EOS_TOKEN_IDS or len(req.generated_tokens) >= req.max_new_tokens
                    or req.current_position >= self.max_seq_len):
                req.status = RequestStatus.FINISHED
                req.finish_reason = "stop" if tok in EOS_TOKEN_IDS else "length"

    def _decode_eager(self, slots, positions, tokens) -> torch.Tensor:
        dev = self.device
        b = len(slots)
        i32 = dict(dtype=torch.int32, device=dev)
        lane_slots = torch.tensor(slots, **i32)
        lane_pos = torch.tensor(positions, **i32)
        indptr = torch.empty(b + 1, **i32)
        indices = torch.empty(b * self.kv_cache.max_pages_per_seq, **i32)
        last = torch.empty(b, **i32)
        apos = torch.empty(b, **i32)
        self.kv_cache.step_prepare(lane_slots, lane_pos, indptr, indices, last, apos, grow=True)
        self._decode_wrapper.plan(indptr, indices, last, self.num_heads, self.num_kv_heads,
                                  self.config.head_dim, self.page_size, q_data_type=self.dtype)
        backend = AttentionBackend(self.kv_cache, self._decode_wrapper, "decode", indptr, indices,
                                   last, torch.arange(b + 1, **i32), torch.arange(b, **i32), apos)
        ids = torch.tensor(tokens, dtype=torch.long, device=dev).unsqueeze(1)
        return self.model(ids, position_ids=None, attn_backend=backend)[:, -1, :]

    # ---- retire (scheduler.py:984-1003) --------------------------------------
    def _retire_finished_requests(self) -> None:
        still, done = [], []
        for req in self.active_requests:
            if req.status == RequestStatus.FINISHED:
                n = len(req.generated_tokens)
                if n > 1 and req.prefill_done_time > 0:
                    t2t = (req.last_token_time - req.prefill_done_time) / (n - 1) * 1000
                    logger.info("Request %s finished: %d tokens, avg token-to-token %.1f ms",
                                req.request_id, n, t2t)
                self._push_token(req, None)
                done.append(req)
            else:
                still.append(req)
        if done:
            # pages held = ceil(current_position / ps): the last sampled token was
            # never appended
            held = sum(math.ceil(r.current_position / self.page_size) for r in done)
            slots = torch.tensor([r.batch_slot for r in done], dtype=torch.int32,
                                 device=self.device)
            self.kv_cache.slot_release(slots, held)
            for r in done:
                self.free_slots.append(r.batch_slot)
            self.free_slots.sort()
        self.active_requests = still

    def _push_token(self, req: Request, token: int | None) -> None:
        if req.loop is not None:
            req.loop.call_soon_threadsafe(req.token_queue.put_nowait, token)
        else:
            req.token_queue.put_nowait(token)
