"""Numpy restatement of the reference's paged-KV hot path -- TEST INFRASTRUCTURE.

This module is the parity oracle. It restates, on the CPU, what the
reference (cartesia-ai/minimal-inference) computes on its paged path:

* RoPE with the reference's rounding (``model.py:92-107``): every op
  (``x*cos``, ``rot*sin``, the sum) is rounded to the storage dtype.
* Paged KV append with FlashInfer's address arithmetic (the reference calls
  ``flashinfer.page.append_paged_kv_cache`` at ``model.py:207-216``; the
  addressing is ``page.cuh:259-283`` of flashinfer-python 0.6.11.post2):
  ``(page_iter, slot) = divmod(indptr[b]*ps + pos, ps)``.
* Paged decode / prefill attention: fp32 softmax attention over the pages a
  request owns, ``kv_len = (npages-1)*ps + last_page_len`` (0 pages -> 0),
  the same math as the reference's SDPA path (``model.py:286-295``).
  Prefill masking is causal, aligned bottom-right (query ``i`` of ``qo_len``
  sees keys ``j <= kv_len - qo_len + i``), as FlashInfer's causal prefill and
  the reference's explicit mask (``model.py:408-420``) both do.
* The page pool: FIFO free list with page ``P-1`` reserved as the scratch page
  (``scheduler.py:191-221``), CSR metadata (``scheduler.py:267-302``) and the
  CUDA-graph lane padding (``scheduler.py:881-896``) with the intended
  scratch-page semantics for padded lanes.

Nothing here is imported by the product package; ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use it as the checker
and as the timed CPU baseline.
"""
from __future__ import annotations

import math
from collections import deque

import numpy as np

# --------------------------------------------------------------------------
# dtype emulation
# --------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even), as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, x, out)
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ("float32", "float16", "bfloat16")."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_round(x)
    raise ValueError(f"unsupported dtype {dtype!r}")


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


# --------------------------------------------------------------------------
# RoPE  (model.py:79-107)
# --------------------------------------------------------------------------


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """Rotate-half RoPE with the reference's three roundings.

    ``x``: ``[..., D]`` values representable in ``dtype``; ``cos``/``sin``:
    broadcastable ``[..., D]`` table rows (already in ``dtype``). Follows
    ``model.py:101-107``: ``x*cos + cat(-x2, x1)*sin`` where torch rounds each
    elementwise result to the tensor dtype. Products of two bf16/fp16 values
    are exact in fp32, so one fp32 multiply + one rounding reproduces torch.
    """
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = round_to(x * cos, dtype)
    b = round_to(rot * sin, dtype)
    return round_to(a + b, dtype)


# --------------------------------------------------------------------------
# Paged KV append  (model.py:199-216 -> flashinfer page.cuh:259-283)
# --------------------------------------------------------------------------


def append_targets(batch_indices, positions, kv_indices, kv_indptr, page_size,
                   scratch_page: int | None = None):
    """Page id and slot of every appended token.

    ``(page_iter, slot) = divmod(indptr[b]*ps + pos, ps)``, page =
    ``indices[page_iter]``. With ``scratch_page`` given, a token whose
    ``page_iter`` lies outside its request's page range ``[indptr[b],
    indptr[b+1])`` goes to the scratch page: the intended behaviour of padded
    CUDA-graph lanes (``scheduler.py:366-369``).
    """
    bi = np.asarray(batch_indices, dtype=np.int64)
    pos = np.asarray(positions, dtype=np.int64)
    indptr = np.asarray(kv_indptr, dtype=np.int64)
    indices = np.asarray(kv_indices, dtype=np.int64)
    flat = indptr[bi] * page_size + pos
    page_iter, slot = np.divmod(flat, page_size)
    if scratch_page is None:
        pages = indices[page_iter]
    else:
        inside = page_iter < indptr[bi + 1]
        safe = np.where(inside, page_iter, 0)
        pages = np.where(inside, indices[safe] if indices.size else 0, scratch_page)
    return pages.astype(np.int64), slot.astype(np.int64)


def append_paged_kv(kv_data: np.ndarray, append_key, append_value, batch_indices,
                    positions, kv_indices, kv_indptr, page_size,
                    scratch_page: int | None = None) -> None:
    """In-place append into ``kv_data[P, 2, ps, Hkv, D]`` (NHD, K at index 0)."""
    pages, slots = append_targets(batch_indices, positions, kv_indices, kv_indptr,
                                  page_size, scratch_page)
    # Sequential semantics: a later token overwrites an earlier one at the same
    # slot (only padded lanes sharing the scratch page can collide).
    for i in range(len(pages)):
        kv_data[pages[i], 0, slots[i]] = append_key[i]
        kv_data[pages[i], 1, slots[i]] = append_value[i]


def append_paged_kv_rope(kv_data, key_raw, append_value, batch_indices, positions,
                         kv_indices, kv_indptr, page_size, cos_table, sin_table,
                         dtype: str, rope_positions=None, scratch_page=None):
    """Append with RoPE applied to K first (model.py:170 then :207-216)."""
    rp = positions if rope_positions is None else rope_positions
    rp = np.asarray(rp, dtype=np.int64)
    k = apply_rope(key_raw, cos_table[rp][:, None, :], sin_table[rp][:, None, :], dtype)
    append_paged_kv(kv_data, k, append_value, batch_indices, positions, kv_indices,
                    kv_indptr, page_size, scratch_page)
    return k


# --------------------------------------------------------------------------
# Paged attention
# --------------------------------------------------------------------------


def kv_length(kv_indptr, kv_last_page_len, page_size, b) -> int:
    """FlashInfer ``paged_kv_t::get_length`` (page.cuh:147-152)."""
    n = int(kv_indptr[b + 1]) - int(kv_indptr[b])
    if n == 0:
        return 0
    return (n - 1) * page_size + int(kv_last_page_len[b])


def gather_kv(kv_data, kv_indptr, kv_indices, kv_last_page_len, page_size, b):
    """Contiguous ``[kv_len, Hkv, D]`` K and V of request ``b``."""
    pages = np.asarray(kv_indices[int(kv_indptr[b]):int(kv_indptr[b + 1])], dtype=np.int64)
    n = len(pages)
    _, _, ps, hkv, d = kv_data.shape
    if n == 0:
        z = np.zeros((0, hkv, d), np.float32)
        return z, z
    kv_len = kv_length(kv_indptr, kv_last_page_len, page_size, b)
    k = kv_data[pages, 0].reshape(n * ps, hkv, d)[:kv_len].astype(np.float32)
    v = kv_data[pages, 1].reshape(n * ps, hkv, d)[:kv_len].astype(np.float32)
    return k, v


def _attend(q, k, v, sm_scale, mask=None):
    """q [Lq, Hkv, g, D], k/v [Lk, Hkv, D] -> out [Lq, Hkv, g, D], lse [Lq, Hkv, g]."""
    s = np.einsum("qhgd,khd->qhgk", q, k, optimize=True).astype(np.float32) * np.float32(sm_scale)
    if mask is not None:
        s = np.where(mask[:, None, None, :], s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    den = p.sum(axis=-1, keepdims=True)
    out = np.einsum("qhgk,khd->qhgd", p, v, optimize=True) / np.where(den > 0, den, 1.0)
    with np.errstate(divide="ignore"):
        lse = (np.log(den) + m)[..., 0]
    return out.astype(np.float32), lse.astype(np.float32)


def decode_attention(q, kv_data, kv_indptr, kv_indices, kv_last_page_len, page_size,
                     sm_scale: float | None = None):
    """Single-query attention per request over its pages.

    ``q``: ``[B, Hq, D]``; query head ``i`` reads KV head ``i // (Hq/Hkv)``
    (``repeat_interleave`` at ``model.py:287-288``). Returns ``out [B, Hq, D]``
    (fp32) and the natural-log ``lse [B, Hq]``; a request with 0 pages yields
    zeros and ``-inf``.
    """
    q = np.asarray(q, dtype=np.float32)
    bsz, hq, d = q.shape
    hkv = kv_data.shape[3]
    g = hq // hkv
    scale = d ** -0.5 if sm_scale is None else sm_scale
    out = np.zeros((bsz, hq, d), np.float32)
    lse = np.full((bsz, hq), -np.inf, np.float32)
    for b in range(bsz):
        k, v = gather_kv(kv_data, kv_indptr, kv_indices, kv_last_page_len, page_size, b)
        if k.shape[0] == 0:
            continue
        o, l = _attend(q[b].reshape(1, hkv, g, d), k, v, scale)
        out[b] = o.reshape(hq, d)
        lse[b] = l.reshape(hq)
    return out, lse


def prefill_attention(q, qo_indptr, kv_data, kv_indptr, kv_indices, kv_last_page_len,
                      page_size, causal: bool = True, sm_scale: float | None = None):
    """Ragged prefill attention: ``q [nnz, Hq, D]`` split by ``qo_indptr``."""
    q = np.asarray(q, dtype=np.float32)
    nnz, hq, d = q.shape
    hkv = kv_data.shape[3]
    g = hq // hkv
    scale = d ** -0.5 if sm_scale is None else sm_scale
    out = np.zeros((nnz, hq, d), np.float32)
    lse = np.full((nnz, hq), -np.inf, np.float32)
    for b in range(len(qo_indptr) - 1):
        q0, q1 = int(qo_indptr[b]), int(qo_indptr[b + 1])
        if q1 == q0:
            continue
        k, v = gather_kv(kv_data, kv_indptr, kv_indices, kv_last_page_len, page_size, b)
        kv_len, qo_len = k.shape[0], q1 - q0
        if kv_len == 0:
            continue
        mask = None
        if causal:
            qi = np.arange(qo_len)[:, None]
            kj = np.arange(kv_len)[None, :]
            mask = kj <= (kv_len - qo_len + qi)
        o, l = _attend(q[q0:q1].reshape(qo_len, hkv, g, d), k, v, scale, mask)
        out[q0:q1] = o.reshape(qo_len, hq, d)
        lse[q0:q1] = l.reshape(qo_len, hq)
    return out, lse


# --------------------------------------------------------------------------
# Page pool, CSR metadata, graph padding  (scheduler.py)
# --------------------------------------------------------------------------


class PagePoolOracle:
    """FIFO page pool of ``PagedKVCache`` (scheduler.py:168-221).

    ``max_num_pages = max_batch * ceil(max_seq/ps)`` (:191-192); page
    ``P-1`` is the scratch page (:204-205); the free list starts as
    ``0..P-2`` in order (:206); allocation pops from the left and raises
    ``RuntimeError`` when short (:208-214); release appends to the right
    (:216-221).
    """

    def __init__(self, max_batch_size: int, max_seq_len: int, page_size: int):
        self.page_size = page_size
        self.max_num_pages = max_batch_size * math.ceil(max_seq_len / page_size)
        self.scratch_page = self.max_num_pages - 1
        self.free_pages: deque[int] = deque(range(self.max_num_pages - 1))

    def allocate_pages(self, num_pages: int) -> list[int]:
        if len(self.free_pages) < num_pages:
            raise RuntimeError(
                f"Cannot allocate {num_pages} pages, only {len(self.free_pages)} free")
        return [self.free_pages.popleft() for _ in range(num_pages)]

    def release_pages(self, page_indices) -> None:
        for idx in page_indices:
            self.free_pages.append(int(idx))


def zero_pages(kv_layers, page_indices) -> None:
    """Zero-on-release of every layer's copy of each page (scheduler.py:218-220)."""
    for idx in page_indices:
        for layer in kv_layers:
            layer[idx] = 0


def build_csr(page_lists, seq_lens, page_size):
    """``build_csr_metadata`` (scheduler.py:267-302) as int32 numpy arrays."""
    indptr = [0]
    flat: list[int] = []
    last: list[int] = []
    for pages, seq_len in zip(page_lists, seq_lens):
        flat.extend(int(p) for p in pages)
        indptr.append(len(flat))
        ll = seq_len % page_size
        if ll == 0 and seq_len > 0:
            ll = page_size
        last.append(ll)
    return (np.asarray(indptr, np.int32), np.asarray(flat, np.int32),
            np.asarray(last, np.int32))


def pad_decode_batch(indptr, indices, last_page_len, positions, padded_bs: int,
                     scratch_page: int, indices_capacity: int):
    """Graph-bucket padding of decode metadata (scheduler.py:881-902).

    Padded lanes repeat the last ``indptr`` value (0 pages), get
    ``last_page_len = 1`` and position 0; ``batch_indices = arange(padded_bs)``.
    The static ``indices`` buffer holds the scratch page past the real prefix
    -- the intended semantics of scheduler.py:366-369, so a padded lane's
    append lands on the scratch page.
    """
    bs = len(last_page_len)
    pad = padded_bs - bs
    indptr_p = np.concatenate([indptr, np.full(pad, indptr[-1], np.int32)]).astype(np.int32)
    last_p = np.concatenate([last_page_len, np.ones(pad, np.int32)]).astype(np.int32)
    pos_p = np.concatenate([positions, np.zeros(pad, np.int32)]).astype(np.int32)
    ind_p = np.full(indices_capacity, scratch_page, np.int32)
    ind_p[:len(indices)] = indices
    batch_indices = np.arange(padded_bs, dtype=np.int32)
    return indptr_p, ind_p, last_p, pos_p, batch_indices


GRAPH_BATCH_SIZES = [1, 2, 4, 8, 16, 32, 48, 64]  # scheduler.py:350


def graph_bucket(batch_size: int) -> int:
    """Smallest captured bucket >= batch_size, or 0 (scheduler.py:882)."""
    return next((bs for bs in GRAPH_BATCH_SIZES if bs >= batch_size), 0)


# --------------------------------------------------------------------------
# Scheduler page-table trace (scheduler.py:589-600, 624-637, 835-847, 984-1003)
# --------------------------------------------------------------------------


def simulate_page_tables(prompt_lens, max_new_tokens, max_batch_size: int,
                         max_seq_len: int, page_size: int):
    """Page tables the reference's paged scheduler produces, step by step.

    Requests are all queued at t=0 in order; tokens never hit EOS, so every
    request runs ``max_new_tokens`` tokens (the prefill token counts,
    ``scheduler.py:750``) or until ``current_position >= max_seq_len``
    (:973). Returns a list of steps; each step is a dict with the admitted
    requests, the decode CSR metadata (or None) and the released pages.
    """
    pool = PagePoolOracle(max_batch_size, max_seq_len, page_size)
    waiting = deque(range(len(prompt_lens)))
    active: list[dict] = []
    trace = []
    while waiting or active:
        step = {"admitted": [], "decode": None, "released": []}
        # admit: head-of-line, prompt pages only (scheduler.py:624-637)
        while waiting and len(active) < max_batch_size:
            rid = waiting[0]
            need = math.ceil(prompt_lens[rid] / page_size)
            if len(pool.free_pages) < need:
                break
            waiting.popleft()
            r = {"id": rid, "pages": pool.allocate_pages(need), "status": "prefill",
                 "pos": 0, "ntok": 0}
            active.append(r)
            step["admitted"].append((rid, list(r["pages"])))
        if not active and waiting:
            raise RuntimeError("request can never be admitted: pool too small")
        # prefill (scheduler.py:684-752): one token, position = prompt_len
        for r in active:
            if r["status"] != "prefill":
                continue
            r["pos"] = prompt_lens[r["id"]]
            r["ntok"] = 1
            r["status"] = "decode"
            if r["ntok"] >= max_new_tokens[r["id"]]:
                r["status"] = "finished"
        # decode (scheduler.py:835-978)
        dec = [r for r in active if r["status"] == "decode"]
        if dec:
            for r in dec:
                need = math.ceil((r["pos"] + 1) / page_size)
                if need > len(r["pages"]):
                    r["pages"].extend(pool.allocate_pages(need - len(r["pages"])))
            indptr, indices, last = build_csr([r["pages"] for r in dec],
                                              [r["pos"] + 1 for r in dec], page_size)
            step["decode"] = {
                "ids": [r["id"] for r in dec],
                "positions": [r["pos"] for r in dec],
                "indptr": indptr.tolist(), "indices": indices.tolist(),
                "last_page_len": last.tolist(),
            }
            for r in dec:
                r["ntok"] += 1
                r["pos"] += 1
                if r["ntok"] >= max_new_tokens[r["id"]] or r["pos"] >= max_seq_len:
                    r["status"] = "finished"
        # retire in active order (scheduler.py:984-1003)
        still = []
        for r in active:
            if r["status"] == "finished":
                pool.release_pages(r["pages"])
                step["released"].append((r["id"], list(r["pages"])))
            else:
                still.append(r)
        active = still
        trace.append(step)
    return trace
