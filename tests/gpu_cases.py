"""Seeded inputs shared by the GPU parity tests and smoke()."""
from __future__ import annotations

import math

import numpy as np

from oracle import paged_oracle as po


def random_page_tables(rng, lens, page_size, num_pages):
    """Disjoint, non-contiguous page lists (a seeded permutation of the pool)."""
    need = [math.ceil(L / page_size) for L in lens]
    assert sum(need) <= num_pages - 1, "pool too small"
    perm = rng.permutation(num_pages - 1)
    out, k = [], 0
    for n in need:
        out.append(perm[k:k + n].tolist())
        k += n
    return out


def paged_case(seed, lens, hq, hkv, d, page_size=16, dtype="bfloat16", num_pages=None,
               scale=1.0):
    """A pool with random contents, random page tables and random queries."""
    rng = np.random.default_rng(seed)
    npages = sum(math.ceil(L / page_size) for L in lens)
    P = num_pages or (npages + 9)
    tables = random_page_tables(rng, lens, page_size, P)
    indptr, indices, last = po.build_csr(tables, lens, page_size)
    # only pages that belong to a request get data; the rest (scratch included)
    # stay zero, as in a fresh pool. Rounded in blocks to bound host memory.
    pool = np.zeros((P, 2, page_size, hkv, d), np.float32)
    used = np.asarray([p for t in tables for p in t], np.int64)
    for k in range(0, len(used), 256):
        blk = used[k:k + 256]
        pool[blk] = po.round_to(
            rng.standard_normal((len(blk), 2, page_size, hkv, d), dtype=np.float32) * scale, dtype)
    q = po.round_to(rng.standard_normal((len(lens), hq, d), dtype=np.float32), dtype)
    return dict(pool=pool, q=q, indptr=indptr, indices=indices, last=last, tables=tables,
                P=P, lens=list(lens), ps=page_size, hq=hq, hkv=hkv, d=d, dtype=dtype)


def config2_lens(seed=0, batch=32, lo=256, hi=4096):
    """Context lengths of BASELINE config 2 (uniform in [256, 4096])."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=batch).tolist()
