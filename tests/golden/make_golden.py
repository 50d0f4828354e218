#!/usr/bin/env python
"""Generate the golden fixtures in this directory from the reference itself.

Run on a machine that has a checkout of cartesia-ai/minimal-inference:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

The reference is imported as-is (its ``model.py`` and ``scheduler.py``) and
run on the CPU. Four fixtures come out:

``rope.npz``
    ``apply_rotary_emb`` (model.py:92-107) on seeded inputs for bf16 / fp16 /
    fp32 and head_dim 64 / 128, with the reference's own cos/sin tables
    (``precompute_rope``, model.py:79-89, cast like ``Model.to(dtype)``).
``attn.npz``
    The reference's padded attention path (``Attention._pytorch_attention``,
    model.py:254-298) driven the way the padded scheduler drives it
    (prefill one request at a time, then batched decode with the per-lane
    mask of scheduler.py:793-800), together with the page tables the
    reference ``PagedKVCache`` / ``build_csr_metadata`` (scheduler.py:168-302)
    hand out for the same requests. The oracle must reproduce the outputs and,
    through the page tables, the exact padded-cache contents.
``sched_trace.json``
    The reference ``Scheduler``'s own paged control flow (admit -> prefill ->
    decode -> retire, scheduler.py:589-1003) run on the CPU with a recording
    stand-in for the FlashInfer wrappers; every ``plan()`` call's CSR
    metadata, every admission and every release is recorded. Tokens never hit
    EOS, so the trace depends only on lengths.
``config1.npz``
    the Qwen2.5-0.5B shape in fp32 with seeded N(0, 0.02)
    weights (``mi_b200.weights.init_random_weights``), four requests of
    37/128/255/500 seeded token ids, 50 greedy decode steps through the
    reference ``Scheduler`` on CPU. Stores the generated tokens (the teacher
    sequence for the GPU run), per-step logit digests and per-layer KV digests
    taken just before each request's cache slot is released.
``config1_bf16.npz``
    The same run with the model (weights, RoPE tables, cache) in bf16 and 8
    greedy decode steps: the reference's bf16 numbers for a model-level GPU
    run whose decode steps go through the fused append + decode kernel
    (bf16 only; the fp32 run takes the two-call path). Also stores the
    reference's own bf16 noise floor (``bf16_noise_floor``): how far its
    logits and K / V move when only the GEMM accumulation changes, the scale
    below which a bf16 comparison of 24 layers cannot resolve anything.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "minimal-inference_b200"))
sys.path.insert(0, REPO)

from oracle import paged_oracle as po  # noqa: E402

CONFIG1 = dict(
    hidden_size=896, num_attention_heads=14, num_key_value_heads=2, head_dim=64,
    num_hidden_layers=24, intermediate_size=4864, vocab_size=151936,
    rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=32768,
    tie_word_embeddings=True, attn_bias=True,
)
CONFIG1_SEED = 20240601
CONFIG1_PROMPTS = [37, 128, 255, 500]
CONFIG1_DECODE_STEPS = 50
CONFIG1_BF16_DECODE_STEPS = 8
LOGIT_SAMPLE_IDS = 128
KV_SAMPLES = 48


def _bits(t: torch.Tensor) -> np.ndarray:
    """Raw storage bits of a CPU tensor (uint16 for 16-bit dtypes)."""
    if t.dtype == torch.float32:
        return t.contiguous().numpy().copy()
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def gen_rope(ref_model) -> dict:
    out = {}
    for dname, dtype in (("bfloat16", torch.bfloat16), ("float16", torch.float16),
                         ("float32", torch.float32)):
        for d in (64, 128):
            cos, sin = ref_model.precompute_rope(d, 32768, 1e6, torch.device("cpu"))
            cos, sin = cos.to(dtype), sin.to(dtype)
            from mi_b200.rope import rope_tables
            c2, s2 = rope_tables(d, 32768, 1e6, dtype)
            assert torch.equal(c2, cos) and torch.equal(s2, sin), \
                "mi_b200.rope.rope_tables differs from the reference's precompute_rope"
            g = torch.Generator().manual_seed(1000 + d)
            n, h = 32, 2
            x = (torch.randn(1, h, n, d, generator=g) * 2).to(dtype)
            pos = torch.randint(0, 32768, (1, n), generator=g)
            pos[0, :6] = torch.arange(6)
            pos[0, 6] = 32767
            y = ref_model.apply_rotary_emb(x, cos[pos], sin[pos])
            key = f"{dname}_d{d}"
            out[f"{key}_x"] = _bits(x[0].transpose(0, 1))        # [n, h, d]
            out[f"{key}_pos"] = pos[0].numpy().astype(np.int32)
            out[f"{key}_cos"] = _bits(cos[pos[0]])                # [n, d]
            out[f"{key}_sin"] = _bits(sin[pos[0]])
            out[f"{key}_y"] = _bits(y[0].transpose(0, 1))         # [n, h, d]
    return out


def gen_attn(ref_model, ref_sched) -> dict:
    out = {}
    cases = [
        ("g7", dict(hq=7, hkv=1, d=32), [5, 17, 33], 3),
        ("g4", dict(hq=8, hkv=2, d=64), [16, 20], 2),
    ]
    ps, max_seq = 16, 64
    for dname, dtype in (("float32", torch.float32), ("bfloat16", torch.bfloat16)):
        for cname, h, prompts, steps in cases:
            key = f"{dname}_{cname}"
            cfg = ref_model.ModelConfig(
                hidden_size=h["hq"] * h["d"], num_attention_heads=h["hq"],
                num_key_value_heads=h["hkv"], head_dim=h["d"], num_hidden_layers=1,
                intermediate_size=64, vocab_size=32)
            attn = ref_model.Attention(cfg).to(dtype)
            b = len(prompts)
            bkv = ref_sched.BatchedKVCache(cfg, b, max_seq, torch.device("cpu"), dtype)
            kc, vc = bkv.caches[0]
            pkv = ref_sched.PagedKVCache(cfg, b, max_seq, ps, torch.device("cpu"), dtype)
            g = torch.Generator().manual_seed(7 + len(key))
            pages: list[list[int]] = []
            records = {}
            # prefill, one request at a time, in admission order
            for r, plen in enumerate(prompts):
                pages.append(pkv.allocate_pages(math.ceil(plen / ps)))
                q = torch.randn(1, h["hq"], plen, h["d"], generator=g).to(dtype)
                k = torch.randn(1, h["hkv"], plen, h["d"], generator=g).to(dtype)
                v = torch.randn(1, h["hkv"], plen, h["d"], generator=g).to(dtype)
                mask = torch.triu(torch.full((plen, plen), float("-inf"), dtype=dtype),
                                  diagonal=1)[None, None]
                pid = torch.arange(plen)[None]
                o = attn._pytorch_attention(q, k, v, mask, (kc[r:r + 1], vc[r:r + 1]),
                                            pid, 1, plen)
                indptr, indices, last = ref_sched.build_csr_metadata(
                    [pages[r]], [plen], ps, torch.device("cpu"))
                records[f"pre{r}_q"] = _bits(q[0].transpose(0, 1))       # [L, hq, d]
                records[f"pre{r}_k"] = _bits(k[0].transpose(0, 1))       # [L, hkv, d]
                records[f"pre{r}_v"] = _bits(v[0].transpose(0, 1))
                records[f"pre{r}_o"] = o[0].float().numpy().reshape(plen, h["hq"], h["d"])
                records[f"pre{r}_indptr"] = indptr.numpy()
                records[f"pre{r}_indices"] = indices.numpy()
                records[f"pre{r}_last"] = last.numpy()
            pos = list(prompts)
            for s in range(steps):
                for r in range(b):
                    need = math.ceil((pos[r] + 1) / ps)
                    if need > len(pages[r]):
                        pages[r].extend(pkv.allocate_pages(need - len(pages[r])))
                indptr, indices, last = ref_sched.build_csr_metadata(
                    pages, [p + 1 for p in pos], ps, torch.device("cpu"))
                q = torch.randn(b, h["hq"], 1, h["d"], generator=g).to(dtype)
                k = torch.randn(b, h["hkv"], 1, h["d"], generator=g).to(dtype)
                v = torch.randn(b, h["hkv"], 1, h["d"], generator=g).to(dtype)
                max_kv = max(pos) + 1
                kb = kc[:, :, :max_kv].contiguous()
                vb = vc[:, :, :max_kv].contiguous()
                mask = torch.zeros(b, 1, 1, max_kv, dtype=dtype)
                for i, p in enumerate(pos):
                    if p + 1 < max_kv:
                        mask[i, 0, 0, p + 1:] = float("-inf")
                pid = torch.tensor(pos)[:, None]
                o = attn._pytorch_attention(q, k, v, mask, (kb, vb), pid, b, 1)
                for i, p in enumerate(pos):
                    kc[i, :, p] = kb[i, :, p]
                    vc[i, :, p] = vb[i, :, p]
                records[f"dec{s}_q"] = _bits(q[:, :, 0])                 # [b, hq, d]
                records[f"dec{s}_k"] = _bits(k[:, :, 0])                 # [b, hkv, d]
                records[f"dec{s}_v"] = _bits(v[:, :, 0])
                records[f"dec{s}_o"] = o[:, 0].float().numpy().reshape(b, h["hq"], h["d"])
                records[f"dec{s}_pos"] = np.asarray(pos, np.int32)
                records[f"dec{s}_indptr"] = indptr.numpy()
                records[f"dec{s}_indices"] = indices.numpy()
                records[f"dec{s}_last"] = last.numpy()
                pos = [p + 1 for p in pos]
            records["final_kc"] = _bits(kc)   # [b, hkv, max_seq, d]
            records["final_vc"] = _bits(vc)
            records["final_len"] = np.asarray(pos, np.int32)
            records["num_pages"] = np.asarray([pkv.max_num_pages], np.int32)
            records["meta"] = np.asarray([h["hq"], h["hkv"], h["d"], ps, b, steps], np.int32)
            for kk, vv in records.items():
                out[f"{key}__{kk}"] = vv
    return out


class _RecordingWrapper:
    """Stands in for a FlashInfer wrapper: records plan() metadata, runs the oracle."""

    def __init__(self, kind, log):
        self.kind, self.log, self.meta = kind, log, None

    def plan(self, *args, **kw):
        if self.kind == "prefill":
            qo, indptr, indices, last = (kw["qo_indptr"], kw["paged_kv_indptr"],
                                         kw["paged_kv_indices"], kw["paged_kv_last_page_len"])
        else:
            qo = None
            indptr, indices, last = kw["indptr"], kw["indices"], kw["last_page_len"]
        self.meta = dict(
            qo=None if qo is None else qo.tolist(), indptr=indptr.tolist(),
            indices=indices.tolist(), last=last.tolist(),
            heads=kw["num_qo_heads"], ps=kw["page_size"])
        self.log.append({"event": "plan_" + self.kind, "indptr": self.meta["indptr"],
                         "indices": self.meta["indices"][:self.meta["indptr"][-1]],
                         "last_page_len": self.meta["last"]})

    def run(self, q, kv_data):
        m = self.meta
        kv = kv_data.numpy()
        if self.kind == "prefill":
            o, _ = po.prefill_attention(q.numpy(), m["qo"], kv, m["indptr"], m["indices"],
                                        m["last"], m["ps"], causal=True)
        else:
            o, _ = po.decode_attention(q.numpy(), kv, m["indptr"], m["indices"], m["last"],
                                       m["ps"])
        return torch.from_numpy(o).to(q.dtype)


def gen_sched_trace(ref_model, ref_sched) -> dict:
    """Run the reference Scheduler's paged control flow on CPU and record it."""
    cfg = ref_model.ModelConfig(hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
                                head_dim=16, num_hidden_layers=2, intermediate_size=96,
                                vocab_size=97, tie_word_embeddings=True, attn_bias=True)
    torch.manual_seed(0)
    results = {}
    cases = {
        # max_batch 3, max_seq 64 -> 12 pages (11 usable + scratch)
        "churn": dict(max_batch=3, max_seq=64, prompts=[20, 5, 33, 16, 40, 1, 12, 9],
                      max_new=[4, 30, 10, 1, 20, 25, 8, 3]),
        # a request that runs into max_seq_len (position 64)
        "seqcap": dict(max_batch=2, max_seq=64, prompts=[60, 3], max_new=[50, 5]),
    }
    for name, c in cases.items():
        model = ref_model.Model(cfg)
        log: list = []
        sched = ref_sched.Scheduler(model, cfg, torch.device("cpu"), torch.float32,
                                    max_batch_size=c["max_batch"], max_seq_len=c["max_seq"],
                                    page_size=16, eos_token_ids=set(), use_flashinfer=True)
        # Force the paged path on CPU: the reference picks it only on CUDA
        # (scheduler.py:504); FlashInfer's kernels are replaced by recorders.
        sched.use_flashinfer = True
        sched.kv_cache = ref_sched.PagedKVCache(cfg, c["max_batch"], c["max_seq"], 16,
                                                torch.device("cpu"), torch.float32)
        sched._prefill_wrapper = _RecordingWrapper("prefill", log)
        sched._decode_wrapper = _RecordingWrapper("decode", log)
        sched._graph_runners = {}
        orig_release = sched.kv_cache.release_pages

        def release(pages, _orig=orig_release, _log=log):
            _log.append({"event": "release", "pages": list(pages)})
            return _orig(pages)

        sched.kv_cache.release_pages = release
        orig_alloc = sched.kv_cache.allocate_pages

        def alloc(n, _orig=orig_alloc, _log=log):
            p = _orig(n)
            _log.append({"event": "alloc", "pages": list(p)})
            return p

        sched.kv_cache.allocate_pages = alloc

        def fake_append(k, v, batch_indices, positions, kv_data, indices, indptr, last,
                        kv_layout="NHD", _log=log):
            po.append_paged_kv(kv_data.numpy(), k.numpy(), v.numpy(), batch_indices.numpy(),
                               positions.numpy(), indices.numpy(), indptr.numpy(), 16)

        ref_model.flashinfer.page.append_paged_kv_cache = fake_append
        for i, (pl, mn) in enumerate(zip(c["prompts"], c["max_new"])):
            ids = torch.randint(0, cfg.vocab_size, (pl,)).tolist()
            sched.submit_request(ref_sched.Request(f"r{i}", ids, mn, 0.0))
        steps = 0
        while sched.active_requests or sched.waiting_queue:
            log.append({"event": "step", "n": steps})
            sched._admit_new_requests()
            sched._prefill_new_requests()
            if any(r.status == ref_sched.RequestStatus.DECODING for r in sched.active_requests):
                sched._decode_step()
            sched._retire_finished_requests()
            steps += 1
            assert steps < 10000
        results[name] = {"config": c, "log": log}
    return results


def _digest_rows(logits: np.ndarray, sample_ids: np.ndarray) -> dict:
    """Per-row digest of [N, V] fp32 logits."""
    top = np.argsort(-logits, axis=-1)[:, :8]
    m = logits.max(axis=-1, keepdims=True)
    lse = (np.log(np.exp(logits - m).sum(axis=-1, keepdims=True)) + m)[:, 0]
    return {"argmax": logits.argmax(-1).astype(np.int32), "top_ids": top.astype(np.int32),
            "top_vals": np.take_along_axis(logits, top, axis=-1).astype(np.float32),
            "lse": lse.astype(np.float32), "sampled": logits[:, sample_ids].astype(np.float32)}


def bf16_noise_floor(model, prompts, generated) -> tuple[float, float]:
    """How far the reference's own bf16 numbers move when only the GEMM
    accumulation changes: every request's teacher-forced sequence (prompt +
    generated tokens) through the reference model twice, with its stock bf16
    ``F.linear`` and with each linear computed in fp32 and rounded to bf16
    once. Returns the largest logit difference over the positions that
    produced a token, and the largest difference of any layer's K / V
    projection output (what the cache stores, before RoPE on K)."""
    import torch.nn.functional as F

    kv_out = []
    hooks = [m.register_forward_hook(lambda _m, _i, o: kv_out.append(o.float()))
             for layer in model.layers for m in (layer.self_attn.k_proj, layer.self_attn.v_proj)]

    def run():
        rows = []
        kv_out.clear()
        with torch.no_grad():
            for ids, toks in zip(prompts, generated):
                seq = torch.tensor(list(ids) + list(toks[:-1])).unsqueeze(0)
                lg = model(seq, position_ids=torch.arange(seq.shape[1]).unsqueeze(0))[0]
                rows.append(lg[len(ids) - 1:].float())
        return rows, list(kv_out)

    stock, kv_stock = run()
    orig = F.linear

    def linear_fp32(x, w, b=None):
        return orig(x.float(), w.float(), None if b is None else b.float()).to(x.dtype)

    F.linear = linear_fp32
    try:
        fp32acc, kv_fp32 = run()
    finally:
        F.linear = orig
        for h in hooks:
            h.remove()
    logit = max(float((a - b).abs().max()) for a, b in zip(stock, fp32acc))
    kv = max(float((a - b).abs().max()) for a, b in zip(kv_stock, kv_fp32))
    return logit, kv


def gen_config1(ref_model, ref_sched, dtype=torch.float32,
                decode_steps: int = CONFIG1_DECODE_STEPS) -> dict:
    from mi_b200.weights import init_random_weights

    torch.set_num_threads(os.cpu_count() or 8)
    cfg = ref_model.ModelConfig(**CONFIG1)
    model = ref_model.Model(cfg)
    t0 = time.time()
    init_random_weights(model, CONFIG1_SEED)
    model = model.to(dtype).eval()
    print(f"config1 ({dtype}): weights in {time.time() - t0:.1f}s", flush=True)
    sched = ref_sched.Scheduler(model, cfg, torch.device("cpu"), dtype,
                                max_batch_size=4, max_seq_len=4096, page_size=16,
                                eos_token_ids=set(), use_flashinfer=True)
    assert not sched.use_flashinfer
    g = torch.Generator().manual_seed(CONFIG1_SEED + 1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist()
               for n in CONFIG1_PROMPTS]
    sample_ids = np.sort(np.random.default_rng(CONFIG1_SEED).choice(
        cfg.vocab_size, LOGIT_SAMPLE_IDS, replace=False)).astype(np.int64)
    calls = []
    orig_forward = model.forward

    def forward(input_ids, *a, **kw):
        lg = orig_forward(input_ids, *a, **kw)
        calls.append(lg[:, -1, :].float().numpy().copy())
        return lg

    model.forward = forward
    kv_digest = {}
    rng = np.random.default_rng(CONFIG1_SEED + 2)
    orig_release = sched.kv_cache.release_slot
    reqs = []

    def release_slot(slot):
        req = next(r for r in reqs if r.batch_slot == slot)
        n = req.current_position
        pos_s = rng.integers(0, n, KV_SAMPLES)
        head_s = rng.integers(0, cfg.num_key_value_heads, KV_SAMPLES)
        dim_s = rng.integers(0, cfg.head_dim, KV_SAMPLES)
        ks, vs, ksum, vsum = [], [], [], []
        for kcache, vcache in sched.kv_cache.caches:
            kk = kcache[slot, :, :n].float()
            vv = vcache[slot, :, :n].float()
            ks.append(kk[head_s, pos_s, dim_s].numpy())
            vs.append(vv[head_s, pos_s, dim_s].numpy())
            ksum.append(float(kk.double().abs().sum()))
            vsum.append(float(vv.double().abs().sum()))
        kv_digest[req.request_id] = dict(len=n, pos=pos_s, head=head_s, dim=dim_s,
                                         k=np.stack(ks), v=np.stack(vs),
                                         kabs=np.asarray(ksum), vabs=np.asarray(vsum))
        return orig_release(slot)

    sched.kv_cache.release_slot = release_slot
    for i, ids in enumerate(prompts):
        r = ref_sched.Request(f"r{i}", ids, decode_steps + 1, 0.0)
        reqs.append(r)
        sched.submit_request(r)
    order = []
    t0 = time.time()
    while sched.active_requests or sched.waiting_queue:
        sched._admit_new_requests()
        n_before = len(calls)
        pre = [r.request_id for r in sched.active_requests
               if r.status == ref_sched.RequestStatus.PREFILLING]
        sched._prefill_new_requests()
        for rid in pre:
            order.append(("prefill", [rid]))
        if any(r.status == ref_sched.RequestStatus.DECODING for r in sched.active_requests):
            dec = [r.request_id for r in sched.active_requests
                   if r.status == ref_sched.RequestStatus.DECODING]
            sched._decode_step()
            order.append(("decode", dec))
        n_decode = 1 if order and order[-1][0] == "decode" and len(calls) > n_before + len(pre) else 0
        assert len(calls) == n_before + len(pre) + n_decode
        sched._retire_finished_requests()
    print(f"config1: reference CPU run {time.time() - t0:.1f}s, {len(calls)} forward calls",
          flush=True)
    # flatten logits rows in call order, with (kind, step, request) labels
    rows, labels = [], []
    dec_step = 0
    for (kind, rids), lg in zip(order, calls):
        for j, rid in enumerate(rids):
            rows.append(lg[j])
            labels.append((0 if kind == "prefill" else 1, dec_step if kind == "decode" else -1,
                           int(rid[1:])))
        if kind == "decode":
            dec_step += 1
    dig = _digest_rows(np.stack(rows), sample_ids)
    out = {f"logit_{k}": v for k, v in dig.items()}
    out["logit_labels"] = np.asarray(labels, np.int32)
    out["sample_ids"] = sample_ids.astype(np.int32)
    out["seed"] = np.asarray([CONFIG1_SEED], np.int64)
    out["dtype"] = np.asarray([str(dtype).removeprefix("torch.")])
    if dtype == torch.bfloat16:
        model.forward = orig_forward
        floor, kv_floor = bf16_noise_floor(model, [r.input_ids for r in reqs],
                                           [r.generated_tokens for r in reqs])
        print(f"config1 ({dtype}): noise floor of the reference itself: logits {floor:.4f}, "
              f"K/V {kv_floor:.4f}", flush=True)
        out["logit_noise_floor"] = np.asarray([floor], np.float32)
        out["kv_noise_floor"] = np.asarray([kv_floor], np.float32)
    out["prompt_lens"] = np.asarray(CONFIG1_PROMPTS, np.int32)
    for i, r in enumerate(reqs):
        out[f"prompt_{i}"] = np.asarray(r.input_ids, np.int32)
        out[f"tokens_{i}"] = np.asarray(r.generated_tokens, np.int32)
        d = kv_digest[r.request_id]
        for k, v in d.items():
            out[f"kv_{i}_{k}"] = np.asarray(v)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (model.py, scheduler.py)")
    ap.add_argument("--only", default="rope,attn,sched,config1,config1_bf16")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import model as ref_model  # noqa: E402
    import scheduler as ref_sched  # noqa: E402

    only = set(args.only.split(","))
    if "rope" in only:
        np.savez_compressed(os.path.join(HERE, "rope.npz"), **gen_rope(ref_model))
    if "attn" in only:
        np.savez_compressed(os.path.join(HERE, "attn.npz"), **gen_attn(ref_model, ref_sched))
    if "sched" in only:
        with open(os.path.join(HERE, "sched_trace.json"), "w") as f:
            json.dump(gen_sched_trace(ref_model, ref_sched), f, separators=(",", ":"))
    if "config1" in only:
        np.savez_compressed(os.path.join(HERE, "config1.npz"), **gen_config1(ref_model, ref_sched))
    if "config1_bf16" in only:
        np.savez_compressed(os.path.join(HERE, "config1_bf16.npz"),
                            **gen_config1(ref_model, ref_sched, torch.bfloat16,
                                          CONFIG1_BF16_DECODE_STEPS))
    for fn in sorted(os.listdir(HERE)):
        if fn.endswith((".npz", ".json")):
            print(fn, os.path.getsize(os.path.join(HERE, fn)))


if __name__ == "__main__":
    main()
