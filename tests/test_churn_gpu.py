"""Serving under churn (BASELINE config 4's pattern, small shapes).

Qwen2.5-0.5B shape cut to 2 layers, max_batch 8, max_seq 512, page_size 16;
40 requests with prompts U[8, 200] and outputs U[1, 40], a new one submitted
whenever one finishes, so admissions, batched prefills, page growth inside the
decode graph and retirements interleave and the free list gets shuffled. At
the end every request has exactly its drawn number of tokens, no device status
bit is set, every page is back in the pool and the free ring holds each page
id exactly once (the scratch page never enters it).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_churn_small_model_returns_every_page():
    import dataclasses

    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Request, Scheduler

    cfg = dataclasses.replace(PRESETS["qwen2.5-0.5b"], num_hidden_layers=2)
    dev = torch.device("cuda", 0)
    model = Model.create(cfg, dev, torch.bfloat16, seed=9)
    sched = Scheduler(model, cfg, dev, torch.bfloat16, max_batch_size=8, max_seq_len=512,
                      page_size=16, eos_token_ids=set())
    rng = np.random.default_rng(12)
    stream = [(rng.integers(0, cfg.vocab_size, int(rng.integers(8, 201))).tolist(),
               int(rng.integers(1, 41))) for _ in range(40)]
    reqs, nxt = [], 0

    def submit(k):
        nonlocal nxt
        for _ in range(k):
            if nxt < len(stream):
                r = Request(f"r{nxt}", stream[nxt][0], stream[nxt][1], 0.0)
                reqs.append(r)
                sched.submit_request(r)
                nxt += 1

    submit(8)
    steps = 0
    while (sched.active_requests or sched.waiting_queue or nxt < len(stream)) and steps < 2000:
        before = sum(r.status.value == "finished" for r in reqs)
        sched.step()
        steps += 1
        submit(sum(r.status.value == "finished" for r in reqs) - before)
    torch.cuda.synchronize()
    kv = sched.kv_cache
    kv.check_status()
    assert steps < 2000
    assert [len(r.generated_tokens) for r in reqs] == [n for _, n in stream]
    P = kv.max_num_pages
    assert int(kv.pool_ctrl[1].item()) == P - 1 == kv.num_free_pages
    head = int(kv.pool_ctrl[0].item())        # FIFO ring: live entries from the head
    ring = kv.free_ring.cpu().numpy()
    live = [int(ring[(head + i) % P]) for i in range(P - 1)]
    assert sorted(live) == list(range(P - 1))
    sched.close()
