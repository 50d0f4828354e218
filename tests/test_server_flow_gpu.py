"""The request flow the reference's ``server.py`` relies on, on a GPU.

``server.py`` builds the engine (``Model(cfg)``, weights, ``.to(device,
dtype).eval()``, ``Scheduler(model=..., config=..., ..., eos_token_ids=...,
use_flashinfer=...)``, ``start()``), then for every HTTP request creates a
``Request(request_id, input_ids, max_new_tokens, temperature, loop)``, calls
``submit_request`` and awaits ``req.token_queue`` on its event loop until
``None``, counting a token in ``EOS_TOKEN_IDS`` as the end of a stopped
completion (``finish_reason``). This test does exactly that with this
package's model and scheduler (a two-layer Qwen2.5-0.5B-shape model with
seeded random bf16 weights): concurrent requests, one consumer that takes
tokens as they stream in and others that collect them all, and an EOS id in
the middle of one request's greedy continuation. The streamed tokens must
equal a direct ``step()`` run of the same requests, the EOS request must end
right after its EOS token with ``finish_reason == "stop"``, and every page
must come back to the pool. The names and call signatures ``server.py`` uses
are checked against its source in ``tests/test_server_contract_cpu.py``.
"""
import asyncio
import dataclasses

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _engine(eos_ids):
    from mi_b200 import scheduler as sched_mod
    from mi_b200.model import PRESETS, Model
    from mi_b200.scheduler import Scheduler
    from mi_b200.weights import init_random_weights
    cfg = dataclasses.replace(PRESETS["qwen2.5-0.5b"], num_hidden_layers=2)
    model = Model(cfg)                       # server.py: Model(cfg) + load_weights + .to().eval()
    init_random_weights(model, 77)
    model = model.to(device="cuda", dtype=torch.bfloat16).eval()
    sched = Scheduler(model=model, config=cfg, device=torch.device("cuda"), dtype=torch.bfloat16,
                      max_batch_size=4, max_seq_len=512, page_size=16,
                      eos_token_ids=eos_ids, use_flashinfer=True)
    return sched_mod, cfg, sched


def _prompts(vocab):
    rng = np.random.default_rng(9)
    return [rng.integers(0, vocab, n).tolist() for n in (23, 150, 61)]


def test_server_request_flow_streams_the_scheduler_tokens():
    from mi_b200.scheduler import Request

    # greedy continuations of the three requests, by stepping the scheduler directly
    sched_mod, cfg, sched = _engine(set())
    saved_eos = sched_mod.EOS_TOKEN_IDS
    try:
        prompts = _prompts(cfg.vocab_size)
        max_new = [12, 9, 15]
        direct = [Request(f"d{i}", p, m, 0.0) for i, (p, m) in enumerate(zip(prompts, max_new))]
        for r in direct:
            sched.submit_request(r)
        while sched.active_requests or sched.waiting_queue:
            sched.step()
        want = [list(r.generated_tokens) for r in direct]
        assert [len(w) for w in want] == max_new
        sched.close()
        del sched
        torch.cuda.empty_cache()

        # the server's flow, with request 1's 5th token declared an EOS id
        eos = want[1][4]
        assert eos not in want[1][:4]
        sched_mod, cfg, sched = _engine({eos})
        sched.start()

        async def serve():
            loop = asyncio.get_event_loop()
            reqs = [Request(request_id=f"chatcmpl-{i}", input_ids=p, max_new_tokens=m,
                            temperature=0.0, loop=loop)
                    for i, (p, m) in enumerate(zip(prompts, max_new))]

            async def collect(req):                  # server.py: non_stream_response
                ids = []
                while True:
                    tok = await asyncio.wait_for(req.token_queue.get(), timeout=120)
                    if tok is None:
                        return ids, req.finish_reason
                    ids.append(tok)

            async def stream(req):                   # server.py: stream_response
                chunks = []
                while True:
                    tok = await asyncio.wait_for(req.token_queue.get(), timeout=120)
                    if tok is None:
                        return chunks, req.finish_reason
                    chunks.append(tok)               # one SSE chunk per token
                    await asyncio.sleep(0)

            for r in reqs:
                sched.submit_request(r)
            return await asyncio.gather(stream(reqs[0]), collect(reqs[1]), collect(reqs[2]))

        got = asyncio.run(serve())
        sched.stop()
        torch.cuda.synchronize()
        sched.kv_cache.check_status()
        (t0, f0), (t1, f1), (t2, f2) = got
        assert t0 == want[0] and f0 == "length"
        assert t2 == want[2] and f2 == "length"
        assert t1 == want[1][:5] and f1 == "stop"   # ends right after the EOS token
        assert sched.kv_cache.num_free_pages == sched.kv_cache.max_num_pages - 1
        sched.close()
    finally:
        sched_mod.EOS_TOKEN_IDS = saved_eos
