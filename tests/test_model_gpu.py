"""Model- and scheduler-level GPU tests.

* BASELINE config 1 (Qwen2.5-0.5B shape, fp32, seeded weights) through this
  package's Scheduler, teacher-forced with the token sequence the reference
  generated on CPU (tests/golden/config1.npz): per-step logit digests and
  per-layer KV samples must match the reference within 2e-2, and every page
  must come back to the pool. The same in bf16 (tests/golden/config1_bf16.npz,
  8 decode steps), where the decode steps run the fused append + decode
  kernel; its logit bar is the reference's own bf16 noise floor when that is
  above 2e-2.
* A Mistral-7B-shaped model (2 layers, bf16): CUDA-graph decode steps agree
  with eager decode steps, padding lanes included.
"""
import math
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
DEV = "cuda"


def _config1():
    from mi_b200.model import PRESETS
    return PRESETS["qwen2.5-0.5b"]


@pytest.mark.parametrize("fixture,dtype", [("config1.npz", torch.float32),
                                           ("config1_bf16.npz", torch.bfloat16)])
def test_config1_parity_with_reference_teacher_forced(fixture, dtype):
    """fp32: the reference's own CPU precision for config 1 (decode steps take
    the append + decode calls). bf16: the reference run in bf16, whose decode
    steps here go through the fused append + decode kernel."""
    from mi_b200.model import Model
    from mi_b200.scheduler import Request, Scheduler
    from mi_b200.weights import init_random_weights
    fx = np.load(os.path.join(GOLDEN, fixture))
    cfg = _config1()
    model = Model(cfg)
    init_random_weights(model, int(fx["seed"][0]))
    model = model.to(device=DEV, dtype=dtype).eval().prepare()
    n_req = len(fx["prompt_lens"])
    teacher = {f"r{i}": fx[f"tokens_{i}"].tolist() for i in range(n_req)}
    sched = Scheduler(model, cfg, torch.device(DEV), dtype, max_batch_size=4,
                      max_seq_len=4096, page_size=16, eos_token_ids=set(),
                      teacher_tokens=teacher)
    sched.record_logits = True
    kv_samples = {}
    orig_release = sched.kv_cache.slot_release

    def release(slots, total_pages):
        # sample the released requests' KV pages, as the reference did before
        # zeroing its padded cache slot
        for req in [r for r in sched.active_requests if r.status.value == "finished"]:
            i = int(req.request_id[1:])
            pages = sched.kv_cache.slot_pages(req.batch_slot)
            pos, head, dim = fx[f"kv_{i}_pos"], fx[f"kv_{i}_head"], fx[f"kv_{i}_dim"]
            pg = np.asarray(pages)[pos // 16]
            ks, vs = [], []
            for layer in sched.kv_cache.kv_data:
                ks.append(layer[pg, 0, pos % 16, head, dim].float().cpu().numpy())
                vs.append(layer[pg, 1, pos % 16, head, dim].float().cpu().numpy())
            kv_samples[i] = (np.stack(ks), np.stack(vs), req.current_position)
        return orig_release(slots, total_pages)

    sched.kv_cache.slot_release = release
    reqs = []
    for i in range(n_req):
        r = Request(f"r{i}", fx[f"prompt_{i}"].tolist(), len(teacher[f"r{i}"]), 0.0)
        reqs.append(r)
        sched.submit_request(r)
    steps = 0
    while sched.active_requests or sched.waiting_queue:
        sched.step()
        steps += 1
        assert steps < 1000
    torch.cuda.synchronize()
    sched.kv_cache.check_status()
    # every request ran to its teacher length
    for i, r in enumerate(reqs):
        assert r.generated_tokens == teacher[f"r{i}"]
    # logits: flatten our recorded rows in the golden's label order
    mine = {}
    dec_step = 0
    for kind, ids, rows in sched.step_logits:
        for j, rid in enumerate(ids):
            key = (0, -1, int(rid[1:])) if kind == "prefill" else (1, dec_step, int(rid[1:]))
            mine[key] = rows[j].numpy()
        if kind == "decode":
            dec_step += 1
    labels = [tuple(int(x) for x in lab) for lab in fx["logit_labels"]]
    assert set(labels) == set(mine)
    sample_ids = fx["sample_ids"]
    # fp32: 2e-2. bf16: no further from the reference than the reference's
    # own bf16 logits move when only its GEMM accumulation changes (stored by
    # the fixture generator; 24 bf16 layers put that above 2e-2)
    tol = max(2e-2, float(fx["logit_noise_floor"][0])) if "logit_noise_floor" in fx else 2e-2
    worst = 0.0
    argmax_match = 0
    for k, lab in enumerate(labels):
        row = mine[lab]
        worst = max(worst, float(np.abs(row[sample_ids] - fx["logit_sampled"][k]).max()))
        top = fx["logit_top_ids"][k]
        worst = max(worst, float(np.abs(row[top] - fx["logit_top_vals"][k]).max()))
        m = row.max()
        lse = float(np.log(np.exp(row - m).sum()) + m)
        worst = max(worst, abs(lse - float(fx["logit_lse"][k])))
        a = int(row.argmax())
        if a == int(fx["logit_argmax"][k]):
            argmax_match += 1
        elif "logit_noise_floor" in fx and a in top:
            # bf16: a near-tie of the reference's best token counts as a match
            near = fx["logit_top_vals"][k][list(top).index(a)] >= fx["logit_top_vals"][k][0] - tol
            argmax_match += int(near)
    assert worst <= tol, f"max logit deviation {worst} > {tol}"
    if "logit_noise_floor" in fx:
        assert argmax_match == len(labels)         # every row's pick is the best or a near-tie
    else:
        assert argmax_match >= 0.95 * len(labels)
    # KV pages vs the reference's padded cache, sampled
    for i in range(n_req):
        ks, vs, n = kv_samples[i]
        assert n == int(fx[f"kv_{i}_len"])
        kv_tol = max(2e-2, float(fx["kv_noise_floor"][0])) if "kv_noise_floor" in fx else 2e-2
        np.testing.assert_allclose(ks, fx[f"kv_{i}_k"], atol=kv_tol, rtol=0)
        np.testing.assert_allclose(vs, fx[f"kv_{i}_v"], atol=kv_tol, rtol=0)
    # all pages back in the pool
    assert int(sched.kv_cache.pool_ctrl[1].item()) == sched.kv_cache.max_num_pages - 1
    assert sched.kv_cache.num_free_pages == sched.kv_cache.max_num_pages - 1


def _mistral_small():
    from mi_b200.model import PRESETS
    import dataclasses
    return dataclasses.replace(PRESETS["mistral-7b"], num_hidden_layers=2)


def _run(cfg, model, graphs, prompts, max_new, teacher=None):
    from mi_b200.scheduler import Request, Scheduler
    sched = Scheduler(model, cfg, torch.device(DEV), torch.bfloat16, max_batch_size=8,
                      max_seq_len=1024, page_size=16, eos_token_ids=set(),
                      use_cuda_graph=graphs, teacher_tokens=teacher)
    sched.record_logits = True
    reqs = [Request(f"r{i}", p, m, 0.0) for i, (p, m) in enumerate(zip(prompts, max_new))]
    for r in reqs:
        sched.submit_request(r)
    while sched.active_requests or sched.waiting_queue:
        sched.step()
    torch.cuda.synchronize()
    sched.kv_cache.check_status()
    free = int(sched.kv_cache.pool_ctrl[1].item())
    return reqs, sched.step_logits, free, sched.kv_cache.max_num_pages - 1


def test_mistral_shape_graph_decode_matches_eager():
    from mi_b200.model import Model
    from mi_b200.weights import init_random_weights
    cfg = _mistral_small()
    model = Model(cfg).to(device=DEV, dtype=torch.bfloat16)
    init_random_weights(model, 11, generator_device="cuda")
    model.eval().prepare()
    rng = np.random.default_rng(5)
    lens = [17, 200, 31, 64, 129]   # 5 requests: bucket 8 with 3 padding lanes
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in lens]
    max_new = [12, 5, 20, 16, 3]
    ra, la, fa, full_a = _run(cfg, model, True, prompts, max_new)
    # eager run forced along the graph run's tokens, so near-tied logits
    # cannot send the two runs down different paths
    teacher = {r.request_id: r.generated_tokens for r in ra}
    rb, lb, fb, full_b = _run(cfg, model, False, prompts, max_new, teacher)
    assert fa == full_a and fb == full_b
    assert [len(r.generated_tokens) for r in ra] == max_new
    assert len(la) == len(lb)
    for (ka, ia, xa), (kb, ib, xb) in zip(la, lb):
        assert ka == kb and ia == ib
        assert float((xa - xb).abs().max()) <= 2e-2
