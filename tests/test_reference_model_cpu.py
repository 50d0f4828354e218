"""The CPU port of the reference's whole padded forward, pinned to the
reference's own config-1 outputs (tests/golden/config1.npz, made by running
the reference's Scheduler on the CPU): prefill and first-decode-step logits
of two requests, same seeded weights, teacher-forced tokens."""
import os

import numpy as np
import torch

from oracle.reference_cpu import PaddedReferenceModel

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _deviation(row: np.ndarray, fx, k: int) -> float:
    sample_ids = fx["sample_ids"]
    worst = float(np.abs(row[sample_ids] - fx["logit_sampled"][k]).max())
    worst = max(worst, float(np.abs(row[fx["logit_top_ids"][k]] - fx["logit_top_vals"][k]).max()))
    m = row.max()
    return max(worst, abs(float(np.log(np.exp(row - m).sum()) + m) - float(fx["logit_lse"][k])))


def test_padded_reference_model_matches_the_reference_outputs():
    from mi_b200.model import PRESETS, Model
    from mi_b200.weights import init_random_weights
    fx = np.load(os.path.join(GOLDEN, "config1.npz"))
    cfg = PRESETS["qwen2.5-0.5b"]
    model = Model(cfg)
    init_random_weights(model, int(fx["seed"][0]))
    ref = PaddedReferenceModel(model.state_dict(), cfg, max_batch=2, max_seq=512)
    labels = {tuple(int(x) for x in lab): k for k, lab in enumerate(fx["logit_labels"])}
    reqs = [0, 1]
    worst = 0.0
    for slot, i in enumerate(reqs):
        row = ref.prefill(slot, fx[f"prompt_{i}"].tolist()).numpy()
        worst = max(worst, _deviation(row, fx, labels[(0, -1, i)]))
        assert row.argmax() == fx["logit_argmax"][labels[(0, -1, i)]]
    positions = [len(fx[f"prompt_{i}"]) for i in reqs]
    tokens = [int(fx[f"tokens_{i}"][0]) for i in reqs]
    rows = ref.decode(list(range(len(reqs))), positions, tokens).numpy()
    for j, i in enumerate(reqs):
        worst = max(worst, _deviation(rows[j], fx, labels[(1, 0, i)]))
    assert worst <= 2e-3, worst
