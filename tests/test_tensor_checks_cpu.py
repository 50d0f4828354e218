"""Host-side argument checks of the op wrappers (no GPU needed).

Caller-provided outputs are written by the kernels as dense rows through a
raw pointer, so a buffer of the wrong shape, dtype, layout or device must be
refused before the launch rather than written out of bounds.
"""
import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "minimal-inference_b200"))

from mi_b200._tensor import check_rows, need_on  # noqa: E402


def test_check_rows_accepts_dense_rows_with_spare_leading_rows():
    t = torch.empty(40, 32, 128, dtype=torch.bfloat16)
    assert check_rows("out", t, 32, (32, 128), torch.bfloat16, "cpu") is t
    assert check_rows("out", t[:32], 32, (32, 128), torch.bfloat16, "cpu") is not None


@pytest.mark.parametrize("bad, match", [
    (torch.empty(31, 32, 128, dtype=torch.bfloat16), r"\[>= 32, 32, 128\]"),     # too few rows
    (torch.empty(32, 28, 128, dtype=torch.bfloat16), r"\[>= 32, 32, 128\]"),     # row shape
    (torch.empty(32, 32 * 128, dtype=torch.bfloat16), r"\[>= 32, 32, 128\]"),    # rank
    (torch.empty(32, 32, 128, dtype=torch.float16), "bfloat16"),                 # dtype
    (torch.empty(32, 128, 32, dtype=torch.bfloat16).transpose(1, 2), "contiguous"),
])
def test_check_rows_refuses(bad, match):
    with pytest.raises(ValueError, match=match):
        check_rows("out", bad, 32, (32, 128), torch.bfloat16, "cpu")


def test_need_on_refuses_another_device():
    t = torch.empty(4)
    assert need_on("x", t, "cpu") is t
    with pytest.raises(ValueError, match="expected meta"):
        need_on("x", t, "meta")
    with pytest.raises(ValueError, match="is on meta"):
        check_rows("out", torch.empty(4, 8, device="meta"), 4, (8,), torch.float32, "cpu")


def test_glue_refuses_bad_out_before_any_launch():
    from mi_b200.glue import add_rmsnorm, silu_mul
    res = torch.empty(4, 64, dtype=torch.bfloat16)
    w = torch.empty(64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="out must be"):
        add_rmsnorm(None, res, w, 1e-6, out=torch.empty(3, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="out must be"):
        add_rmsnorm(None, res, w, 1e-6, out=torch.empty(4, 64, dtype=torch.float32))
    with pytest.raises(ValueError, match="weight is on meta"):
        add_rmsnorm(None, res, torch.empty(64, dtype=torch.bfloat16, device="meta"), 1e-6)
    gu = torch.empty(4, 2 * 96, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="out must be"):
        silu_mul(gu, out=torch.empty(4, 95, dtype=torch.bfloat16))
