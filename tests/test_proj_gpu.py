"""The small-M projection (``mi_proj_small_m``) against an fp32 torch
reference of the same ``F.linear``.

Shapes: the decode step's projections of the Mistral-7B shape (QKV,
o_proj, gate/up, down_proj) and Qwen2.5-0.5B's (with QKV bias), 1 to 32
rows, a column count that is not a multiple of the 128-column block, strided
rows, fp16, and m = 0. K-split partials are added in a fixed order, so
repeated calls give identical bits. Tolerance: the output is
rounded once to bf16 / fp16 from an fp32 sum, so it is within one rounding
of the fp32 reference (rtol 2^-7 for bf16, 2^-10 for fp16) plus the fp32
summation-order difference (atol 1e-3 of the output scale).
"""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SHAPES = [  # (m, n, k, bias)
    (32, 6144, 4096, False),    # Mistral QKV
    (32, 4096, 4096, False),    # o_proj
    (32, 28672, 4096, False),   # gate/up
    (32, 4096, 14336, False),   # down_proj
    (1, 4096, 14336, False),
    (7, 1152, 896, True),       # Qwen2.5-0.5B QKV (bias)
    (16, 896, 4864, False),     # Qwen2.5-0.5B down_proj
    (5, 1000, 128, True),       # last 128-column block partial
    (32, 64, 64, False),        # one block, one K step
    (17, 1001, 2048, True),     # odd column count: the reduction's 4-column groups end mid-group
    (1, 4608, 3584, True),      # Qwen2.5-7B QKV (bias), one row
    (32, 3584, 18944, False),   # Qwen2.5-7B down_proj
]


def _ref(x, w, b):
    y = x.float() @ w.float().t()
    return y + b.float() if b is not None else y


def _check(out, ref, dtype):
    scale = ref.abs().max().item() + 1e-6
    rtol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    torch.testing.assert_close(out.float(), ref, rtol=rtol, atol=1e-3 * scale)


@pytest.mark.parametrize("m,n,k,bias", SHAPES)
def test_proj_matches_fp32_linear(m, n, k, bias):
    from mi_b200 import glue
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(m * 1000 + n + k)
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, device=dev, generator=g) * 0.5).to(torch.bfloat16) if bias else None
    out = glue.proj_small_m(x, w, b)
    torch.cuda.synchronize()
    assert int(glue.proj_status(dev).item()) == 0
    _check(out, _ref(x, w, b), torch.bfloat16)
    # deterministic: a second call gives the same bits
    again = glue.proj_small_m(x, w, b)
    torch.cuda.synchronize()
    assert torch.equal(out, again)


def test_proj_fp16_strided_rows_and_3d_input():
    from mi_b200 import glue
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    base = torch.randn(4, 3, 4096 + 64, device=dev, generator=g).to(torch.float16)
    x = base[..., :4096]                             # rows 4160 elements apart
    w = (torch.randn(2048, 4096, device=dev, generator=g) * 0.02).to(torch.float16)
    out_base = torch.zeros(12, 2048 + 128, dtype=torch.float16, device=dev)
    out = out_base[:, :2048]
    glue.proj_small_m(x.reshape(12, 4096), w, out=out)
    torch.cuda.synchronize()
    _check(out, _ref(x.reshape(12, 4096), w, None), torch.float16)
    assert torch.count_nonzero(out_base[:, 2048:]) == 0     # nothing written past n
    y3 = glue.proj_small_m(base[..., :4096].contiguous(), w)
    assert y3.shape == (4, 3, 2048)
    _check(y3.reshape(12, 2048), _ref(x.reshape(12, 4096), w, None), torch.float16)


def test_proj_zero_rows_and_bad_arguments():
    from mi_b200 import capi, glue
    dev = torch.device("cuda", 0)
    w = torch.zeros(256, 128, dtype=torch.bfloat16, device=dev)
    y = glue.proj_small_m(torch.zeros(0, 128, dtype=torch.bfloat16, device=dev), w)
    assert y.shape == (0, 256)
    with pytest.raises(ValueError):
        glue.proj_small_m(torch.zeros(33, 128, dtype=torch.bfloat16, device=dev), w)
    with pytest.raises(capi.MiError):                         # k not a multiple of 64
        glue.proj_small_m(torch.zeros(2, 96, dtype=torch.bfloat16, device=dev),
                          torch.zeros(256, 96, dtype=torch.bfloat16, device=dev))
