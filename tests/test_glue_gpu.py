"""Decode-step glue kernels (libmi_paged.so) against torch.

* residual add: bit-identical to torch's ``x + y`` in the storage dtype;
* RMSNorm: within one storage-dtype rounding of the fp32 formula
  ``h * rsqrt(mean(h^2) + eps) * w`` (model.py:121-122);
* SiLU * up: within one rounding of torch's ``F.silu(g) * u`` (model.py:311).
"""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from mi_b200.glue import add_rmsnorm, silu_mul  # noqa: E402

# one rounding of the storage dtype, relative
ULP = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10, torch.float32: 4e-6}


def _norm_ref(h, w, eps):
    hf = h.float()
    return hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,hidden", [(32, 4096), (1, 896), (7, 3584), (3, 8192),
                                         (5, 100), (2, 40000)])
@pytest.mark.parametrize("with_x", [True, False])
def test_add_rmsnorm(dtype, rows, hidden, with_x):
    g = torch.Generator(device="cuda").manual_seed(rows * 131 + hidden)
    res = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype) if with_x else None
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(dtype)
    want_h = res + x if with_x else res.clone()
    out = add_rmsnorm(x, res, w, 1e-5)
    torch.cuda.synchronize()
    assert torch.equal(res, want_h)                       # residual updated in place, exact
    want = _norm_ref(want_h, w, 1e-5)
    err = (out.float() - want).abs() / want.abs().clamp_min(1e-3)
    assert err.max().item() <= 1.01 * ULP[dtype], err.max().item()


def test_add_rmsnorm_matches_torch_rms_norm_on_model_shape():
    g = torch.Generator(device="cuda").manual_seed(5)
    h = torch.randn(32, 4096, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(4096, device="cuda", generator=g)).bfloat16()
    ours = add_rmsnorm(None, h.clone(), w, 1e-6)
    theirs = torch.nn.functional.rms_norm(h, (4096,), w, 1e-6)
    diff = (ours.float() - theirs.float()).abs() / theirs.float().abs().clamp_min(1e-3)
    assert diff.max().item() <= 2.02 * ULP[torch.bfloat16]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,inter", [(32, 14336), (1, 4864), (9, 18944), (4, 100),
                                        (0, 64)])
def test_silu_mul(dtype, rows, inter):
    g = torch.Generator(device="cuda").manual_seed(rows + inter)
    gu = (3 * torch.randn(rows, 2 * inter, device="cuda", generator=g)).to(dtype)
    out = silu_mul(gu)
    gate, up = gu.chunk(2, dim=-1)
    want = torch.nn.functional.silu(gate) * up
    torch.cuda.synchronize()
    assert out.shape == want.shape
    if rows:
        err = (out.float() - want.float()).abs() / want.float().abs().clamp_min(1e-3)
        assert err.max().item() <= 1.01 * ULP[dtype], err.max().item()


def test_glue_rejects_bad_arguments():
    h = torch.zeros(2, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        add_rmsnorm(None, h, torch.ones(63, device="cuda", dtype=torch.bfloat16), 1e-6)
    with pytest.raises(ValueError):
        silu_mul(torch.zeros(2, 63, device="cuda", dtype=torch.bfloat16))
