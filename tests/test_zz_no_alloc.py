"""The allocation-free decode entry point agrees with the workspace one.

``mi_paged_decode_noalloc`` serves callers that cannot allocate GPU memory
themselves -- a host whose own allocator owns the device (a serving
runtime's caching pool, a fixed arena given to plugins), or code running
where a cudaMalloc is not allowed -- by keeping its split-K scratch in a
fixed array inside the library. This test calls it through the C ABI twice
in a row on different problems (so stale scratch from the first call would
show in the second) and compares each result with ``mi_paged_decode`` run
with a caller-provided workspace, within the decode tolerance. It lives in
its own file, collected last, and passes alone or after the other tests.
"""
import numpy as np
import pytest

from tests.gpu_cases import paged_case

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = 2e-2  # bf16 decode tolerance used by the other decode tests


def _i32(x):
    return torch.as_tensor(np.asarray(x, dtype=np.int32)).to(DEV)


def _tensors(c):
    return dict(q=torch.from_numpy(c["q"]).to(torch.bfloat16).to(DEV),
                pool=torch.from_numpy(c["pool"]).to(torch.bfloat16).to(DEV),
                indptr=_i32(c["indptr"]), indices=_i32(c["indices"]), last=_i32(c["last"]))


def _noalloc(c, t, out, lse, status):
    from mi_b200 import capi
    q, pool = t["q"], t["pool"]
    return capi.lib().mi_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), pool.data_ptr(), c["P"], c["ps"], c["hkv"],
        c["d"], capi.DTYPE_BF16, t["indptr"].data_ptr(), t["indices"].data_ptr(),
        t["last"].data_ptr(), len(c["lens"]), c["hq"], 1.0 / np.sqrt(c["d"]), out.data_ptr(),
        lse.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _with_workspace(c, t):
    from mi_b200.decode import BatchDecodeWithPagedKVCacheWrapper
    w = BatchDecodeWithPagedKVCacheWrapper(torch.zeros(64 << 20, dtype=torch.uint8, device=DEV))
    w.plan(t["indptr"], t["indices"], t["last"], c["hq"], c["hkv"], c["d"], c["ps"])
    return w.run(t["q"], t["pool"], return_lse=True)


def test_noalloc_decode_matches_workspace_decode_on_two_calls_in_a_row():
    cases = [
        paged_case(101, [300, 4096, 17, 1, 2500, 0, 900, 64], 32, 8, 128),
        paged_case(102, [1023, 33, 3000, 5, 700], 28, 4, 128),
    ]
    for c in cases:
        t = _tensors(c)
        b = len(c["lens"])
        out = torch.empty(b, c["hq"], c["d"], dtype=torch.bfloat16, device=DEV)
        lse = torch.empty(b, c["hq"], dtype=torch.float32, device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        rc = _noalloc(c, t, out, lse, status)
        assert rc == 0
        want, want_lse = _with_workspace(c, t)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert float((out.float() - want.float()).abs().max()) <= TOL
        fin = torch.isfinite(want_lse)
        assert torch.equal(torch.isfinite(lse), fin)
        assert float((lse[fin] - want_lse[fin]).abs().max()) <= TOL


def test_noalloc_decode_refuses_problems_beyond_its_fixed_scratch():
    from mi_b200 import capi
    c = paged_case(103, [1] * 512, 32, 8, 128)  # 512 x 8 split-K slots > 8 MiB
    t = _tensors(c)
    out = torch.empty(512, 32, 128, dtype=torch.bfloat16, device=DEV)
    lse = torch.empty(512, 32, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _noalloc(c, t, out, lse, status)
    assert rc == 3  # MI_ERR_WORKSPACE
    assert b"fixed" in capi.lib().mi_last_error()
