"""Peer-memory plumbing of the tensor-parallel all-reduce on one GPU.

* The bounded barrier of ``mi_allreduce_add_rmsnorm`` gives up: world 2 on
  one GPU, both "peer" bases pointing at this GPU's own buffer, so the second
  rank's flag is never written. With a 10 ms limit the launch must end, flag
  MI_STATUS_TIMEOUT, leave the outputs unwritten, and the GPU must take the
  next launch (the same call at world 1, checked against torch).
* The IPC mapping (``mi_ipc_export`` / ``mi_ipc_open``) works between two
  processes on the same GPU: the child maps the parent's buffer, reads a
  pattern through the mapping and writes one back. Plain copies only: no
  kernel waits on another process.
"""
import multiprocessing as mp

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TIMEOUT_BIT = 64


def _ar_call(lib, bases, rank, world, residual, weight, out, rows, hidden, status, counters):
    return lib.mi_allreduce_add_rmsnorm(
        bases.data_ptr(), 4096, 0, counters.data_ptr(), rank, world, residual.data_ptr(),
        weight.data_ptr(), out.data_ptr(), rows, hidden, 1e-6, 2, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_peer_barrier_wait_runs_out_and_gpu_stays_usable():
    from mi_b200 import capi

    lib = capi.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows, hidden = 4, 256
    buf = torch.zeros(4096 + rows * hidden * 2, dtype=torch.uint8, device=dev)
    partial = buf[4096:].view(torch.bfloat16).view(rows, hidden)
    g = torch.Generator(device=dev).manual_seed(0)
    partial.copy_(torch.randn(rows, hidden, device=dev, generator=g).to(torch.bfloat16))
    residual = torch.randn(rows, hidden, device=dev, generator=g).to(torch.bfloat16)
    res0 = residual.clone()
    weight = torch.randn(hidden, device=dev, generator=g).to(torch.bfloat16)
    out = torch.full((rows, hidden), 7.0, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    counters = torch.zeros(256, dtype=torch.int32, device=dev)
    bases = torch.tensor([buf.data_ptr(), buf.data_ptr()], dtype=torch.int64, device=dev)
    assert lib.mi_set_peer_wait_limit_ns(10_000_000) == 0          # 10 ms
    try:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        assert _ar_call(lib, bases, 0, 2, residual, weight, out, rows, hidden, status,
                        counters) == 0
        ev1.record()
        torch.cuda.synchronize()
    finally:
        lib.mi_set_peer_wait_limit_ns(0)
    assert int(status.item()) & TIMEOUT_BIT
    ms = ev0.elapsed_time(ev1)
    assert 5.0 <= ms < 2000.0, ms                      # gave up near the limit, not at 10 s
    assert torch.equal(residual, res0)                  # nothing written after the give-up
    assert torch.equal(out, torch.full_like(out, 7.0))

    # the context is still usable: the same call at world 1 runs and is right
    status.zero_()
    one = bases[:1].clone()
    assert _ar_call(lib, one, 0, 1, residual, weight, out, rows, hidden, status,
                    counters) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    h = (res0.float() + partial.float()).to(torch.bfloat16)
    assert torch.equal(residual, h)
    want = torch.nn.functional.rms_norm(h.float(), (hidden,), eps=1e-6) * weight.float()
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=1e-2)


def test_ipc_mapping_between_two_processes_on_one_gpu():
    import ctypes

    from mi_b200 import capi

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = 1 << 20
    pad = torch.empty(12345, dtype=torch.uint8, device=dev)      # buffer not at a segment start
    buf = torch.zeros(n, dtype=torch.uint8, device=dev)
    pattern = (torch.arange(n // 2, device=dev) * 7 % 251).to(torch.uint8)
    buf[: n // 2].copy_(pattern)
    torch.cuda.synchronize()
    handle = ctypes.create_string_buffer(capi.IPC_HANDLE_BYTES)
    offset = ctypes.c_int64(-1)
    capi.call("mi_ipc_export", buf.data_ptr(), ctypes.addressof(handle), ctypes.addressof(offset))
    assert offset.value >= 0
    from tests.tp_workers import ipc_child

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=ipc_child, args=(bytes(handle.raw), offset.value, n, q))
    p.start()
    res = q.get(timeout=300)
    p.join(timeout=120)
    assert res[0] == "ok", res
    assert p.exitcode == 0
    assert res[2] == 0
    assert res[1] == pattern.cpu().numpy().tobytes()
    want = (np.arange(n - n // 2) & 0xFF).astype(np.uint8) ^ 0x5A
    assert np.array_equal(buf[n // 2:].cpu().numpy(), want)
    del pad
