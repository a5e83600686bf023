"""GPU tests of dg_launch_static_scratch, the entry point that allocates
nothing: its split-K tickets and workspace live in the library's static
__device__ array.  Each case runs two calls in a row through the C ABI (the
second sees the first call's leftover scratch) and requires both outputs to
equal, bit for bit, dg_launch's on caller-allocated workspace: both run the
same plan and the split reduction sums the slabs in a fixed order, so the
results are deterministic.  Neither torch's allocator nor the device's free
memory (cudaMemGetInfo) may change across the calls.  Named so pytest
collects it last.
"""

import ctypes

import pytest

import decode_opt_b200 as dg
from decode_opt_b200 import _lib

pytestmark = pytest.mark.gpu

N, K = 4096, 7168


def _inputs(m, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    act = (torch.randn(m, K, device="cuda", generator=g) * 2).to(torch.float8_e4m3fn)
    a_s = torch.rand(m, K // 128, device="cuda", generator=g) * 0.02 + 0.001
    return act, a_s


def _weight(layout):
    import torch
    g = torch.Generator(device="cuda").manual_seed(7)
    w = (torch.randn(N, K, device="cuda", generator=g) * 2).to(torch.float8_e4m3fn)
    w_s = torch.rand((N + 127) // 128, K // 128, device="cuda", generator=g) * 0.02 + 0.001
    w_dev = w if layout == dg.LAYOUT_RAW else dg.prepack_weight(w, 256, layout)
    return w_dev, w_s


def _with_workspace(cfg, m, act, a_s, w_dev, w_s, status):
    """dg_launch with caller-allocated split-K scratch (the existing path)."""
    import torch
    plan = cfg.plan(m, N, K)
    assert plan.error is None, plan.error
    ws = torch.empty(max(plan.ws_floats, 1), dtype=torch.float32, device="cuda")
    sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device="cuda")
    out = torch.zeros(m, N, dtype=torch.bfloat16, device="cuda")
    p = dg.Problem(m, N, K, act, w_dev, w_s, a_s, out, ws, sem, status)
    rc = _lib.lib().dg_launch(ctypes.byref(cfg.to_dg()), ctypes.byref(p.to_dg()),
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out


def _static_call(cfg, m, act, a_s, w_dev, w_s, out, status, stream=None):
    import torch
    # splitk_ws / splitk_sem are ignored: pass NULL.
    p = dg.Problem(m, N, K, act, w_dev, w_s, a_s, out, None, None, status)
    info = _lib.DgPlanInfo()
    s = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
    rc = _lib.lib().dg_launch_static_scratch(ctypes.byref(cfg.to_dg()), ctypes.byref(p.to_dg()), s,
                                             ctypes.byref(info))
    return rc, info


def _bit_equal(got, want):
    import torch
    return torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("m,layout", [(1, dg.LAYOUT_PACKED_SWIZZLED), (8, dg.LAYOUT_RAW),
                                      (32, dg.LAYOUT_PACKED_SWIZZLED)])
def test_static_scratch_matches_dg_launch_twice(m, layout):
    import torch
    cfg = dg.default_config(m, N, K, layout=layout, schedule="stream_k")
    w_dev, w_s = _weight(layout)
    inputs = [_inputs(m, 100 + m), _inputs(m, 200 + m)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    wants = [_with_workspace(cfg, m, a, s, w_dev, w_s, status) for a, s in inputs]
    outs = [torch.zeros(m, N, dtype=torch.bfloat16, device="cuda") for _ in inputs]
    warm = torch.zeros(m, N, dtype=torch.bfloat16, device="cuda")
    # One call first: the library looks up its array's address on the first
    # call on a device and the kernel module may load lazily.
    rc, info = _static_call(cfg, m, *inputs[0], w_dev, w_s, warm, status)
    assert rc == 0, info.error
    torch.cuda.synchronize()
    allocated = torch.cuda.memory_allocated()
    free_before, _ = torch.cuda.mem_get_info()
    for (act, a_s), out in zip(inputs, outs):
        rc, info = _static_call(cfg, m, act, a_s, w_dev, w_s, out, status)
        assert rc == 0, info.error
        assert info.max_slabs > 1, "the case must split tiles, so that the static scratch is used"
        assert info.ws_floats <= _lib.STATIC_WS_FLOATS
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == allocated
    assert free_after == free_before, (free_before, free_after)
    assert int(status.item()) == 0, dg.status_string(int(status.item()))
    for got, want in zip(outs, wants):
        assert _bit_equal(got, want)


def test_static_scratch_recovers_after_an_aborted_call():
    """A call whose CTAs abort (the test hook makes one bounded wait run out)
    leaves tickets of the shared array non-zero; the next call clears the
    tickets it uses and must again equal dg_launch bit for bit."""
    import torch
    m, layout = 8, dg.LAYOUT_PACKED_SWIZZLED
    cfg = dg.default_config(m, N, K, layout=layout, schedule="stream_k")
    w_dev, w_s = _weight(layout)
    act, a_s = _inputs(m, 300)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = _with_workspace(cfg, m, act, a_s, w_dev, w_s, status)
    torch.cuda.synchronize()
    from dataclasses import replace
    bad = replace(cfg, flags=cfg.flags | dg.FLAG_INJECT_TIMEOUT, timeout_ns=20_000_000)
    junk = torch.zeros(m, N, dtype=torch.bfloat16, device="cuda")
    # On caller-allocated scratch the same aborted call visibly leaves a
    # ticket non-zero (CTA 0 never arrives at the tile it shares).
    plan = cfg.plan(m, N, K)
    sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device="cuda")
    ws = torch.empty(max(plan.ws_floats, 1), dtype=torch.float32, device="cuda")
    p = dg.Problem(m, N, K, act, w_dev, w_s, a_s, junk, ws, sem, status)
    assert _lib.lib().dg_launch(ctypes.byref(bad.to_dg()), ctypes.byref(p.to_dg()),
                                torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == dg.ERR_INJECTED_TIMEOUT
    assert int(sem.ne(0).sum().item()) > 0
    status.zero_()
    rc, info = _static_call(bad, m, act, a_s, w_dev, w_s, junk, status)
    assert rc == 0, info.error
    torch.cuda.synchronize()
    assert int(status.item()) == dg.ERR_INJECTED_TIMEOUT, dg.status_string(int(status.item()))
    status.zero_()
    out = torch.zeros(m, N, dtype=torch.bfloat16, device="cuda")
    rc, info = _static_call(cfg, m, act, a_s, w_dev, w_s, out, status)
    assert rc == 0, info.error
    torch.cuda.synchronize()
    assert int(status.item()) == 0, dg.status_string(int(status.item()))
    assert _bit_equal(out, want)


def test_static_scratch_rejects_plans_over_the_limit():
    import torch
    m, n, k = 128, 7168, 16384
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_RAW, schedule="stream_k")
    plan = cfg.plan(m, n, k)
    assert plan.error is None and plan.ws_floats > _lib.STATIC_WS_FLOATS
    act = torch.zeros(m, k, dtype=torch.uint8, device="cuda")
    w = torch.zeros(n, k, dtype=torch.uint8, device="cuda")
    w_s = torch.ones((n + 127) // 128, k // 128, device="cuda")
    a_s = torch.ones(m, k // 128, device="cuda")
    out = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    p = dg.Problem(m, n, k, act, w, w_s, a_s, out, None, None, None)
    info = _lib.DgPlanInfo()
    rc = _lib.lib().dg_launch_static_scratch(ctypes.byref(cfg.to_dg()), ctypes.byref(p.to_dg()),
                                             torch.cuda.current_stream().cuda_stream, ctypes.byref(info))
    assert rc == dg.CUDA_ERROR_INVALID_VALUE
    assert b"static scratch too small" in info.error
    torch.cuda.synchronize()
    assert not out.any()
