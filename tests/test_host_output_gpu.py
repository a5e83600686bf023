"""GPU test of the zero-copy output (dg_host_device_pointer): a GEMM given the
device address of pinned host memory as its output writes the bf16 result
straight into host memory.  It must equal, bit for bit, the same launch into
a device buffer, on the cluster and stream-K schedules, and the lines gather
with a world of one may unpack into host memory the same way.  Memory that is
not pinned is refused by the library before any launch."""

import ctypes

import numpy as np
import pytest
import torch

import decode_opt_b200 as dg
from decode_opt_b200 import _lib, tp

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed):
    import oracle
    w, ws = oracle.gen_weight_smoke(n, k, seed)
    a, as_ = oracle.gen_activation_smoke(m, k, seed + 1)
    return w, ws, a, as_


@pytest.mark.parametrize("schedule", ["cluster", "stream_k"])
@pytest.mark.parametrize("m", [1, 8])
def test_output_into_pinned_host_memory(m, schedule):
    n, k = 2048, 4096
    w, ws, a, as_ = _case(m, n, k, 1234 + m)
    dev = "cuda"
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, schedule=schedule)
    plan = cfg.plan(m, n, k)
    wt = dg.prepack_weight(torch.from_numpy(w).to(dev), cfg.block_n, cfg.layout)
    wsb = torch.zeros(max(plan.ws_floats, 1), device=dev)
    sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    act, asd, wsd = torch.from_numpy(a).to(dev), torch.from_numpy(as_).to(dev), torch.from_numpy(ws).to(dev)
    out_d = torch.zeros((m, n), dtype=torch.bfloat16, device=dev)
    out_h = torch.full((m, n), 3.0, dtype=torch.bfloat16).pin_memory()
    p_d = dg.Problem(m, n, k, act, wt, wsd, asd, out_d, wsb, sem, status)
    p_h = dg.Problem(m, n, k, act, wt, wsd, asd, dg.host_device_pointer(out_h), wsb, sem, status)
    assert dg.launch(cfg, p_d) == 0
    assert dg.launch(cfg, p_h) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out_h.view(torch.int16), out_d.cpu().view(torch.int16))


def test_lines_world_one_unpacks_into_host_memory():
    m, n, k = 3, 1024, 2048
    w, ws, a, as_ = _case(m, n, k, 555)
    dev = "cuda"
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED)
    wt = dg.prepack_weight(torch.from_numpy(w).to(dev), cfg.block_n, cfg.layout)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out_d = torch.zeros((m, n), dtype=torch.bfloat16, device=dev)
    p = dg.Problem(m, n, k, torch.from_numpy(a).to(dev), wt, torch.from_numpy(ws).to(dev),
                   torch.from_numpy(as_).to(dev), out_d, None, None, status)
    wm, am = dg.make_weight_tma(cfg, p), dg.make_activation_tma(cfg, p)
    assert dg.launch_with_maps(cfg, p, wm, am) == 0
    out_h = torch.zeros((m, n), dtype=torch.bfloat16).pin_memory()
    sync = torch.zeros(2, dtype=torch.int32, device=dev)
    g = tp.lines_descriptor(1, 0, n, dg.host_device_pointer(out_h), [0], sync.data_ptr())
    assert dg.launch_gather(cfg, p, g, wm, am) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(out_h.view(torch.int16), out_d.cpu().view(torch.int16))


def test_unpinned_memory_is_refused():
    buf = np.zeros(64, np.uint16)
    out = ctypes.c_void_p(7)
    rc = _lib.lib().dg_host_device_pointer(ctypes.c_void_p(buf.ctypes.data), ctypes.byref(out))
    assert rc != 0 and out.value == 7
    with pytest.raises(ValueError):
        dg.host_device_pointer(torch.zeros(4))
    # the refusal left no error behind
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0
