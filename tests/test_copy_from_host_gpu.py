"""GPU tests of dg_copy_from_host, the input copy done by a kernel that reads
pinned host memory, so that it can sit between two GEMMs under programmatic
dependent launch.

* Bytes: every size (1 byte to 100 KB) and alignment (16-byte vector path,
  byte tail, unaligned source or destination) equals the host bytes, with and
  without the PDL attribute.
* Ordering: three requests captured in one CUDA graph as "copy request i's
  input (pinned host -> the one device input buffer), GEMM request i" with
  the PDL attribute on every launch.  The copy releases the next GEMM at once
  and waits for the previous GEMM before writing the buffer, and each GEMM
  waits for its copy before reading it: every request's output must equal,
  bit for bit, a plain launch of the same configuration on that request's
  input (a GEMM that read the buffer early would see the previous request's
  bytes).
"""

import pytest
import torch

import decode_opt_b200 as dg
import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes,src_off,dst_off", [(1, 0, 0), (15, 0, 0), (16, 0, 0), (16896, 0, 0),
                                                   (100003, 0, 0), (4099, 1, 0), (4099, 0, 3), (4096, 8, 8)])
@pytest.mark.parametrize("pdl", [False, True])
def test_copy_from_host_bytes(nbytes, src_off, dst_off, pdl):
    g = torch.Generator().manual_seed(nbytes + 7 * src_off + dst_off)
    host = torch.randint(0, 256, (nbytes + src_off,), dtype=torch.uint8, generator=g).pin_memory()
    dev = torch.full((nbytes + dst_off + 5,), 0xA5, dtype=torch.uint8, device="cuda")
    src = host[src_off:]
    assert src.is_pinned()
    dg.copy_from_host(dev[dst_off:dst_off + nbytes], src, pdl_attr=pdl)
    torch.cuda.synchronize()
    assert torch.equal(dev[dst_off:dst_off + nbytes].cpu(), src)
    assert bool((dev[:dst_off] == 0xA5).all()) and bool((dev[dst_off + nbytes:] == 0xA5).all())


def test_copy_then_gemm_chain_in_graph_keeps_request_order():
    m, n, k = 4, 2048, 4096
    kb = k // 128
    w, ws = oracle.gen_weight_smoke(n, k, 31)
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, pdl=True)
    wt = dg.prepack_weight(torch.from_numpy(w).cuda(), cfg.packed_rows, cfg.layout)
    wsc = torch.from_numpy(ws).cuda()
    in_bytes = m * k + m * kb * 4
    hosts = []
    for r in range(3):
        a, a_s = oracle.gen_activation_smoke(m, k, 500 + r)
        h = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
        h[: m * k].copy_(torch.from_numpy(a).view(torch.uint8).reshape(-1))
        h[m * k:].copy_(torch.from_numpy(a_s).reshape(-1).view(torch.uint8))
        hosts.append(h)
    dev_in = torch.empty(in_bytes, dtype=torch.uint8, device="cuda")
    act = dev_in[: m * k].view(m, k)
    sc = dev_in[m * k:].view(torch.float32).view(m, kb)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.full((m, n), 3.0, dtype=torch.bfloat16, device="cuda") for _ in hosts]
    probs = [dg.Problem(m, n, k, act, wt, wsc, sc, o, None, None, status) for o in outs]
    wm = dg.make_weight_tma(cfg, probs[0])
    am = dg.make_activation_tma(cfg, probs[0])
    devptrs = [dg.host_device_pointer(h) for h in hosts]
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for h, d, p in zip(hosts, devptrs, probs):
                dg.copy_from_host(dev_in, h, stream, pdl_attr=True, src_device=d)
                assert dg.launch_with_maps(cfg, p, wm, am, stream, pdl_attr=True) == 0
    for o in outs:
        o.fill_(3.0)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, dg.status_string(int(status.item()))
    for h, o in zip(hosts, outs):
        a_dev = h[: m * k].cuda().view(m, k)
        s_dev = h[m * k:].cuda().view(torch.float32).view(m, kb)
        want = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        assert dg.launch(cfg, dg.Problem(m, n, k, a_dev, wt, wsc, s_dev, want, None, None, status)) == 0
        torch.cuda.synchronize()
        assert torch.equal(o.view(torch.int16), want.view(torch.int16))
    del graph
