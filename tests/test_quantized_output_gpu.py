"""GPU parity of the GEMM with the next layer's activation quantisation fused
into its cluster reduction (``dg_launch_quantized``).

The reference's decode chain quantises every layer's bf16 output into the
next layer's e4m3 activation with fp32 1x128 scales as a separate step (the
host block quantisation of bench/bench_decode.cu:459-467; here the
standalone ``dg_quantize_act`` kernel).  The fused launch must give, on the
same inputs:

* the bf16 output bit-identical to the unfused launch of the same
  configuration (the reduction sums the same partials in the same order),
  and within the reference's gate of the oracle;
* e4m3 bytes and scales identical to the standalone quantiser's on that
  output, and to the oracle's restatement of the reference's quantisation.

Then a dependent chain of fused layers captured in a CUDA graph with
programmatic dependent launch (one kernel per layer instead of two) must end
on exactly the bytes of the unfused chain, with every layer checked against
the oracle.  Every buffer the kernels write starts as random bytes.
"""

import numpy as np
import pytest
import torch

import decode_opt_b200 as dg
import oracle
from helpers import check_against_oracle

pytestmark = pytest.mark.gpu


def quantize_blocks(w):
    """float32 [n, k] (device) -> e4m3 bytes [n, k] and 128x128 block scales."""
    n, k = w.shape
    nb = (n + 127) // 128
    wp = torch.zeros((nb * 128, k), device=w.device)
    wp[:n] = w
    blocks = wp.view(nb, 128, k // 128, 128)
    scale = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-4) / 448.0
    q = (blocks / scale[:, None, :, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.view(nb * 128, k)[:n].contiguous().view(torch.uint8), scale.contiguous()


def garbage(t, gen):
    b = t.view(torch.uint8).view(-1)
    b.copy_(torch.randint(0, 256, b.shape, device=t.device, dtype=torch.uint8, generator=gen))


class Layer:
    def __init__(self, m, n, k, seed, layout=dg.LAYOUT_PACKED_SWIZZLED, independent=False, scale=1.0):
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(seed)
        self.m, self.n, self.k = m, n, k
        self.w, self.w_sc = quantize_blocks(torch.randn((n, k), device=dev, generator=g) * scale / k ** 0.5)
        self.cfg = dg.default_config(m, n, k, layout=layout, pdl=True, independent_inputs=independent,
                                     quantized_output=True)
        self.w_dev = self.w if layout == dg.LAYOUT_RAW else dg.prepack_weight(self.w, self.cfg.packed_rows, layout)
        plan = self.cfg.plan(m, n, k)
        assert plan.error is None and plan.cluster >= 2 and self.cfg.block_n % 128 == 0, plan.error
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    def problem(self, act, act_sc, out):
        return dg.Problem(self.m, self.n, self.k, act, self.w_dev, self.w_sc, act_sc, out, None, None, self.status)


SHAPES = [
    (1, 7168, 16384), (1, 16384, 7168), (8, 7168, 16384), (16, 2048, 7168), (32, 4096, 2048),
    (64, 2048, 4096), (128, 2048, 4096), (5, 384, 1024), (3, 640, 512), (128, 128, 256),
]


@pytest.mark.parametrize("independent", [False, True])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_fused_quantisation_equals_gemm_then_quantiser(m, n, k, independent):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1000 + m + n + k)
    L = Layer(m, n, k, seed=7 * m + n, independent=independent)
    a, a_sc = dg.quantize_activation(torch.randn((m, k), device=dev, generator=g).bfloat16())
    out_ref = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(out_ref)
    q = torch.empty((m, n), dtype=torch.uint8, device=dev)
    qs = torch.empty((m, n // 128), dtype=torch.float32, device=dev)
    for t in (out_ref, out, q, qs):
        garbage(t, g)

    p_ref = L.problem(a, a_sc, out_ref)
    wm, am = dg.make_weight_tma(L.cfg, p_ref), dg.make_activation_tma(L.cfg, p_ref)
    assert dg.launch_with_maps(L.cfg, p_ref, wm, am) == 0
    torch.cuda.synchronize()
    assert int(L.status.item()) == 0
    p = L.problem(a, a_sc, out)
    assert dg.launch_quantized(L.cfg, p, wm, dg.make_activation_tma(L.cfg, p), q, qs) == 0
    torch.cuda.synchronize()
    assert int(L.status.item()) == 0, dg.status_string(int(L.status.item()))

    assert torch.equal(out.view(torch.int16), out_ref.view(torch.int16))
    want_q, want_s = dg.quantize_activation(out)
    torch.cuda.synchronize()
    assert torch.equal(q, want_q)
    assert torch.equal(qs, want_s)
    host = out.float().cpu().numpy()
    oq, os_ = oracle.quantize_rows(host)
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(qs.cpu().numpy(), os_)
    if m * n * k <= 64 * 2048 * 4096:
        want = oracle.compute_reference(a.cpu().numpy(), a_sc.cpu().numpy(), L.w.cpu().numpy(),
                                        L.w_sc.cpu().numpy(), threads=8)
        ok, rl2, worst = check_against_oracle(host, want)
        assert ok, (rl2, worst)


def test_saturation_and_tiny_blocks():
    """Large outputs clamp at +-448 after scaling (the amax element maps to
    exactly 448) and an all-zero block gets the 1e-4 floor: one row of zero
    activations and one of huge ones."""
    dev = torch.device("cuda")
    m, n, k = 4, 1024, 1024
    g = torch.Generator(device=dev).manual_seed(5)
    L = Layer(m, n, k, seed=5, scale=300.0)
    x = torch.randn((m, k), device=dev, generator=g)
    x[1] = 0.0
    x[2] *= 1000.0
    a, a_sc = dg.quantize_activation(x.bfloat16())
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    q = torch.empty((m, n), dtype=torch.uint8, device=dev)
    qs = torch.empty((m, n // 128), dtype=torch.float32, device=dev)
    for t in (out, q, qs):
        garbage(t, g)
    p = L.problem(a, a_sc, out)
    assert dg.launch_quantized(L.cfg, p, dg.make_weight_tma(L.cfg, p), dg.make_activation_tma(L.cfg, p), q, qs) == 0
    torch.cuda.synchronize()
    assert int(L.status.item()) == 0
    oq, os_ = oracle.quantize_rows(out.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), oq) and np.array_equal(qs.cpu().numpy(), os_)
    assert float(qs[1].max()) == np.float32(1e-4) / np.float32(448.0)
    assert bool((q[1] == 0).all())
    assert 0x7e in set(q[2].cpu().numpy().tolist()) or 0xfe in set(q[2].cpu().numpy().tolist())   # +-448


def test_rejections():
    """Configurations the fused quantiser cannot serve are refused with
    cudaErrorInvalidValue before any launch: a stream-K plan, 224-row tiles,
    N not a multiple of 128, a misaligned destination, wrong shapes."""
    dev = torch.device("cuda")
    m, n, k = 2, 1792, 1024
    L = Layer(m, n, k, seed=11)
    a, a_sc = dg.quantize_activation(torch.randn((m, k), device=dev).bfloat16())
    out = torch.zeros((m, n), dtype=torch.bfloat16, device=dev)
    q = torch.zeros((m, n), dtype=torch.uint8, device=dev)
    qs = torch.zeros((m, n // 128), dtype=torch.float32, device=dev)
    p = L.problem(a, a_sc, out)
    wm, am = dg.make_weight_tma(L.cfg, p), dg.make_activation_tma(L.cfg, p)
    from dataclasses import replace
    sk = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, schedule="stream_k")
    assert dg.launch_quantized(sk, p, wm, am, q, qs) == dg.CUDA_ERROR_INVALID_VALUE
    c224 = replace(L.cfg, block_n=224)
    assert dg.launch_quantized(c224, p, wm, am, q, qs) == dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_quantized(L.cfg, p, wm, am, q[:, 1:], qs) == dg.CUDA_ERROR_INVALID_VALUE
    q_off = torch.zeros(m * n + 4, dtype=torch.uint8, device=dev)[1:1 + m * n].view(m, n)
    assert dg.launch_quantized(L.cfg, p, wm, am, q_off, qs) == dg.CUDA_ERROR_INVALID_VALUE
    with pytest.raises(ValueError):
        dg.default_config(m, 1000, k, quantized_output=True)
    torch.cuda.synchronize()
    assert int(L.status.item()) == 0
    assert not bool(q.any()) and not bool(out.view(torch.int16).any())


@pytest.mark.parametrize("m,n,k,layers", [(1, 7168, 16384, 6), (8, 7168, 16384, 4), (64, 2048, 4096, 6)])
def test_fused_chain_in_graph_equals_unfused_chain(m, n, k, layers):
    dev = torch.device("cuda")
    shapes = [(n, k) if i % 2 == 0 else (k, n) for i in range(layers)]
    Ls = [Layer(m, nn, kk, seed=300 + i) for i, (nn, kk) in enumerate(shapes)]
    g = torch.Generator(device=dev).manual_seed(99)
    a0, s0 = dg.quantize_activation(torch.randn((m, k), device=dev, generator=g).bfloat16())
    torch.cuda.synchronize()

    def buffers():
        acts = [a0.clone()] + [torch.empty((m, nn), dtype=torch.uint8, device=dev) for (nn, _) in shapes]
        scs = [s0.clone()] + [torch.empty((m, nn // 128), device=dev) for (nn, _) in shapes]
        outs = [torch.empty((m, nn), dtype=torch.bfloat16, device=dev) for (nn, _) in shapes]
        for t in acts[1:] + scs[1:] + outs:
            garbage(t, g)
        return acts, scs, outs

    def capture(fused, acts, scs, outs):
        stream = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(graph, stream=stream):
                for j, L in enumerate(Ls):
                    p = L.problem(acts[j], scs[j], outs[j])
                    wm, am = dg.make_weight_tma(L.cfg, p), dg.make_activation_tma(L.cfg, p)
                    if fused:
                        assert dg.launch_quantized(L.cfg, p, wm, am, acts[j + 1], scs[j + 1], stream,
                                                   pdl_attr=True) == 0
                    else:
                        assert dg.launch_with_maps(L.cfg, p, wm, am, stream, pdl_attr=True) == 0
                        dg.quantize_activation(outs[j], out=acts[j + 1], scales=scs[j + 1], stream=stream,
                                               pdl_attr=True)
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        return graph

    fa, fs, fo = buffers()
    gf = capture(True, fa, fs, fo)
    ua, us, uo = buffers()
    gu = capture(False, ua, us, uo)
    assert all(int(L.status.item()) == 0 for L in Ls)
    for j, L in enumerate(Ls):
        assert torch.equal(fo[j].view(torch.int16), uo[j].view(torch.int16)), j
        assert torch.equal(fa[j + 1], ua[j + 1]) and torch.equal(fs[j + 1], us[j + 1]), j
        got = fo[j].float().cpu().numpy()
        want = oracle.compute_reference(fa[j].cpu().numpy(), fs[j].cpu().numpy(), L.w.cpu().numpy(),
                                        L.w_sc.cpu().numpy(), threads=8)
        ok, rl2, worst = check_against_oracle(got, want)
        assert ok, (j, rl2, worst)
        oq, os_ = oracle.quantize_rows(got)
        assert np.array_equal(fa[j + 1].cpu().numpy(), oq) and np.array_equal(fs[j + 1].cpu().numpy(), os_), j
    del gf, gu
