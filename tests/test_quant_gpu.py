"""GPU tests of the activation quantiser (dg_quantize_act) and of a
two-layer decode chain through it.

The quantiser must reproduce the reference's host block quantisation
(bench/bench_decode.cu:459-467, restated in the oracle) bit for bit: e4m3
bytes and fp32 scales, for any M, K, a zero block, large magnitudes and a
row stride wider than K.  The chain -- GEMM, quantise its bf16 output, GEMM
-- checks the second layer against the oracle on the quantised bytes."""

import numpy as np
import pytest
import torch

import decode_opt_b200 as dg
import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,ldx", [(1, 128, 128), (1, 16384, 16384), (3, 4096, 4096), (8, 7168, 7296),
                                     (64, 2048, 2048), (128, 16384, 16384)])
def test_quantiser_matches_oracle_bit_exact(m, k, ldx):
    g = torch.Generator().manual_seed(m * 131 + k)
    x = (torch.randn(m, ldx, generator=g) * 2.5).bfloat16()
    if k >= 256:
        x[0, 128:256] = 0.0
    if m > 1:
        x[1, :128] *= 1e4
    xd = x.cuda()
    q, s = dg.quantize_activation(xd[:, :k])
    torch.cuda.synchronize()
    want_q, want_s = oracle.quantize_rows(x[:, :k].float().numpy())
    assert np.array_equal(s.cpu().numpy(), want_s)
    assert np.array_equal(q.cpu().numpy(), want_q)


def test_two_layer_chain_through_quantiser():
    n1, k1 = 4096, 2048        # layer 1: [M, 2048] -> [M, 4096]
    n2, k2 = 2048, 4096        # layer 2: [M, 4096] -> [M, 2048]
    m = 4
    w1, ws1 = oracle.gen_weight_smoke(n1, k1, 7)
    w2, ws2 = oracle.gen_weight_smoke(n2, k2, 8)
    a, as_ = oracle.gen_activation_smoke(m, k1, 9)
    dev = "cuda"
    out1 = dg.fp8_decode_gemm(torch.from_numpy(a).to(dev), torch.from_numpy(as_).to(dev),
                              torch.from_numpy(w1).to(dev), torch.from_numpy(ws1).to(dev))
    q, s = dg.quantize_activation(out1)
    out2 = dg.fp8_decode_gemm(q, s, torch.from_numpy(w2).to(dev), torch.from_numpy(ws2).to(dev))
    torch.cuda.synchronize()
    want_q, want_s = oracle.quantize_rows(out1.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), want_q) and np.array_equal(s.cpu().numpy(), want_s)
    ref2 = oracle.compute_reference(want_q, want_s, w2, ws2, threads=8)
    from helpers import check_against_oracle
    ok, rl2, worst = check_against_oracle(out2.float().cpu().numpy(), ref2)
    assert ok, (rl2, worst)
