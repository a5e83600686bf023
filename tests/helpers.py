"""Shared test helpers: oracle data on the host, device copies, one GEMM call
through the C ABI, and the reference's acceptance checks."""

from __future__ import annotations

import functools

import numpy as np

import oracle


@functools.lru_cache(maxsize=8)
def smoke_weight(n: int, k: int, seed: int):
    return oracle.gen_weight_smoke(n, k, seed)


@functools.lru_cache(maxsize=32)
def smoke_case(n: int, k: int, seed: int, m: int):
    """Inputs and the oracle output of one reference smoke-test case."""
    w, ws = smoke_weight(n, k, seed)
    a, as_ = oracle.gen_activation_smoke(m, k, oracle.smoke_act_seed(seed, m))
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    return w, ws, a, as_, ref


class DeviceCase:
    """Device copies of one problem plus the buffers a launch needs."""

    def __init__(self, w, ws, a, as_, n: int, device="cuda"):
        import torch
        self.torch = torch
        self.n = n
        self.k = w.shape[1]
        self.m = a.shape[0]
        self.w = torch.from_numpy(np.ascontiguousarray(w)).to(device)
        self.ws = torch.from_numpy(np.ascontiguousarray(ws)).to(device)
        self.a = torch.from_numpy(np.ascontiguousarray(a)).to(device)
        self.as_ = torch.from_numpy(np.ascontiguousarray(as_)).to(device)
        self.out = torch.zeros((self.m, n), dtype=torch.bfloat16, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.splitk_ws = None
        self.sem = None
        self.packed = {}

    def weight_for(self, cfg):
        import decode_opt_b200 as dg
        if cfg.layout == dg.LAYOUT_RAW:
            return self.w
        key = (cfg.packed_rows, cfg.layout)
        if key not in self.packed:
            self.packed[key] = dg.prepack_weight(self.w, cfg.packed_rows, cfg.layout)
        return self.packed[key]

    def run(self, cfg, clear_out: bool = True, stream=None, ws_offset: int = 0):
        """One launch through the C ABI; returns (rc, out as float32 numpy, status).
        ``ws_offset`` floats shift the split workspace off its 16-byte alignment."""
        import decode_opt_b200 as dg
        torch = self.torch
        plan = cfg.plan(self.m, self.n, self.k)
        assert plan.error is None, plan.error
        need = plan.ws_floats + ws_offset
        if plan.ws_floats and (self.splitk_ws is None or self.splitk_ws.numel() < need):
            self.splitk_ws = torch.zeros(need, dtype=torch.float32, device=self.w.device)
        if plan.sem_ints and (self.sem is None or self.sem.numel() < plan.sem_ints):
            self.sem = torch.zeros(plan.sem_ints, dtype=torch.int32, device=self.w.device)
        if clear_out:
            self.out.zero_()
        self.status.zero_()
        ws = self.splitk_ws[ws_offset:] if (self.splitk_ws is not None and ws_offset) else self.splitk_ws
        p = dg.Problem(self.m, self.n, self.k, self.a, self.weight_for(cfg), self.ws, self.as_, self.out,
                       ws, self.sem, self.status)
        rc = dg.launch(cfg, p, stream)
        torch.cuda.synchronize()
        got = self.out.float().cpu().numpy()
        return rc, got, int(self.status.item())

    def sem_clean(self) -> bool:
        return self.sem is None or int(self.sem.abs().sum().item()) == 0


def check_against_oracle(got: np.ndarray, ref: np.ndarray):
    """The reference's gate (rel_l2 <= 2e-3, all finite) plus the per-element
    bound |got-want| <= 1e-2 * max(|want|, 1e-2*rms(want))."""
    rl2 = oracle.rel_l2(got, ref)
    ok_elem, worst = oracle.elementwise_ok(got, ref, rel=1e-2, floor_frac=1e-2)
    finite = bool(np.isfinite(got).all())
    return finite and rl2 <= oracle.REL_L2_GATE and ok_elem, rl2, worst
