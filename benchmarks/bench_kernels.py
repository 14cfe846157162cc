"""Kernel microbenchmarks: the sm_100a flash-attention forward/backward against PyTorch's
cuDNN SDPA (the reference's attention backend on cc 10.0), and the flash-attention JVP forward
against the reference's own Triton kernel (`_attention` in
train/wan/rcm/utils/flash_attention_jvp_triton.py, run from the installed copy under
baseline/_ref), at Wan shapes.

    python -m benchmarks.bench_kernels --L 32760 --H 12 --B 1          # timing (CUDA events)
    python -m benchmarks.bench_kernels --L 4096 --H 4 --iters 1 --warmup 1 --only fwd   # small case for ncu

Prints one JSON line per op: ms, achieved TFLOP/s and the fraction of the measured
cuBLAS bf16 peak (MEASURED_PEAKS.json when present).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch


def peak_tflops():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def _peak_hbm():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"])
    except Exception:
        return 6650.0


def _reference_jvp():
    """The reference's Triton JVP attention (`_attention.apply`) from baseline/_ref, or None."""
    import sys

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "rcm")):
        return None
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        import matplotlib.pyplot  # noqa: F401
    except ImportError:
        # the reference's mask module imports pyplot for a debug plot only; matplotlib is not in this
        # image, so an empty stand-in module lets the (unmodified) kernel module import
        import types

        class _Stub(types.ModuleType):
            def __getattr__(self, name):  # any attribute used only in annotations / plotting code
                if name.startswith("__"):
                    raise AttributeError(name)
                return type(name, (), {})

        for name in ("matplotlib", "matplotlib.pyplot", "matplotlib.patches"):
            sys.modules.setdefault(name, _Stub(name))
        sys.modules["matplotlib"].pyplot = sys.modules["matplotlib.pyplot"]
        sys.modules["matplotlib"].patches = sys.modules["matplotlib.patches"]
    from rcm.utils.flash_attention_jvp_triton import attention

    return attention


def timeit(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--L", type=int, default=32760)
    ap.add_argument("--Lk", type=int, default=None)
    ap.add_argument("--H", type=int, default=12)
    ap.add_argument("--D", type=int, default=128, choices=[64, 128], help="head dim of the attention benchmarks")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", default="all", choices=["all", "fwd", "bwd", "bwd_fused", "sdpa", "jvp", "ref_jvp", "gemm",
                                                      "rows"])
    ap.add_argument("--gemm", default="32760,8960,1536", help="M,N,K of the GEMM benchmark")
    ap.add_argument("--rank", type=int, default=128, help="LoRA rank of the GEMM benchmark")
    a = ap.parse_args()
    from dmad_b200 import ops

    e = ops.ext()
    B, L, H = a.B, a.L, a.H
    Lk = a.Lk or L
    torch.manual_seed(0)
    D = a.D
    q = torch.randn(B, L, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, Lk, H, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, Lk, H, D, device="cuda", dtype=torch.bfloat16)
    do = torch.randn_like(q)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(L), device="cuda")
    scale = 1 / math.sqrt(D)
    fl_fwd = 4.0 * B * H * L * Lk * D
    peak, src = peak_tflops()
    res = []
    if a.only in ("all", "fwd"):
        ms = timeit(lambda: e.flash_fwd(q, k, v, o, lse, scale), a.iters, a.warmup)
        res.append(("flash_fwd_sm100", ms, fl_fwd))
    if a.only in ("all", "bwd"):
        e.flash_fwd(q, k, v, o, lse, scale)
        dq, dk, dv, dd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(lse)
        ms = timeit(lambda: e.flash_bwd(q, k, v, o, do, lse, dq, dk, dv, dd, scale), a.iters, a.warmup)
        res.append(("flash_bwd_sm100", ms, 2.5 * fl_fwd))
    if a.only in ("all", "bwd", "bwd_fused") and D == 128:
        e.flash_fwd(q, k, v, o, lse, scale)
        dq, dk, dv, dd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(lse)
        acc = torch.empty(B * H * lse.shape[-1] * 128, device="cuda")
        ms = timeit(lambda: e.flash_bwd_fused(q, k, v, o, do, lse, dq, dk, dv, dd, acc, scale), a.iters, a.warmup)
        res.append(("flash_bwd_fused_sm100", ms, 2.5 * fl_fwd))
    if a.only in ("all", "sdpa"):
        from torch.nn.attention import SDPBackend, sdpa_kernel

        qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            ms = timeit(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt), a.iters, a.warmup)
            res.append(("cudnn_sdpa_fwd", ms, fl_fwd))
            qg, kg, vg = (t.detach().requires_grad_(True) for t in (qt, kt, vt))
            out = torch.nn.functional.scaled_dot_product_attention(qg, kg, vg)
            gt = do.transpose(1, 2)
            ms = timeit(lambda: torch.autograd.grad(out, (qg, kg, vg), gt, retain_graph=True), a.iters, a.warmup)
            res.append(("cudnn_sdpa_bwd", ms, 2.5 * fl_fwd))
    if a.only in ("all", "jvp", "ref_jvp") and D == 128:
        tq, tk, tv = (torch.randn_like(t) * 0.5 for t in (q, k, v))
        to = torch.empty_like(q)
        fl_jvp = 3.0 * fl_fwd  # S, tq k^T, q tk^T, P V, P tV, (P * tS) V
        if a.only in ("all", "jvp"):
            ms = timeit(lambda: e.flash_jvp_fwd(q, k, v, tq, tk, tv, o, to, lse, scale), a.iters, a.warmup)
            res.append(("flash_jvp_fwd_sm100", ms, fl_jvp))
        if a.only in ("all", "ref_jvp"):
            ref = _reference_jvp()
            if ref is None:
                print(json.dumps({"op": "reference_triton_jvp_fwd", "unavailable": "baseline/_ref not installed"}))
            else:
                qt, kt, vt, tqt, tkt, tvt = (t.transpose(1, 2).contiguous() for t in (q, k, v, tq, tk, tv))
                ms = timeit(lambda: ref(qt, kt, vt, tqt, tkt, tvt, scale), a.iters, a.warmup)
                res.append(("reference_triton_jvp_fwd", ms, fl_jvp))
    if a.only == "gemm":
        M, N, K = (int(v) for v in a.gemm.split(","))
        r = a.rank
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * K ** -0.5
        la = torch.randn(r, K, device="cuda", dtype=torch.bfloat16) * K ** -0.5
        lb = torch.randn(N, r, device="cuda", dtype=torch.bfloat16) * 0.01
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        xa = torch.empty(M, r, device="cuda", dtype=torch.bfloat16)
        fl = 2.0 * M * N * K
        ms = timeit(lambda: e.gemm_bf16(x, w, None, None, None, y, 1.0, 0), a.iters, a.warmup)
        res.append(("gemm_sm100", ms, fl))
        ms = timeit(lambda: torch.matmul(x, w.t(), out=y), a.iters, a.warmup)
        res.append(("cublas_gemm", ms, fl))

        def ours_lora():
            e.gemm_bf16(x, la, None, None, None, xa, 0.5, 0)
            e.gemm_bf16(x, w, xa, lb, None, y, 1.0, 0)

        def peft_lora():
            torch.matmul(x, w.t(), out=y)
            y.add_(torch.matmul(torch.matmul(x, la.t()), lb.t()), alpha=0.5)

        fl_lora = fl + 2.0 * M * r * (K + N)
        res.append(("lora_linear_sm100", timeit(ours_lora, a.iters, a.warmup), fl_lora))
        res.append(("cublas_linear_plus_lora", timeit(peft_lora, a.iters, a.warmup), fl_lora))
    if a.only == "rows":
        # the memory-bound row kernels of a Wan-1.3B block at 32,760 tokens: bytes moved per call against
        # the measured copy bandwidth
        import torch.nn.functional as F
        from dmad_b200 import ops as O
        R, D, F_ = 32760, 1536, 8960
        hbm = _peak_hbm()
        x = torch.randn(R, D, device="cuda", dtype=torch.bfloat16)
        amod = torch.randn(21, D, device="cuda") * 0.1
        cmod = torch.randn(21, D, device="cuda") * 0.1
        qkv = torch.randn(R, 3 * D, device="cuda", dtype=torch.bfloat16)
        wq, wk = torch.ones(D, device="cuda"), torch.ones(D, device="cuda")
        ang = torch.rand(R, 64, device="cuda")
        cos, sin = ang.cos(), ang.sin()
        h = torch.randn(R, F_, device="cuda", dtype=torch.bfloat16)
        gate = torch.randn(21, D, device="cuda") * 0.1
        y = torch.randn_like(x)
        rows = [
            ("ln_mod_fwd", lambda: O.ln_mod(x, amod, cmod, 1.0, 1560, eps=1e-6), 2 * R * D * 2),
            ("gate_residual_fwd", lambda: O.gate_residual(x, y, gate, 1560), 3 * R * D * 2),
            ("qk_norm_rope_fwd", lambda: O.qk_norm_rope(qkv, wq, wk, cos, sin, D, 128), (3 + 2) * R * D * 2),
            ("gelu_tanh_fwd", lambda: O.gelu_tanh(h), 2 * R * F_ * 2),
        ]
        e = O.ext()
        dy, dxb = torch.randn_like(x), torch.empty_like(x)
        xf = x.float()
        mean, rstd = xf.mean(1), torch.rsqrt(xf.var(1, unbiased=False) + 1e-6)
        da, dc, dg = torch.zeros_like(amod), torch.zeros_like(cmod), torch.zeros_like(gate)
        gqk = torch.randn(R, 2 * D, device="cuda", dtype=torch.bfloat16)
        dqk = torch.empty(R, 2 * D, device="cuda", dtype=torch.bfloat16)
        rq, rk = torch.rand(R, device="cuda") + 0.5, torch.rand(R, device="cuda") + 0.5
        dwq, dwk = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
        rows += [  # backward kernels: algorithmic bytes (each input read once, each output written once)
            ("ln_mod_bwd", lambda: e.ln_mod_bwd(dy, x, mean, rstd, amod, 1.0, 1560, None, False, dxb, None, da, dc,
                                                None, None, None, None), 3 * R * D * 2),
            ("gate_residual_bwd", lambda: e.gate_res_bwd(dy, y, dxb, gate, dg, 1560, None), 3 * R * D * 2),
            ("qk_norm_rope_bwd", lambda: e.qk_norm_rope_bwd(gqk[:, :D], gqk[:, D:], qkv, dqk, wq, wk, cos, sin, rq, rk,
                                                            dwq, dwk, D, 128), 6 * R * D * 2),
        ]
        for name, fn, nbytes in rows:
            ms = timeit(fn, a.iters, a.warmup)
            print(json.dumps({"op": name, "rows": R, "ms": round(ms, 4), "GB/s": round(nbytes / ms / 1e6, 1),
                              "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3)}))
        return
    for name, ms, fl in res:
        tf = fl / (ms * 1e-3) / 1e12
        print(json.dumps({"op": name, "B": B, "L": L, "Lk": Lk, "H": H, "D": a.D, "ms": round(ms, 4), "tflops": round(tf, 1),
                          f"frac_of_{src}_bf16_peak": round(tf / peak, 3)}))


if __name__ == "__main__":
    main()
