#!/usr/bin/env python
"""GEMM microbenchmark: the tcgen05 GEMM against cuBLAS (torch.matmul) on the
GPT-1B training shapes (T = 16384 tokens, d 2048, d_ff 8192, vocab 50304).

    python bench/gemm_bench.py [--case NAME] [--group mx] [--stalls]

Times each case with CUDA events after warm-up (median of --iters), prints
TFLOP/s and the fraction of the measured bf16 peak (MEASURED_PEAKS.json).
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from mtorus.ops import kernels as K  # noqa: E402


STALLS = False


def stalls(fn, n=5):
    """Shares of the MMA issuer's time spent waiting for operands / for a free accumulator,
    and of the producer's time waiting for a free stage (gemm_profile counters)."""
    from mtorus._ext import cuda

    torch.cuda.synchronize()
    cuda().gemm_profile(True)
    for _ in range(n):
        fn()
    torch.cuda.synchronize()
    p = cuda().gemm_profile_read()
    cuda().gemm_profile(False)
    if p[4] == 0:
        return None
    return {"mma_wait_operands": round(p[2] / p[4], 3), "mma_wait_accumulator": round(p[3] / p[4], 3),
            "mma_wait_shared_chunk": round(p[5] / p[4], 3),
            "producer_wait_free_stage": round(p[0] / max(1, p[1]), 3)}


def timeit(fn, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return ts[len(ts) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    ap.add_argument("--case", default=None, help="run only the named case (e.g. ffn1_fwd_fp8)")
    ap.add_argument("--group", default=None, choices=["mx"], help="run only the MXFP8 own-vs-library cases")
    ap.add_argument("--stalls", action="store_true",
                    help="also report, per case, where the CTA-pair kernel's MMA issuer waited (for loaded "
                         "operand stages vs for the epilogue to free an accumulator) over 5 extra launches")
    args = ap.parse_args()
    global STALLS
    STALLS = args.stalls
    peak = 1607.9
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        peak = json.load(open(p)).get("bf16_tflops", peak)
    T, d, F, V = 16384, 2048, 8192, 50304
    cases = [  # name, M, N, K, layout
        ("qkv_fwd", T, 3 * d, d, "tn"), ("out_fwd", T, d, d, "tn"), ("ffn1_fwd", T, F, d, "tn"),
        ("ffn2_fwd", T, d, F, "tn"), ("lm_fwd", T, V, d, "tn"),
        ("ffn1_dgrad", T, d, F, "dgrad"), ("ffn2_dgrad", T, F, d, "dgrad"), ("lm_dgrad", T, d, V, "dgrad"),
        ("ffn1_wgrad", F, d, T, "wgrad"), ("ffn2_wgrad", d, F, T, "wgrad"), ("qkv_wgrad", 3 * d, d, T, "wgrad"),
        ("lm_wgrad", V, d, T, "wgrad"), ("square8k", 8192, 8192, 8192, "tn"),
    ]
    rows = []
    from mtorus.ops import fp8 as F8

    fp8_cases = [("qkv_fwd_fp8", T, 3 * d, d, "tn"), ("ffn1_fwd_fp8", T, F, d, "tn"), ("ffn2_fwd_fp8", T, d, F, "tn"),
                 ("ffn2_dgrad_fp8", T, F, d, "dgrad"), ("ffn1_wgrad_fp8", F, d, T, "wgrad"),
                 ("square8k_fp8", 8192, 8192, 8192, "tn"),
                 # the same shapes with the epilogues the training step uses
                 ("ffn1_fwd_fp8_gelu8", T, F, d, "tn_gelu8"), ("ffn2_fwd_fp8_bias_res", T, d, F, "tn_res"),
                 ("ffn2_dgrad_fp8_dgelu", T, F, d, "dgrad_aux"), ("ffn1_wgrad_fp8_acc", F, d, T, "wgrad_acc")]
    one = torch.ones(1, device="cuda")
    if args.case:
        fp8_cases = [c for c in fp8_cases if c[0] == args.case]
        cases = [c for c in cases if c[0] == args.case]
    if args.group == "mx":
        fp8_cases, cases = [], []
    for name, M, N, Kd, lay in fp8_cases:
        A = (torch.randn(M, Kd, device="cuda") if not lay.startswith("wgrad") else
             torch.randn(Kd, M, device="cuda")).to(torch.float8_e4m3fn).view(torch.uint8)
        B = (torch.randn(N, Kd, device="cuda") if lay.startswith("tn") else
             torch.randn(Kd, N, device="cuda")).to(torch.float8_e4m3fn).view(torch.uint8)
        if lay == "tn":
            mine = lambda: F8.gemm_fp8(A, 0, B, 0, alpha=one)
            ref = lambda: torch._scaled_mm(A.view(torch.float8_e4m3fn), B.view(torch.float8_e4m3fn).t(), one, one,
                                           out_dtype=torch.bfloat16)
        elif lay == "tn_gelu8":
            pre = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            a8 = torch.empty(M, N, device="cuda", dtype=torch.uint8)
            bias = torch.zeros(N, device="cuda")
            amax = torch.zeros(1, device="cuda")
            mine = lambda: F8.gemm_fp8_gelu8(A, 0, B, 0, pre, a8, one, amax, 0, bias=bias, alpha=one, alpha2=one)
            ref = None
        elif lay == "tn_res":
            bias = torch.zeros(N, device="cuda")
            res = torch.randn(M, N, device="cuda").bfloat16()
            mine = lambda: F8.gemm_fp8(A, 0, B, 0, bias=bias, residual=res, alpha=one, alpha2=one)
            ref = None
        elif lay == "dgrad_aux":
            aux = torch.randn(M, N, device="cuda").bfloat16()
            mine = lambda: F8.gemm_fp8(A, 1, B, 0, b_mn=True, aux=aux, alpha=one, alpha2=one)
            ref = None
        elif lay == "wgrad_acc":
            out = torch.zeros(M, N, device="cuda")
            mine = lambda: F8.gemm_fp8(A, 1, B, 0, out=out, a_mn=True, b_mn=True, accumulate=True, alpha=one,
                                       alpha2=one)
            ref = None
        elif lay == "dgrad":
            mine = lambda: F8.gemm_fp8(A, 1, B, 0, b_mn=True, alpha=one)
            ref = None
        else:
            out = torch.empty(M, N, device="cuda")
            mine = lambda: F8.gemm_fp8(A, 1, B, 0, out=out, a_mn=True, b_mn=True, alpha=one)
            ref = None
        flops = 2.0 * M * N * Kd
        tm = timeit(mine, args.iters)
        tr = timeit(ref, args.iters) if ref is not None else float("nan")
        r = {"case": name, "M": M, "N": N, "K": Kd, "layout": lay, "mine_ms": round(tm, 4),
             "cublas_ms": round(tr, 4), "mine_tflops": round(flops / tm / 1e9, 1),
             "cublas_tflops": round(flops / tr / 1e9, 1) if tr == tr else None,
             "mine_frac_of_2x_measured_bf16_peak": round(flops / tm / 1e9 / (2 * peak), 3)}
        if STALLS:
            r["stalls"] = stalls(mine)
        rows.append(r)
        print(json.dumps(r), flush=True)
        del A, B
    # MXFP8 (1x32 UE8M0 block scales), K-major operands; cuBLAS through torch._scaled_mm with
    # the same scale bytes (its MX scale layout is the tcgen05 atom layout mx_quantize writes)
    from mtorus.ops import mxfp8 as MX

    E4, E5 = MX.E4M3, MX.E5M2
    bf, f32 = torch.bfloat16, torch.float32
    # (name, M, N, K, A format, B format, output dtype): forward E4M3 x E4M3; dgrad E5M2 gradient x
    # E4M3 weight (column codes); wgrad E5M2 gradient x E4M3 activation, fp32 out
    mx_cases = [("qkv_fwd_mx", T, 3 * d, d, E4, E4, bf), ("out_fwd_mx", T, d, d, E4, E4, bf),
                ("ffn1_fwd_mx", T, F, d, E4, E4, bf), ("ffn2_fwd_mx", T, d, F, E4, E4, bf),
                ("qkv_dgrad_mx", T, d, 3 * d, E5, E4, bf), ("out_dgrad_mx", T, d, d, E5, E4, bf),
                ("ffn1_dgrad_mx", T, d, F, E5, E4, bf), ("ffn2_dgrad_mx", T, F, d, E5, E4, bf),
                ("qkv_wgrad_mx", 3 * d, d, T, E5, E4, f32), ("out_wgrad_mx", d, d, T, E5, E4, f32),
                ("ffn1_wgrad_mx", F, d, T, E5, E4, f32), ("ffn2_wgrad_mx", d, F, T, E5, E4, f32),
                ("square8k_mx", 8192, 8192, 8192, E4, E4, bf)]
    if args.case:
        mx_cases = [c for c in mx_cases if c[0] == args.case]
    for name, M, N, Kd, fa, fb, odt in mx_cases:
        a = MX.mx_quantize(torch.randn(M, Kd, device="cuda").bfloat16(), fa)
        b = MX.mx_quantize(torch.randn(N, Kd, device="cuda").bfloat16(), fb)
        out = torch.empty(M, N, device="cuda", dtype=odt)
        out2 = torch.empty_like(out)
        mine = lambda: MX.gemm_mxfp8(a, b, out, impl="own")
        try:  # cuBLASLt's block-scaled kernel through the library route (torch._scaled_mm)
            ref = lambda: MX.gemm_mxfp8(a, b, out2, impl="library")
            ref()
        except (RuntimeError, AttributeError, TypeError) as e:
            print(f"[{name}] torch._scaled_mm MX path unavailable: {e}", file=sys.stderr)
            ref = None
        flops = 2.0 * M * N * Kd
        tm = timeit(mine, args.iters)
        tr = timeit(ref, args.iters) if ref is not None else float("nan")
        r = {"case": name, "M": M, "N": N, "K": Kd, "layout": "tn_mx", "formats": f"{'E4M3' if fa == E4 else 'E5M2'}"
             f" x {'E4M3' if fb == E4 else 'E5M2'} -> {'bf16' if odt == bf else 'fp32'}", "mine_ms": round(tm, 4),
             "cublas_ms": round(tr, 4) if tr == tr else None, "mine_tflops": round(flops / tm / 1e9, 1),
             "cublas_tflops": round(flops / tr / 1e9, 1) if tr == tr else None,
             "mine_frac_of_2x_measured_bf16_peak": round(flops / tm / 1e9 / (2 * peak), 3)}
        if STALLS:
            r["stalls"] = stalls(mine)
        rows.append(r)
        print(json.dumps(r), flush=True)
        del a, b, out, out2
    # the MXFP8 epilogues of the fused path: FFN1 forward (bias, GELU, pre-activation stored, GELU
    # quantised to row + column MX codes) and FFN2 dgrad (dGELU, E5M2 row + column codes, bias-gradient
    # column sums, no bf16 store), against the same GEMM followed by the separate quantiser
    epi_cases = [("ffn1_fwd_mx_gelu_mxout", T, F, d), ("ffn2_dgrad_mx_dgelu_mxout", T, F, d)]
    if args.case:
        epi_cases = [c for c in epi_cases if c[0] == args.case]
    if args.group == "mx":
        epi_cases = []
    for name, M, N, Kd in epi_cases:
        dgrad = "dgrad" in name
        a = MX.mx_quantize(torch.randn(M, Kd, device="cuda").bfloat16(), MX.E5M2 if dgrad else MX.E4M3)
        b = MX.mx_quantize((torch.randn(N, Kd, device="cuda") * 0.02).bfloat16())
        bias = torch.randn(N, device="cuda") * 0.1
        pre = torch.randn(M, N, device="cuda").bfloat16()
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        cs = torch.zeros(N, device="cuda")
        if dgrad:
            mine = lambda: MX.gemm_mxfp8_mx_out(a, b, MX.E5M2, aux=pre, colsum=cs, store_d=False)

            def unfused():
                d_ = MX.gemm_mxfp8(a, b, out, aux=pre)
                MX.mx_quantize_rc(d_, MX.E5M2, colsum=cs)
        else:
            mine = lambda: MX.gemm_mxfp8_mx_out(a, b, MX.E4M3, out, bias=bias, gelu=True)
            act = torch.empty_like(out)

            def unfused():
                MX.gemm_mxfp8(a, b, out, bias=bias, act=act)
                MX.mx_quantize_rc(act, MX.E4M3)
        flops = 2.0 * M * N * Kd
        tm = timeit(mine, args.iters)
        tu = timeit(unfused, args.iters)
        r = {"case": name, "M": M, "N": N, "K": Kd, "layout": "tn_mx", "formats": f"{'E4M3' if fa == E4 else 'E5M2'}"
             f" x {'E4M3' if fb == E4 else 'E5M2'} -> {'bf16' if odt == bf else 'fp32'}", "mine_ms": round(tm, 4),
             "unfused_ms": round(tu, 4), "mine_tflops": round(flops / tm / 1e9, 1)}
        if STALLS:
            r["stalls"] = stalls(mine)
        rows.append(r)
        print(json.dumps(r), flush=True)
        del a, b, out, pre
    for name, M, N, Kd, lay in cases:
        A = torch.randn(M, Kd, device="cuda").bfloat16() if lay != "wgrad" else torch.randn(Kd, M, device="cuda").bfloat16()
        if lay == "tn":
            B = torch.randn(N, Kd, device="cuda").bfloat16()
            mine = lambda: K.gemm(A, B)
            ref = lambda: torch.matmul(A, B.t())
        elif lay == "dgrad":
            B = torch.randn(Kd, N, device="cuda").bfloat16()
            mine = lambda: K.gemm(A, B, b_mn=True)
            ref = lambda: torch.matmul(A, B)
        else:
            B = torch.randn(Kd, N, device="cuda").bfloat16()
            out = torch.empty(M, N, device="cuda")
            mine = lambda: K.gemm(A, B, out=out, a_mn=True, b_mn=True)
            ref = lambda: torch.mm(A.t(), B, out_dtype=torch.float32)
        flops = 2.0 * M * N * Kd
        tm = timeit(mine, args.iters)
        tr = timeit(ref, args.iters)
        r = {"case": name, "M": M, "N": N, "K": Kd, "layout": lay, "mine_ms": round(tm, 4),
             "cublas_ms": round(tr, 4), "mine_tflops": round(flops / tm / 1e9, 1),
             "cublas_tflops": round(flops / tr / 1e9, 1), "mine_frac_of_measured_peak": round(flops / tm / 1e9 / peak, 3)}
        if STALLS:
            r["stalls"] = stalls(mine)
        rows.append(r)
        print(json.dumps(r), flush=True)
        del A, B
    if args.json:
        json.dump(rows, open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
