#!/usr/bin/env python
"""MXFP8 quantisers of the block-scaled training recipe on the GPT-1B shapes.

    python bench/mx_quant_bench.py [--case NAME]

Row- plus column-wise MXFP8 of a [T, C] bf16 tensor (``mx_quantize_rc``: the
operands that contract over C and over T, with the bias-gradient column sums of
the same pass), the same with GELU applied to the tile (the FFN1 output) or the
tile times GELU' of the pre-activation (the FFN2 dgrad), and LayerNorm straight to
MXFP8 (``mx_layernorm_rc``).  Bytes = 2 read + 2 written per element (+ scales, + 2
read for the dGELU pre-activation); CUDA events, median of 20 launches on inputs
larger than L2; roofline = measured HBM copy bandwidth (MEASURED_PEAKS.json).
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402


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
    import argparse

    from mtorus.ops import mxfp8 as MX

    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="run only the named case")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()

    hbm = 6551.0
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(p):
        hbm = json.load(open(p)).get("hbm_gbs", hbm)
    T = 16384
    for name, C, colsum, act in (("rc_act_16384x8192", 8192, True, None), ("rc_qkvgrad_16384x6144", 6144, True, None),
                                 ("rc_out_16384x2048", 2048, True, None), ("rc_weight_8192x2048", 2048, False, None),
                                 ("rc_gelu_16384x8192", 8192, False, "gelu"),
                                 ("rc_dgelu_16384x8192", 8192, True, "dgelu")):
        if args.case and name != args.case:
            continue
        R = 8192 if name.startswith("rc_weight") else T
        x = torch.randn(R, C, device="cuda").bfloat16()
        aux = torch.randn(R, C, device="cuda").bfloat16() if act == "dgelu" else None
        cs = torch.zeros(C, device="cuda") if colsum else None
        ms = timeit(lambda: MX.mx_quantize_rc(x, MX.E5M2, colsum=cs, act=act, aux=aux), args.iters)
        nbytes = R * C * (6 if act == "dgelu" else 4) + 2 * R * C // 32
        print(json.dumps({"case": name, "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
                          "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3)}), flush=True)
    if args.case and args.case != "layernorm_mx_16384x2048":
        return
    x = torch.randn(T, 2048, device="cuda").bfloat16()
    g, b = torch.rand(2048, device="cuda") + 0.5, torch.randn(2048, device="cuda") * 0.1
    ms = timeit(lambda: MX.mx_layernorm_rc(x, g, b), args.iters)
    nbytes = T * 2048 * 4 + T * 2048 * 2  # x read twice (statistics, then the tiles), codes written both ways
    print(json.dumps({"case": "layernorm_mx_16384x2048", "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
                      "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm, 3)}), flush=True)


if __name__ == "__main__":
    main()
