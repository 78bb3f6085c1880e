"""Runs one fused model kernel on GPT-2-small training shapes (8 x 1024 rows),
for ncu captures and CUDA-event timing of the kernel alone.

    python benchmarks/ops_kernels.py --kernel ln_bwd --iters 20 [--graph]
Kernels: ln_fwd, ln_bwd, cross_entropy, adamw, gelu_bwd (GELU backward + bias
gradient of the MLP), gemm_gelu (the tcgen05 GEMM of
the MLP's first layer with its bias + GELU epilogue, M = rows, N = 3072,
K = 768; reported in TFLOP/s) and gemm_gelu_ref (cuBLAS addmm + GELU on the
same shapes, for comparison).
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="ln_bwd")
    ap.add_argument("--rows", type=int, default=8 * 1024)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--persistent", action="store_true",
                    help="gemm_gelu: one CTA per SM with two TMEM accumulators")
    ap.add_argument("--k", type=int, default=768, help="gemm_gelu: inner dimension")
    ap.add_argument("--no-gelu", action="store_true", help="gemm_gelu: bias only (pre)")
    ap.add_argument("--pair", action="store_true",
                    help="gemm_gelu: persistent CTA pairs (cta_group::2, 256 x 256 tiles)")
    ap.add_argument("--graph", action="store_true",
                    help="time the launches as one CUDA-graph replay (no host launch cost)")
    args = ap.parse_args()
    import tiny_nccl_b200 as tn

    ops = tn.load().ops
    rows, C, V = args.rows, 768, 50257
    dev = "cuda"
    torch.manual_seed(0)
    if args.kernel in ("ln_fwd", "ln_bwd"):
        # Three input sets used in turn: consecutive launches do not find
        # each other's data in L2 (8192 rows take about 100 MB per launch).
        sets = []
        for _ in range(3):
            x = torch.randn(rows, C, device=dev)
            d = torch.randn(rows, C, device=dev).to(torch.bfloat16)
            w = torch.ones(C, device=dev)
            b = torch.zeros(C, device=dev)
            xo, y, mean, rstd = ops.ln_fwd(x, d, w, b, 1e-5)
            gy = torch.randn(rows, C, device=dev).to(torch.bfloat16)
            gr = torch.randn(rows, C, device=dev)
            sets.append((x, d, w, b, xo, mean, rstd, gy, gr))
        turn = [0]

        def next_set():
            turn[0] = (turn[0] + 1) % len(sets)
            return sets[turn[0]]
        if args.kernel == "ln_fwd":
            def fn():
                x, d, w, b = next_set()[:4]
                return ops.ln_fwd(x, d, w, b, 1e-5)
            nbytes = rows * C * (4 + 2 + 4 + 2)
        else:
            def fn():
                _, _, w, _, xo, mean, rstd, gy, gr = next_set()
                return ops.ln_bwd(gy, gr, xo, w, mean, rstd, True)
            nbytes = rows * C * (2 + 4 + 4 + 4 + 2)
    elif args.kernel == "cross_entropy":
        Vp = 50304
        logits = torch.randn(rows, Vp, device=dev).to(torch.bfloat16)
        tgt = torch.randint(0, V, (rows,), device=dev)
        fn = lambda: ops.cross_entropy_fwd_bwd(logits, tgt, rows, V)  # noqa: E731
        nbytes = rows * Vp * 2 * 2
    elif args.kernel == "adamw":
        from tiny_nccl_b200.models import GPT2, GPT2Config
        m = GPT2(GPT2Config()).to(dev)
        ps = list(m.parameters())
        gs = [torch.randn_like(p) for p in ps]
        ms = [torch.zeros_like(p) for p in ps]
        vs = [torch.zeros_like(p) for p in ps]
        wd = [0.1] * len(ps)
        step = [0]

        def fn():
            step[0] += 1
            ops.adamw(ps, gs, ms, vs, wd, 6e-4, 0.9, 0.95, 1e-8, step[0], 1.0)
        nbytes = sum(p.numel() for p in ps) * 4 * 7
    elif args.kernel == "gelu_bwd":
        # The MLP's GELU backward fused with its bias gradient, [rows, 3072].
        gy = torch.randn(rows, 4 * C, device=dev).to(torch.bfloat16)
        pre = (2 * torch.randn(rows, 4 * C, device=dev)).to(torch.bfloat16)
        fn = lambda: ops.gelu_bwd_bias(gy, pre)  # noqa: E731
        nbytes = rows * 4 * C * 2 * 3
    elif args.kernel in ("gemm_gelu", "gemm_gelu_ref"):
        x = (torch.randn(rows, args.k, device=dev) * 0.5).to(torch.bfloat16)
        w = (torch.randn(4 * C, args.k, device=dev) * 0.02).to(torch.bfloat16)
        b = (torch.randn(4 * C, device=dev) * 0.02).to(torch.bfloat16)
        if args.kernel == "gemm_gelu":
            variant = 2 if args.pair else 1 if args.persistent else 0
            fn = lambda: ops.gemm_bias_act(x, w, b, not args.no_gelu, variant)  # noqa: E731
        else:
            fn = lambda: torch.nn.functional.gelu(torch.addmm(b, x, w.t()),  # noqa: E731
                                                  approximate="tanh")
        flops = 2.0 * rows * 4 * C * args.k
        nbytes = None
    else:
        raise SystemExit(f"unknown kernel {args.kernel}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    run = lambda: [fn() for _ in range(args.iters)]  # noqa: E731
    if args.graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            run()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run()
        graph.replay()
        torch.cuda.synchronize()
        run = graph.replay
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    if nbytes is None:
        print(f"{args.kernel}: {ms * 1e3:.1f} us/launch, {flops / ms / 1e9:.0f} TFLOP/s")
        if args.kernel == "gemm_gelu":
            assert ops.tcgen05_status(True) == 0, "a tcgen05 GEMM wait timed out"
    else:
        print(f"{args.kernel}: {ms * 1e3:.1f} us/launch, {nbytes / ms / 1e6:.0f} GB/s algorithmic")


if __name__ == "__main__":
    main()
