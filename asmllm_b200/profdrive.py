"""Small, bounded workload for profiling the matvec kernels under ncu.

    python -m asmllm_b200.profdrive [--fmt q4|q8] [--mode fused|image] [--launches N]
                                    [--path tma|ldg] [--layout planes|packed]
                                    [--chain dependent|independent] MxK [MxK ...]
    python -m asmllm_b200.profdrive --decode N [--layers L] [--warm W]
    python -m asmllm_b200.profdrive --gemm N [--launches L] MxK [MxK ...]

For each shape it builds one weight matrix on cuda:0 (random seeded quants,
fp16 scales, declared static like model weights), then runs N matvecs
(default 2) on torch's current stream.  Device memory stays at the size of
the largest matrix, so an ncu capture of it ends quickly.  --layout packed
streams packed rows (asm_pack_rows_async) as the bench's headline does;
--chain independent launches with ASM_MV_INDEPENDENT.

--gemm N runs the tensor-core batched product (N tokens, Q4_0) L times per
shape, from one activation image of N rows.

--decode N builds the random-init Llama-7B-shaped decoder (L layers, default
32: 4.2 GB on the device), runs W greedy steps through CUDA graphs (default
24, to fill the KV cache), then N eager steps: 5 * L + 1 launches each.
"""
from __future__ import annotations

import argparse

import torch

from . import ops
from .native import FMT_Q4_0, FMT_Q8_0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("shapes", nargs="*")
    ap.add_argument("--decode", type=int, default=0)
    ap.add_argument("--gemm", type=int, default=0)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--warm", type=int, default=24)
    ap.add_argument("--fmt", choices=["q4", "q8"], default="q4")
    ap.add_argument("--mode", choices=["fused", "image"], default="fused")
    ap.add_argument("--launches", type=int, default=2)
    ap.add_argument("--path", choices=["tma", "ldg"], default="tma")
    ap.add_argument("--layout", choices=["planes", "packed"], default="planes")
    ap.add_argument("--chain", choices=["dependent", "independent"], default="dependent")
    args = ap.parse_args()
    if args.decode:
        from dataclasses import replace

        from . import decode as D

        dec = D.LlamaDecoder(replace(D.LLAMA_7B, n_layers=args.layers), ctx=512, seed=0)
        dec.generate(list(range(1, 17)), args.warm)
        dec.step(args.decode)
        torch.cuda.synchronize()
        err = ops.device_error()
        print(f"profdrive: decode {args.layers} layers, {args.warm} graph steps + {args.decode} eager steps "
              f"({dec.launches_per_step} launches each), position {dec.position()}, device error word {err}")
        dec.close()
        raise SystemExit(1 if err else 0)
    fmt = FMT_Q4_0 if args.fmt == "q4" else FMT_Q8_0
    if args.gemm:
        dev = torch.device("cuda", 0)
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        for shape in args.shapes:
            M, K = (int(v) for v in shape.lower().split("x"))
            qs = torch.randint(0, 256, (M, K // 32, 16), dtype=torch.uint8, device=dev, generator=gen)
            d = torch.randn((M, K // 32), device=dev, generator=gen).abs_().mul_(0.02).half()
            img = ops.act_image_dev(torch.randn((args.gemm, K), device=dev, generator=gen))
            out = torch.empty((args.gemm, M), device=dev)
            for _ in range(args.launches):
                ops.gemm_image(FMT_Q4_0, qs, d, img, K, out=out)
            torch.cuda.synchronize()
        err = ops.device_error()
        print(f"profdrive: gemm N={args.gemm}, {len(args.shapes)} shape(s) x {args.launches} launch(es), "
              f"device error word {err}")
        raise SystemExit(1 if err else 0)
    ops.set_option("tma", 1 if args.path == "tma" else 0)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    for shape in args.shapes:
        M, K = (int(v) for v in shape.lower().split("x"))
        if fmt == FMT_Q4_0:
            qs = torch.randint(0, 256, (M, K // 32, 16), dtype=torch.uint8, device=dev, generator=gen)
        else:
            qs = torch.randint(-127, 128, (M, K // 32, 32), dtype=torch.int8, device=dev, generator=gen)
        d = torch.randn((M, K // 32), device=dev, generator=gen).abs_().mul_(0.02).half()
        x = torch.randn(K, device=dev, generator=gen)
        y = torch.empty(M, device=dev)
        torch.cuda.synchronize()
        indep = args.chain == "independent"
        if args.layout == "packed":
            w = ops.pack_rows(fmt, qs, d)
            del qs, d
            qs, d = w, None
            ops.mark_static(w)
        else:
            ops.mark_static(qs, d)
        for _ in range(args.launches):
            if args.layout == "packed":
                ops.matvec_packed(fmt, qs, x, out=y, independent=indep)
            elif args.mode == "fused":
                ops.matvec(fmt, qs, d, x, out=y, independent=indep)
            else:
                img = ops.act_image_dev(x)
                ops.matvec_image(fmt, qs, d, img, K, out=y)
        torch.cuda.synchronize()
        ops.unmark_static(*([qs] if d is None else [qs, d]))
        del qs, d
    err = ops.device_error()
    print(f"profdrive: {len(args.shapes)} shape(s) x {args.launches} launch(es), device error word {err}")
    if err:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
