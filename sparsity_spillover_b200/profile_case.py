"""Run a few launches of one kernel on a benchmark config, for profilers (ncu).

    python -m sparsity_spillover_b200.profile_case --case mlp  [--tokens 32768] [--iters 3]
    python -m sparsity_spillover_b200.profile_case --case tile [--p 0.1] [--skip fine]
    python -m sparsity_spillover_b200.profile_case --case head [--d 128] [--frac 0.1] [--kappa K]
    python -m sparsity_spillover_b200.profile_case --case joint [--tokens 32768]
    python -m sparsity_spillover_b200.profile_case --case corner [--tokens 32768] [--p 0.01] [--skip compact_fine]

* ``mlp``  one cfg1 layer (d=512, F=2048, fp16, one-sided gate at 10% density):
           up_gate then down_sparse with the residual, ``iters`` times.
* ``tile`` cfg2: a tile-structured bf16 h (64x64 tiles live with probability p),
           its bitmap, and the tile-skipping down_sparse (d=512, F=2048) in the
           ``--skip`` mode (coarse: 256-token pair tiles, fine: 128-token tiles).
* ``head`` cfg4: the N-gated vocabulary head on Zipf-chosen 128-column tiles, or with
           ``--kappa`` the K-gated head (16x16 corner certificates of an fp32 N(0,1) input).
* ``joint`` the joint consumer on a cfg1 layer: up_gate (identity, then gated) once,
           then the joint kernel ``iters`` times (h at 10% density, z ~ N(0,1)).
* ``corner`` h with the reference's corner-tile structure (8-token x 16-feature tiles kept
           with probability p, fp16, F=2048) through the down projection (d=512) in the
           ``--skip`` mode (compact modes read the 16x16 bitmap).

Inputs are seeded synthetic tensors; device memory stays well under 1 GB.
"""
from __future__ import annotations

import argparse

import torch

from . import ops, workloads


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--case", choices=["mlp", "tile", "head", "joint", "corner"], default="mlp")
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--p", type=float, default=0.1)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--frac", type=float, default=0.1)
    ap.add_argument("--skip", choices=["coarse", "fine", "compact", "compact_fine"], default="coarse")
    ap.add_argument("--kappa", type=float, default=None, help="head: K gate with this threshold")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    with torch.inference_mode():
        if args.case in ("mlp", "joint"):
            cfg = workloads.CONFIGS["cfg1"]
            layer = workloads.make_weights(cfg, dev)[0]
            x = workloads.make_input(cfg, dev, tokens=args.tokens)
            z = torch.empty(args.tokens, cfg.F, dtype=cfg.dtype, device=dev)
            ops.up_gate(x, layer.w_in, layer.b_in, {"operator": "identity"}, z_out=z)
            gate = {"operator": "one_sided_threshold", "kappa": workloads.quantile_threshold(z, 0.1)}
            del z
            h = torch.empty(args.tokens, cfg.F, dtype=cfg.dtype, device=dev)
            bits = torch.empty(ops.tile_bits_size(args.tokens, cfg.F), dtype=torch.int32, device=dev)
            y = torch.empty_like(x)
            if args.case == "joint":
                ops.up_gate(x, layer.w_in, layer.b_in, gate, h=h, bits=bits)
                g = torch.Generator(device=dev).manual_seed(77)
                z = torch.randn(args.tokens, cfg.d, generator=g, device=dev).to(cfg.dtype)
                wo = (torch.randn(cfg.d, cfg.d, generator=g, device=dev) * 0.02).to(cfg.dtype)
                bo = (torch.randn(cfg.d, generator=g, device=dev) * 0.02).to(cfg.dtype)
            for _ in range(args.iters):
                if args.case == "joint":
                    ops.joint(h, bits, z, layer.w_out, layer.b_out, wo, bo, x, out=y)
                    continue
                ops.up_gate(x, layer.w_in, layer.b_in, gate, h=h, bits=bits)
                ops.down_sparse(h, bits, layer.w_out, layer.b_out, x, y=y)
        elif args.case == "corner":
            h, _ = workloads.corner_tile_h(args.tokens, 2048, args.p, seed=3, device=dev)
            w = (torch.randn(512, 2048, device=dev) * 0.02).half()
            compact = args.skip.startswith("compact")
            bits = ops.tile_bits16_from_h(h) if compact else ops.tile_bits_from_h(h)
            y = torch.empty(args.tokens, 512, dtype=torch.float16, device=dev)
            for _ in range(args.iters):
                ops.down_sparse(h, bits, w, None, skip=args.skip, y=y)
        elif args.case == "tile":
            h, _ = workloads.tile_structured_h(args.tokens, 2048, args.p, seed=3, device=dev)
            w = (torch.randn(512, 2048, device=dev) * 0.02).bfloat16()
            bits = ops.tile_bits_from_h(h)
            y = torch.empty(args.tokens, 512, dtype=torch.bfloat16, device=dev)
            for _ in range(args.iters):
                ops.tile_bits_from_h(h, bits)
                ops.down_sparse(h, bits, w, None, skip=args.skip, y=y)
        else:
            x, w = workloads.head_inputs(args.tokens, args.d, seed=4, device=dev)
            logits = torch.empty(args.tokens, workloads.VOCAB, dtype=torch.float16, device=dev)
            if args.kappa is not None:
                xf = torch.randn(args.tokens, args.d, generator=torch.Generator(device=dev).manual_seed(68), device=dev)
                xh, support = ops.head_prepare(xf, args.kappa, torch.float16)
                for _ in range(args.iters):
                    ops.head_sparse(xh, w, support=support, logits=logits)
            else:
                tiles = torch.from_numpy(workloads.zipf_active_tiles(workloads.VOCAB // 128, args.frac, 5)).to(dev)
                for _ in range(args.iters):
                    ops.head_sparse(x, w, active_tiles=tiles, logits=logits)
        torch.cuda.synchronize(dev)
    print(f"profile_case {args.case}: ok, device status {ops.device_status(0)}")


if __name__ == "__main__":
    main()
