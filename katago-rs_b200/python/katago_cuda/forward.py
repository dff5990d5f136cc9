"""Run forward passes of a seeded benchmark net at a fixed batch, reading all outputs back each pass.

The shape of the reference's bench harness (crates/katago-nn-burn/examples/bench.rs:20-62): synthetic inputs,
warm-up, then timed passes that read every output row back. Used for quick runs and as the command that profiler
captures wrap:

    python -m katago_cuda.forward --net b18c384nbt --batch 256 --iters 2
    KATAGO_CUDA_NO_GRAPHS=1 ncu ... python -m katago_cuda.forward ...
"""

from __future__ import annotations

import argparse
import time

import numpy as np

from . import api, inputs, netgen


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--net", default="b18c384nbt", choices=sorted(netgen.NETS))
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--precision", default="auto", choices=["auto", "f32", "f16", "bf16"])
    ap.add_argument("--gpu", type=int, default=0)
    args = ap.parse_args(argv)
    prec = {"auto": api.PRECISION_AUTO, "f32": api.PRECISION_F32, "f16": api.PRECISION_F16,
            "bf16": api.PRECISION_BF16}[args.precision]
    model = api.Model(netgen.net_bytes(args.net))
    handle = api.Handle(api.Context(model, [args.gpu], prec), args.batch, args.gpu)
    d = model.desc
    spatial, glob, meta, _ = inputs.synthetic_inputs(args.batch, 0xB200, (19,), d.num_input_channels,
                                                     d.num_input_global_channels, d.num_input_meta_channels)
    t0 = time.perf_counter()
    checksum = 0.0
    for _ in range(args.iters):
        out = handle.forward(spatial, glob, meta)
        checksum += float(np.sum(out["value"]))
    dt = time.perf_counter() - t0
    print(f"{args.net} batch {args.batch}: {args.iters} passes in {dt * 1e3:.1f} ms "
          f"({args.iters * args.batch / dt:.0f} evals/s incl. first-pass setup), value checksum {checksum:.6f}")


if __name__ == "__main__":
    main()
