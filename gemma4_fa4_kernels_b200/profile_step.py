"""Run a few forward+backward steps of one benchmark configuration, for profilers.

    python -m gemma4_fa4_kernels_b200.profile_step --config c1 --steps 1

Configs: c0 (local d256 W1024, S=2048, 32Q/16KV) and c1 (global d512 causal,
S=4096, 32Q/4KV), B=1, BF16, inputs as in bench.py; decode (one query token
against a 32768-token global d512 32Q/4KV static cache, forward only); prep
(the fused preparation of the c1 layer's Q rows, 4096 x 32 x 512: forward,
then backward with the norm-scale gradient).  Inputs exceed the 126 MB L2 for
c1, decode and prep.  Prints nothing but the per-step wall time; meant to be
wrapped by ncu with -k/-c filters.
"""

from __future__ import annotations

import argparse
import time

import torch

from . import ops

CONFIGS = {
    "c0": dict(seq=2048, hq=32, hkv=16, d=256, window=1024),
    "c1": dict(seq=4096, hq=32, hkv=4, d=512, window=0),
    "decode": dict(seq=32768, hq=32, hkv=4, d=512, window=0),
    "prep": dict(seq=4096, hq=32, hkv=4, d=512, window=0),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c1")
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--seq", type=int, default=None, help="override the sequence length")
    ap.add_argument("--fwd", choices=("auto", "single"), default="auto",
                    help="forward algorithm (auto: two-pass for d512 when the scratch fits)")
    ap.add_argument("--bwd", choices=("auto", "recompute"), default="auto",
                    help="backward algorithm (auto: materialised P/dS when the scratch fits)")
    args = ap.parse_args()
    c = dict(CONFIGS[args.config])
    if args.seq:
        c["seq"] = args.seq
    g = torch.Generator().manual_seed(0)
    dev = torch.device("cuda", 0)

    def rms(x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    s, hq, hkv, d = c["seq"], c["hq"], c["hkv"], c["d"]
    if args.config == "decode":
        # static cache backings (B, H, capacity, D), read through (B, S, H, D) views
        kc = rms(torch.randn(1, hkv, s, d, generator=g)).to(torch.bfloat16).to(dev)
        vc = rms(torch.randn(1, hkv, s, d, generator=g)).to(torch.bfloat16).to(dev)
        q = rms(torch.randn(1, 1, hq, d, generator=g)).to(torch.bfloat16).to(dev)
        for _ in range(args.steps):
            t0 = time.perf_counter()
            ops.attn_fwd(q, kc.transpose(1, 2), vc.transpose(1, 2), window=c["window"])
            torch.cuda.synchronize()
            print(f"step {time.perf_counter() - t0:.4f} s", flush=True)
        return
    if args.config == "prep":
        from .prep import prep_bwd, prep_fwd

        x = torch.randn(1, s, hq, d, generator=g).to(torch.bfloat16).to(dev)
        gr = torch.randn(1, s, hq, d, generator=g).to(torch.bfloat16).to(dev)
        w = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16).to(dev)
        ang = torch.rand(1, s, d // 2, generator=g, dtype=torch.float64) * 6.0
        ang = torch.cat((ang, ang), dim=-1)
        cos, sin = ang.cos().to(torch.bfloat16).to(dev), ang.sin().to(torch.bfloat16).to(dev)
        for _ in range(args.steps):
            t0 = time.perf_counter()
            prep_fwd(x, w, cos, sin, d)
            prep_bwd(x, w, cos, sin, d, gr, None)
            torch.cuda.synchronize()
            print(f"step {time.perf_counter() - t0:.4f} s", flush=True)
        return
    q = rms(torch.randn(1, s, hq, d, generator=g)).to(torch.bfloat16).to(dev)
    k = rms(torch.randn(1, s, hkv, d, generator=g)).to(torch.bfloat16).to(dev)
    v = rms(torch.randn(1, s, hkv, d, generator=g)).to(torch.bfloat16).to(dev)
    do = torch.randn(1, s, hq, d, generator=g).to(torch.bfloat16).to(dev)
    for _ in range(args.steps):
        t0 = time.perf_counter()
        out, lse = ops.attn_fwd(q, k, v, window=c["window"], algorithm=args.fwd)
        ops.attn_bwd(q, k, v, out, lse, do, window=c["window"], algorithm=args.bwd)
        torch.cuda.synchronize()
        print(f"step {time.perf_counter() - t0:.4f} s", flush=True)


if __name__ == "__main__":
    main()
