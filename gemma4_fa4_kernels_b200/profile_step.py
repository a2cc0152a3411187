"""Run a few forward+backward steps of one benchmark configuration, for profilers.

    python -m gemma4_fa4_kernels_b200.profile_step --config c1 --steps 1

Configs: c0 (local d256 W1024, S=2048, 32Q/16KV) and c1 (global d512 causal,
S=4096, 32Q/4KV), B=1, BF16, inputs as in bench.py; c2 (local d256 W1024,
B=2, S=8192, six 256-token images per sequence) and c3l (the packed
T=131072 mix of documents and images, local d256 layer), whose metadata comes
from bench.py's generators (run from the repository root); decode (one query token
against a 32768-token global d512 32Q/4KV static cache, forward only) and
decode_local (one token against a 1024-token local d256 32Q/16KV cache); prep
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
    "decode_local": dict(seq=1024, hq=32, hkv=16, d=256, window=1024),
    "prep": dict(seq=4096, hq=32, hkv=4, d=512, window=0),
    "c2": dict(seq=8192, hq=32, hkv=16, d=256, window=1024),
    "c3l": dict(seq=131072, hq=32, hkv=16, d=256, window=1024),
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
    if args.config in ("decode", "decode_local"):
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
    kw = dict(window=c["window"])
    lead = (1, s)
    if args.config in ("c2", "c3l"):
        import bench  # the repository root's workload generators

        if args.config == "c2":
            lead = (2, s)
            kw["vision_ids"] = torch.from_numpy(bench.c2_metadata(s=s)).to(dev)
        else:
            lens, cu, doc, vis = bench.c3_packing(total=s)
            lead = (s,)
            cu_t = torch.from_numpy(cu).to(dev)
            kw.update(cu_seqlens_q=cu_t, cu_seqlens_k=cu_t, max_seqlen_q=int(max(lens)),
                      max_seqlen_k=int(max(lens)), vision_ids=torch.from_numpy(vis).to(dev),
                      document_ids=torch.from_numpy(doc).to(dev))
    q = rms(torch.randn(*lead, hq, d, generator=g)).to(torch.bfloat16).to(dev)
    k = rms(torch.randn(*lead, hkv, d, generator=g)).to(torch.bfloat16).to(dev)
    v = rms(torch.randn(*lead, hkv, d, generator=g)).to(torch.bfloat16).to(dev)
    do = torch.randn(*lead, hq, d, generator=g).to(torch.bfloat16).to(dev)
    for _ in range(args.steps):
        t0 = time.perf_counter()
        out, lse = ops.attn_fwd(q, k, v, algorithm=args.fwd, **kw)
        ops.attn_bwd(q, k, v, out, lse, do, algorithm=args.bwd, **kw)
        torch.cuda.synchronize()
        print(f"step {time.perf_counter() - t0:.4f} s", flush=True)


if __name__ == "__main__":
    main()
