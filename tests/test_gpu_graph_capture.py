"""CUDA-graph capture of whole forward + backward steps.

Fixed-layout calls whose plan fits one band enqueue no host synchronisation,
so a training step can be captured once and replayed; the replay must equal the
eager calls bit for bit (same kernels, same workspace plan).  Captured here:
a local d256 step (window, GQA 2) and a global d512 step (two-pass forward,
materialised backward), each against fresh eager results after the inputs
change in place between replays."""

import pytest
import torch

from parity_util import make_inputs

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import ops  # noqa: E402


@pytest.mark.parametrize("d,heads,window,s", [(256, (8, 4), 1024, 1500), (512, (8, 1), 0, 1100)],
                         ids=["local_d256", "global_d512"])
def test_step_replays_bit_identically(d, heads, window, s):
    hq, hkv = heads
    q, k, v, do = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=31)

    def step():
        out, lse = ops.attn_fwd(q, k, v, window=window)
        return (out, lse) + tuple(ops.attn_bwd(q, k, v, out, lse, do, window=window))

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up outside the capture (allocator pools, attributes)
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step()
    for seed in (32, 33):
        q2, k2, v2, do2 = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=seed)
        for dst, src in ((q, q2), (k, k2), (v, v2), (do, do2)):
            dst.copy_(src)
        graph.replay()
        eager = step()
        torch.cuda.synchronize()
        for name, a, b in zip(("out", "lse", "dq", "dk", "dv"), captured, eager):
            assert torch.equal(a, b), f"{name} differs between replay and eager"
