"""Static-cache decode ops without a GPU: operator registration, fake
(tracing) implementations and the call-boundary checks."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from gemma4_fa4_kernels_b200 import UnsupportedB200Path
from gemma4_fa4_kernels_b200 import decode_ops as d


def _global_args(device="cpu", capacity=64):
    bf = dict(dtype=torch.bfloat16, device=device)
    return [torch.zeros(1, 1, d.HIDDEN_SIZE, **bf), torch.zeros(1, 1, 512, **bf),
            torch.zeros(1, 1, 512, **bf), torch.full((1, 1), 5, dtype=torch.int64, device=device),
            torch.zeros(1, 4, capacity, 512, **bf), torch.zeros(1, 4, capacity, 512, **bf),
            torch.tensor(5, dtype=torch.int64, device=device),
            torch.zeros(32 * 512, d.HIDDEN_SIZE, **bf), torch.zeros(4 * 512, d.HIDDEN_SIZE, **bf),
            torch.zeros(d.HIDDEN_SIZE, 32 * 512, **bf), torch.zeros(512, **bf),
            torch.zeros(512, **bf)]


def _local_args(device="cpu"):
    bf = dict(dtype=torch.bfloat16, device=device)
    return [torch.zeros(1, 1, d.HIDDEN_SIZE, **bf), torch.zeros(1, 1, 256, **bf),
            torch.zeros(1, 1, 256, **bf), torch.full((1, 1), 5, dtype=torch.int64, device=device),
            torch.zeros(1, 16, 1024, 256, **bf), torch.zeros(1, 16, 1024, 256, **bf),
            torch.tensor(5, dtype=torch.int64, device=device),
            torch.zeros(32 * 256, d.HIDDEN_SIZE, **bf), torch.zeros(16 * 256, d.HIDDEN_SIZE, **bf),
            torch.zeros(16 * 256, d.HIDDEN_SIZE, **bf), torch.zeros(d.HIDDEN_SIZE, 32 * 256, **bf),
            torch.zeros(256, **bf), torch.zeros(256, **bf)]


def test_ops_are_registered_under_the_b200_namespace():
    assert hasattr(torch.ops.gemma4_fa4_b200, "global_static_cache_decode_fwd")
    assert hasattr(torch.ops.gemma4_fa4_b200, "local_static_cache_decode_fwd")
    schema = str(torch.ops.gemma4_fa4_b200.global_static_cache_decode_fwd.default._schema)
    assert "Tensor(a4!) cache_k" in schema and "Tensor(a6!) cache_length" in schema
    schema = str(torch.ops.gemma4_fa4_b200.local_static_cache_decode_fwd.default._schema)
    assert "cache_k" in schema and "Tensor cache_length" in schema  # read only


@pytest.mark.parametrize("op,make", [
    (torch.ops.gemma4_fa4_b200.global_static_cache_decode_fwd, _global_args),
    (torch.ops.gemma4_fa4_b200.local_static_cache_decode_fwd, _local_args),
])
def test_fake_implementations_describe_fresh_outputs(op, make):
    with FakeTensorMode():
        out, lse = op(*make())
    assert out.shape == (1, 1, d.HIDDEN_SIZE) and out.dtype == torch.bfloat16
    assert lse.shape == (1, 32, 1) and lse.dtype == torch.float32


def test_call_boundary_requires_no_grad_mode():
    args = _global_args()
    with torch.enable_grad(), pytest.raises(UnsupportedB200Path, match="no-grad"):
        d.global_static_cache_decode_fwd(*args)
    args = _local_args()
    args[0].requires_grad_(True)
    with torch.no_grad(), pytest.raises(UnsupportedB200Path, match="requires_grad"):
        d.local_static_cache_decode_fwd(*args)


def test_host_tensors_are_refused_before_any_work():
    with torch.no_grad(), pytest.raises(UnsupportedB200Path, match="CUDA device"):
        d.global_static_cache_decode_fwd(*_global_args())
    with torch.no_grad(), pytest.raises(UnsupportedB200Path, match="CUDA device"):
        d.local_static_cache_decode_fwd(*_local_args())
