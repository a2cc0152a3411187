"""Opaque prepared and whole-layer ops without a GPU: registration under the
B200 namespace, fake (tracing) implementations and the call-boundary checks."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from gemma4_fa4_kernels_b200 import UnsupportedB200Path
from gemma4_fa4_kernels_b200 import layer_ops as L

H = L.HIDDEN_SIZE
BF = dict(dtype=torch.bfloat16)


def _layer_args(kind, s=8):
    hq, hkv, d = L.LOCAL_GEOMETRY if kind == "local" else L.GLOBAL_GEOMETRY
    args = [torch.zeros(1, s, H, **BF), torch.zeros(1, s, d, **BF), torch.zeros(1, s, d, **BF),
            torch.arange(s).unsqueeze(0), torch.zeros(1, s, dtype=torch.int64),
            torch.zeros(hq * d, H, **BF), torch.zeros(hkv * d, H, **BF)]
    if kind == "local":
        args.append(torch.zeros(hkv * d, H, **BF))
    args += [torch.zeros(H, hq * d, **BF), torch.zeros(d, **BF), torch.zeros(d, **BF)]
    return args


def _prepared_args(kind, s=8):
    hq, hkv, d = L.LOCAL_GEOMETRY if kind == "local" else L.GLOBAL_GEOMETRY
    return [torch.zeros(1, hq, s, d, **BF), torch.zeros(1, hkv, s, d, **BF),
            torch.zeros(1, hkv, s, d, **BF), torch.arange(s).unsqueeze(0),
            torch.zeros(1, s, dtype=torch.int64)]


def test_ops_are_registered_under_the_b200_namespace():
    for name in ("local_fwd", "global_fwd", "local_layer_fwd", "global_layer_fwd"):
        assert hasattr(torch.ops.gemma4_fa4_b200, name)
    schema = str(torch.ops.gemma4_fa4_b200.global_layer_fwd.default._schema)
    assert "Tensor hidden_states" in schema and "Tensor k_norm_weight" in schema
    assert "!" not in schema  # nothing is mutated


@pytest.mark.parametrize("kind", ["local", "global"])
def test_fake_implementations_describe_fresh_outputs(kind):
    op = getattr(torch.ops.gemma4_fa4_b200, f"{kind}_layer_fwd")
    with FakeTensorMode():
        out, lse = op(*_layer_args(kind, s=12))
    assert out.shape == (1, 12, H) and out.dtype == torch.bfloat16
    assert lse.shape == (1, 32, 12) and lse.dtype == torch.float32
    op = getattr(torch.ops.gemma4_fa4_b200, f"{kind}_fwd")
    d = 256 if kind == "local" else 512
    with FakeTensorMode():
        out, lse = op(*_prepared_args(kind, s=12))
    assert out.shape == (1, 12, 32, d) and lse.shape == (1, 32, 12)


def test_layer_ops_require_no_grad_mode():
    with torch.enable_grad(), pytest.raises(UnsupportedB200Path, match="no-grad"):
        L.global_layer_fwd(*_layer_args("global"))
    args = _layer_args("local")
    args[1].requires_grad_(True)
    with torch.no_grad(), pytest.raises(UnsupportedB200Path, match="requires_grad"):
        L.local_layer_fwd(*args)


def test_host_tensors_are_refused_before_any_work():
    with torch.no_grad(), pytest.raises(UnsupportedB200Path, match="CUDA"):
        L.local_layer_fwd(*_layer_args("local"))
    with pytest.raises(UnsupportedB200Path, match="CUDA"):
        L.global_fwd(*_prepared_args("global"))
    args = _prepared_args("local")
    args[0] = torch.zeros(1, 32, 8, 256, **BF).requires_grad_(True)
    with pytest.raises(UnsupportedB200Path, match="requires_grad"):
        L.local_fwd(*args)
