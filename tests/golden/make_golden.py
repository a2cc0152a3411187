"""Generate the golden vectors that pin ``oracle/`` to the reference project.

Run from the repository root in a container where the reference project is
mounted (its ``src`` directory on ``sys.path``)::

    python tests/golden/make_golden.py /path/to/reference/src

It imports the reference package ``gemma4_fa4`` unmodified and records, for
small seeded cases, the outputs of its own CPU path:

* ``reference_attention`` / ``reference_attention_varlen`` forward outputs and
  natural-log LSE, plus float64 autograd gradients for a given ``dO`` and
  ``dLSE`` (``reference.py:23-198``);
* ``gemma4_attention_mask`` bool masks (``masks.py:8-80``);
* ``build_gemma4_local_sparse_schedule`` rows and storage bytes
  (``sparse_schedule.py:291-374``) and the storage upper bound;
* ``attention_flops`` (``reference.py:338-356``);
* the Q/K/V preparation: ``prepare_global_kv_from_projection_source``
  (``reference.py:306-328``) and the layer ops' ``_rms_norm`` /
  ``_apply_rotary`` (``h100_torch_ops.py:302-326``), with float64 autograd
  gradients of the source and the learned norm scale.

``--prep-only`` regenerates just the preparation fixtures.

The fixtures are written to ``tests/golden/*.npz`` / ``*.json`` next to this
script.  Nothing under ``tests/`` reads the reference at test time.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _attention_case(ref, name, *, b, hq, hkv, sq, sk, d, dv, window, vision=None, docs=None,
                    padding=None, bidir=False, seed=0, with_dlse=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, hq, sq, d, dtype=torch.float64, generator=g, requires_grad=True)
    k = torch.randn(b, hkv, sk, d, dtype=torch.float64, generator=g, requires_grad=True)
    v = torch.randn(b, hkv, sk, dv, dtype=torch.float64, generator=g, requires_grad=True)
    dout = torch.randn(b, hq, sq, dv, dtype=torch.float64, generator=g)
    # dLSE is rounded to float32 values: the reference returns an FP32 LSE,
    # so autograd carries its gradient in float32 through that cast.
    dlse = (torch.randn(b, hq, sq, dtype=torch.float64, generator=g).float().double()
            if with_dlse else None)
    kw = dict(sliding_window=window, allow_vision_bidirectional=bidir)
    if vision is not None:
        kw["vision_block_ids"] = torch.tensor(vision, dtype=torch.int32)
    if docs is not None:
        kw["document_ids"] = torch.tensor(docs, dtype=torch.int32)
    if padding is not None:
        kw["key_padding_mask"] = torch.tensor(padding, dtype=torch.bool)
    out, lse = ref.reference_attention(q, k, v, return_lse=True, **kw)
    # LSE is returned as float32; differentiate the float64 graph through it.
    loss = (out * dout).sum()
    if dlse is not None:
        finite = torch.isfinite(lse)
        loss = loss + (torch.where(finite, lse.double(), torch.zeros_like(lse.double())) * dlse).sum()
    loss.backward()
    arrays = dict(q=q.detach().numpy(), k=k.detach().numpy(), v=v.detach().numpy(),
                  dout=dout.numpy(), out=out.detach().numpy(), lse=lse.detach().numpy(),
                  dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy())
    if dlse is not None:
        arrays["dlse"] = dlse.numpy()
    meta = dict(window=-1 if window is None else window, bidir=int(bidir))
    for key, val in (("vision", vision), ("docs", docs), ("padding", padding)):
        if val is not None:
            arrays[key] = np.asarray(val)
    np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), **arrays,
                        meta=json.dumps(meta))


def _varlen_case(ref, name, *, cu_q, cu_k, hq, hkv, d, window, vision=None, docs=None,
                 bidir=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    tq, tk = cu_q[-1], cu_k[-1]
    q = torch.randn(tq, hq, d, dtype=torch.float64, generator=g, requires_grad=True)
    k = torch.randn(tk, hkv, d, dtype=torch.float64, generator=g, requires_grad=True)
    v = torch.randn(tk, hkv, d, dtype=torch.float64, generator=g, requires_grad=True)
    dout = torch.randn(tq, hq, d, dtype=torch.float64, generator=g)
    kw = dict(sliding_window=window, allow_vision_bidirectional=bidir)
    if vision is not None:
        kw["vision_block_ids"] = torch.tensor(vision, dtype=torch.int32)
    if docs is not None:
        kw["document_ids"] = torch.tensor(docs, dtype=torch.int32)
    out, lse = ref.reference_attention_varlen(
        q, k, v, torch.tensor(cu_q, dtype=torch.int32), torch.tensor(cu_k, dtype=torch.int32),
        return_lse=True, **kw)
    (out * dout).sum().backward()
    arrays = dict(q=q.detach().numpy(), k=k.detach().numpy(), v=v.detach().numpy(),
                  dout=dout.numpy(), out=out.detach().numpy(), lse=lse.detach().numpy(),
                  dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy(),
                  cu_q=np.asarray(cu_q, np.int32), cu_k=np.asarray(cu_k, np.int32))
    for key, val in (("vision", vision), ("docs", docs)):
        if val is not None:
            arrays[key] = np.asarray(val, np.int32)
    meta = dict(window=-1 if window is None else window, bidir=int(bidir))
    np.savez_compressed(os.path.join(HERE, f"varlen_{name}.npz"), **arrays, meta=json.dumps(meta))


def _prep_case(name, fn, arrays_in, grads_seed):
    """Run ``fn`` (returning (rot, plain)) under float64 autograd; save inputs,
    outputs, the cotangents and the gradients of x and the norm weight."""
    x = torch.from_numpy(arrays_in["x"]).requires_grad_(True)
    w = torch.from_numpy(arrays_in["weight"]).requires_grad_(True)
    cos, sin = torch.from_numpy(arrays_in["cos"]), torch.from_numpy(arrays_in["sin"])
    rot, plain = fn(x, w, cos, sin)
    g = torch.Generator().manual_seed(grads_seed)
    g_rot = torch.randn(rot.shape, dtype=torch.float64, generator=g)
    g_plain = torch.randn(plain.shape, dtype=torch.float64, generator=g)
    torch.autograd.backward((rot, plain), (g_rot, g_plain))
    np.savez_compressed(os.path.join(HERE, f"prep_{name}.npz"), **arrays_in,
                        rot=rot.detach().numpy(), plain=plain.detach().numpy(),
                        g_rot=g_rot.numpy(), g_plain=g_plain.numpy(), dx=x.grad.numpy(),
                        dweight=w.grad.numpy(),
                        meta=json.dumps(dict(rotary_dim=arrays_in["rotary_dim"].item())))


def prep_cases() -> None:
    import gemma4_fa4.h100_torch_ops as layer_ops
    import gemma4_fa4.reference as ref

    rng = np.random.default_rng(41)
    # global shared source Z in the reference helper's (B, H, S, D) layout with
    # (B, S, rotary_dim) tables: K = partial_RoPE(KNorm(Z)), V = VNorm(Z).
    x = rng.standard_normal((1, 2, 3, 512)) * 1.7
    ang = rng.uniform(0.0, 6.0, size=(1, 3, 128))
    arrays = dict(x=x, weight=rng.uniform(0.5, 1.5, size=512), cos=np.cos(ang), sin=np.sin(ang),
                  rotary_dim=np.array(128))

    def global_kv(x, w, cos, sin):
        return ref.prepare_global_kv_from_projection_source(
            x, k_norm_weight=w, cos=cos, sin=sin, partial_rotary_factor=0.25)

    _prep_case("global_kv_partial", global_kv, arrays, 42)

    # layer-op order: (B, S, H, D) operand, full-width HF tables (B, S, D).
    x = rng.standard_normal((1, 3, 2, 256)) * 0.6
    ang = rng.uniform(0.0, 6.0, size=(1, 3, 128))
    ang = np.concatenate((ang, ang), axis=-1)
    arrays = dict(x=x, weight=rng.uniform(0.5, 1.5, size=256), cos=np.cos(ang), sin=np.sin(ang),
                  rotary_dim=np.array(256))

    def layer_qk(x, w, cos, sin):
        return (layer_ops._apply_rotary(layer_ops._rms_norm(x, w), cos, sin),
                layer_ops._rms_norm(x, None))

    _prep_case("layer_full_d256", layer_qk, arrays, 43)


def main(reference_src: str) -> None:
    sys.path.insert(0, reference_src)
    prep_cases()
    import gemma4_fa4.reference as ref
    from gemma4_fa4.masks import gemma4_attention_mask
    from gemma4_fa4.model_spec import GLOBAL_ATTENTION, SLIDING_ATTENTION
    from gemma4_fa4.sparse_schedule import (
        build_gemma4_local_sparse_schedule,
        gemma4_local_sparse_storage_upper_bound,
    )

    # --- attention forward + float64 autograd backward -------------------------------
    _attention_case(ref, "local_text", b=1, hq=4, hkv=2, sq=37, sk=37, d=16, dv=16, window=8,
                    bidir=True, seed=1)
    vis = [[-1] * 5 + [3] * 7 + [-1] * 6 + [9] * 6 + [-1] * 5,
           [2] * 4 + [-1] * 10 + [2] * 3 + [-1] * 12]
    docs = [[0] * 15 + [1] * 14, [4] * 20 + [5] * 9]
    _attention_case(ref, "local_vision_doc", b=2, hq=4, hkv=2, sq=29, sk=29, d=16, dv=16,
                    window=6, vision=vis, docs=docs, bidir=True, seed=2)
    _attention_case(ref, "global_rect_gqa8", b=1, hq=8, hkv=1, sq=11, sk=23, d=16, dv=16,
                    window=None, seed=3)
    _attention_case(ref, "global_d512_gqa8", b=1, hq=8, hkv=1, sq=9, sk=9, d=512, dv=512,
                    window=None, seed=4)
    _attention_case(ref, "local_d256_gqa2", b=1, hq=2, hkv=1, sq=13, sk=13, d=256, dv=256,
                    window=4, bidir=True, seed=5)
    _attention_case(ref, "masked_row", b=1, hq=2, hkv=1, sq=4, sk=4, d=8, dv=8, window=None,
                    padding=[[False, True, True, False]], seed=6, with_dlse=False)
    # A fully masked query row (query 0 only sees key 0, which is padded out).
    _attention_case(ref, "all_masked_first_row", b=1, hq=1, hkv=1, sq=3, sk=3, d=8, dv=8,
                    window=None, padding=[[False, True, True]], seed=7, with_dlse=False)

    # --- packed varlen: mixed empty segments, vision + documents ---------------------
    _varlen_case(ref, "mixed_empty", cu_q=[0, 3, 3, 7, 9], cu_k=[0, 5, 6, 13, 15], hq=4, hkv=2,
                 d=8, window=4, seed=11)
    vis_p = [-1, 1, 1, 1, -1, -1, 2, 2, -1, 1, 1, -1, -1, -1, 3, 3, 3]
    docs_p = [0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 2, 2, 2, 2, 2]
    _varlen_case(ref, "vision_doc", cu_q=[0, 4, 9, 12], cu_k=[0, 5, 12, 17], hq=2, hkv=1, d=8,
                 window=3, vision=vis_p, docs=docs_p, bidir=True, seed=12)

    # --- masks -----------------------------------------------------------------------
    masks = {}
    rng = np.random.default_rng(21)
    for i in range(24):
        b = int(rng.integers(1, 3))
        kv_len = int(rng.integers(1, 40))
        q_len = int(rng.integers(0, kv_len + 1))
        window = [None, 1, 3, 8, 1024][i % 5]
        vis_a = rng.integers(-1, 3, size=(b, kv_len)).astype(np.int32)
        doc_a = rng.integers(0, 2, size=(b, kv_len)).astype(np.int32)
        pad_a = rng.random((b, kv_len)) > 0.2
        bidir = bool(i % 2)
        m = gemma4_attention_mask(
            batch_size=b, q_len=q_len, kv_len=kv_len, device="cpu", sliding_window=window,
            vision_block_ids=torch.from_numpy(vis_a) if i % 3 else None,
            document_ids=torch.from_numpy(doc_a) if i % 4 else None,
            key_padding_mask=torch.from_numpy(pad_a) if i % 5 == 0 else None,
            allow_vision_bidirectional=bidir)
        masks[f"case{i}"] = dict(b=b, q_len=q_len, kv_len=kv_len, window=window, bidir=bidir,
                                 vision=vis_a.tolist() if i % 3 else None,
                                 docs=doc_a.tolist() if i % 4 else None,
                                 padding=pad_a.tolist() if i % 5 == 0 else None,
                                 mask=m.numpy().astype(np.uint8).tolist(),
                                 shape=list(m.shape))
    with open(os.path.join(HERE, "masks.json"), "w") as f:
        json.dump(masks, f)

    # --- sparse schedules ------------------------------------------------------------
    scheds = {}
    rng = np.random.default_rng(31)
    for i in range(40):
        k_len = int(rng.integers(1, 70))
        q_len = int(rng.integers(1, k_len + 1))
        vis_s = rng.integers(-1, 4, size=k_len).tolist()
        doc_s = np.sort(rng.integers(0, 3, size=k_len)).tolist() if i % 2 else \
            rng.integers(0, 2, size=k_len).tolist()
        window = [4, 7, 16, 1024][i % 4]
        fb = [(8, 5), (16, 16), (4, 4), (128, 80)][i % 4]
        bb = [(4, 4), (8, 8), (2, 3), (64, 64)][i % 4]
        s = build_gemma4_local_sparse_schedule(
            vis_s, doc_s, q_length=q_len, k_length=k_len, sliding_window=window,
            forward_block_size=fb, backward_block_size=bb)
        scheds[f"case{i}"] = dict(q_length=q_len, k_length=k_len, vision=vis_s, docs=doc_s,
                                  window=window, forward_block_size=fb, backward_block_size=bb,
                                  forward=[list(r) for r in s.forward.rows],
                                  backward=[list(r) for r in s.backward.rows],
                                  forward_storage_bytes=s.forward.storage_bytes,
                                  backward_storage_bytes=s.backward.storage_bytes)
    # the reference pins this bound for the model maximum (test_sparse_schedule.py:174-175)
    scheds["upper_bound_262144"] = gemma4_local_sparse_storage_upper_bound(262144, 262144)
    with open(os.path.join(HERE, "schedules.json"), "w") as f:
        json.dump(scheds, f)

    # --- FLOP counter ----------------------------------------------------------------
    flops = {}
    for label, spec in (("local", SLIDING_ATTENTION), ("global", GLOBAL_ATTENTION)):
        for s in (1, 100, 1024, 2048, 4096, 8192):
            for mode in ("fwd", "bwd", "fwd_bwd"):
                flops[f"{label}_{s}_{mode}"] = ref.attention_flops(spec, batch=1, seqlen=s, mode=mode)
    with open(os.path.join(HERE, "flops.json"), "w") as f:
        json.dump(flops, f, indent=0)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        sys.exit("usage: python tests/golden/make_golden.py <reference src dir> [--prep-only]")
    src = args[0]
    if "--prep-only" in sys.argv:
        sys.path.insert(0, src)
        prep_cases()
    else:
        main(src)
