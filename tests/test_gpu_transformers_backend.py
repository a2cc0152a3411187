"""A Gemma-4 text model (Transformers' own modeling code, random weights) run with
``attn_implementation="gemma4_fa4_b200"``: hidden states, weight gradients,
packed sequences and cached decoding.  The reference is the same model in FP32
with Transformers' eager attention; the B200 backend in BF16 must be no worse
than twice the error of BF16 eager attention against it (eager forms the d512
scores with BF16 matmuls, so it is the looser of the two)."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)
transformers = pytest.importorskip("transformers")

from gemma4_fa4_kernels_b200 import transformers_backend as tb  # noqa: E402

SLACK = 2e-3  # absolute slack on the rel-L2 comparison for cases where eager is near-exact


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-6)).item()


def _no_worse(mine, eager, ref, what=""):
    e_mine, e_eager = _rel(mine, ref), _rel(eager, ref)
    assert e_mine <= 2.0 * e_eager + SLACK, f"{what}: {e_mine:.3e} vs eager {e_eager:.3e}"
    return e_mine, e_eager


def _models():
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextModel

    tb.register_gemma4_fa4_b200()
    cfg = Gemma4TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                           num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                           head_dim=256, global_head_dim=512, num_global_key_value_heads=1,
                           attention_k_eq_v=True, sliding_window=1024,
                           layer_types=["sliding_attention", "full_attention"],
                           vocab_size_per_layer_input=512, hidden_size_per_layer_input=0,
                           max_position_embeddings=8192)
    torch.manual_seed(0)
    eager = Gemma4TextModel(cfg).to(device="cuda", dtype=torch.bfloat16)
    cfg2 = Gemma4TextConfig(**cfg.to_dict())
    mine = Gemma4TextModel(cfg2).to(device="cuda", dtype=torch.bfloat16)
    mine.load_state_dict(eager.state_dict())
    ref = Gemma4TextModel(Gemma4TextConfig(**cfg.to_dict())).to(device="cuda")
    ref.load_state_dict({k: v.float() for k, v in eager.state_dict().items()})
    eager.config._attn_implementation = "eager"
    ref.config._attn_implementation = "eager"
    mine.config._attn_implementation = tb.BACKEND_NAME
    return eager, mine, ref


def _paths(model):
    return [layer.self_attn._gemma4_fa4_b200_last_path for layer in model.layers]


def test_prefill_matches_the_fp32_model():
    eager, mine, ref = _models()
    ids = torch.randint(0, 512, (2, 300), device="cuda")
    with torch.no_grad():
        r = ref(input_ids=ids).last_hidden_state
        e = eager(input_ids=ids).last_hidden_state
        out = mine(input_ids=ids).last_hidden_state
    assert _paths(mine) == ["sliding_attention_fixed", "full_attention_fixed"]
    _no_worse(out, e, r, "hidden")


def test_gradients_match_the_fp32_model():
    eager, mine, ref = _models()
    ids = torch.randint(0, 512, (1, 257), device="cuda")
    for m in (eager, mine, ref):
        m(input_ids=ids).last_hidden_state.float().square().mean().backward()
    for layer_e, layer_m, layer_r in zip(eager.layers, mine.layers, ref.layers):
        for name in ("q_proj", "k_proj", "o_proj"):
            g = [getattr(layer.self_attn, name).weight.grad for layer in (layer_m, layer_e, layer_r)]
            _no_worse(*g, what=name)


def test_packed_sequences_use_documents():
    eager, mine, ref = _models()
    ids = torch.randint(0, 512, (1, 400), device="cuda")
    pos = torch.cat([torch.arange(150), torch.arange(100), torch.arange(150)])[None].cuda()
    with torch.no_grad():
        r = ref(input_ids=ids, position_ids=pos).last_hidden_state
        e = eager(input_ids=ids, position_ids=pos).last_hidden_state
        out = mine(input_ids=ids, position_ids=pos).last_hidden_state
    paths = _paths(mine)
    assert paths[0] in ("sliding_attention_documents", "sliding_attention_fixed")
    _no_worse(out, e, r, "hidden")
    if paths[0] == "sliding_attention_documents":
        assert paths[1] == "full_attention_packed"


def test_cached_decoding_matches_eager_attention():
    from transformers.cache_utils import DynamicCache

    eager, mine, ref = _models()
    ids = torch.randint(0, 512, (1, 120), device="cuda")
    caches = {}
    outs = {}
    with torch.no_grad():
        for name, m in (("eager", eager), ("mine", mine), ("ref", ref)):
            cache = DynamicCache(config=m.config)
            m(input_ids=ids, past_key_values=cache, use_cache=True)
            steps = []
            for t in range(3):
                torch.manual_seed(100 + t)
                nxt = torch.randint(0, 512, (1, 1), device="cuda")
                steps.append(m(input_ids=nxt, past_key_values=cache, use_cache=True)
                             .last_hidden_state)
            caches[name] = cache
            outs[name] = torch.cat(steps, dim=1)
    assert _paths(mine) == ["decode", "decode"]
    _no_worse(outs["mine"], outs["eager"], outs["ref"], "decode")


def _mask_mapping(model, ids, attention_mask, position_ids, image_types=None):
    """The masks a multimodal Gemma-4 forward builds: causal for full layers;
    sliding for local layers, with the image overlay (same image group in
    either direction) when ``image_types`` marks image tokens (Transformers'
    create_causal_mask_mapping for Gemma-4)."""
    from transformers.masking_utils import create_causal_mask, create_sliding_window_causal_mask
    from transformers.models.gemma4.modeling_gemma4 import token_type_ids_mask_function

    emb = model.embed_tokens(ids)
    kw = dict(config=model.config, inputs_embeds=emb, attention_mask=attention_mask,
              past_key_values=None, position_ids=position_ids)
    sliding_kw = dict(kw)
    if image_types is not None:
        is_img = image_types == 1
        prev = torch.roll(is_img, shifts=1, dims=-1)
        prev[..., 0] = False
        groups = torch.cumsum((is_img & ~prev).int(), dim=1) - 1
        groups = torch.where(is_img, groups, -1)
        sliding_kw["or_mask_function"] = token_type_ids_mask_function(image_types, groups)
    return {"full_attention": create_causal_mask(**kw),
            "sliding_attention": create_sliding_window_causal_mask(**sliding_kw)}


def _padded_inputs(b=2, s=300):
    ids = torch.randint(0, 512, (b, s), device="cuda")
    att = torch.ones(b, s, dtype=torch.long, device="cuda")
    att[0, :37] = 0      # left padding
    att[1, s - 51:] = 0  # right padding
    pos = (att.cumsum(-1) - 1).clamp_min(0)
    return ids, att, pos


def test_padded_batches_are_packed_into_varlen_calls():
    eager, mine, ref = _models()
    ids, att, pos = _padded_inputs()
    outs = {}
    with torch.no_grad():
        for name, m in (("ref", ref), ("eager", eager), ("mine", mine)):
            masks = _mask_mapping(m, ids, att, pos)
            outs[name] = m(input_ids=ids, attention_mask=masks,
                           position_ids=pos).last_hidden_state
    assert _paths(mine) == ["sliding_attention_padded", "full_attention_padded"]
    keep = att.bool()
    _no_worse(outs["mine"][keep], outs["eager"][keep], outs["ref"][keep], "padded hidden")


def test_multimodal_padded_batch_routes_images_to_the_kernels():
    """Image tokens (bidirectional within an image on the sliding layers) in a
    padded batch, forward and weight gradients, against the FP32 model."""
    eager, mine, ref = _models()
    ids, att, pos = _padded_inputs()
    types = torch.zeros_like(ids)
    types[0, 60:124] = 1     # an image of 64 tokens in row 0
    types[0, 200:300] = 1    # and one of 100 that ends the row
    types[1, 10:42] = 1      # an image in row 1, before its right padding
    keep = att.bool()
    outs = {}
    for name, m in (("ref", ref), ("eager", eager), ("mine", mine)):
        masks = _mask_mapping(m, ids, att, pos, types)
        h = m(input_ids=ids, attention_mask=masks, position_ids=pos).last_hidden_state
        h[keep].float().square().mean().backward()
        outs[name] = h.detach()
    assert _paths(mine) == ["sliding_attention_padded", "full_attention_padded"]
    _no_worse(outs["mine"][keep], outs["eager"][keep], outs["ref"][keep], "multimodal hidden")
    for layer_e, layer_m, layer_r in zip(eager.layers, mine.layers, ref.layers):
        for pname in ("q_proj", "k_proj", "o_proj"):
            g = [getattr(layer.self_attn, pname).weight.grad for layer in (layer_m, layer_e, layer_r)]
            _no_worse(*g, what=f"multimodal {pname}")


def test_multimodal_unpadded_uses_the_vision_kernels():
    eager, mine, ref = _models()
    ids = torch.randint(0, 512, (1, 400), device="cuda")
    types = torch.zeros_like(ids)
    types[0, 100:228] = 1
    pos = torch.arange(400, device="cuda")[None]
    outs = {}
    with torch.no_grad():
        for name, m in (("ref", ref), ("eager", eager), ("mine", mine)):
            masks = _mask_mapping(m, ids, None, pos, types)
            outs[name] = m(input_ids=ids, attention_mask=masks, position_ids=pos).last_hidden_state
    assert _paths(mine) == ["sliding_attention_vision", "full_attention_fixed"]
    _no_worse(outs["mine"], outs["eager"], outs["ref"], "vision hidden")
