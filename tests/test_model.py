"""Model on CPU: architecture variants, KV cache, masking, generation, initialisation, accounting."""
import math

import pytest
import torch
import torch.nn.functional as F

from olmo_b200.config import ActivationCheckpointingStrategy, InitFnType, ModelConfig
from olmo_b200.models.blocks import OLMoBlockGroup, OLMoLlamaBlock, OLMoSequentialBlock
from olmo_b200.models.layers import LayerNorm, RMSLayerNorm
from olmo_b200.models.olmo import OLMo


def cfg(**kw) -> ModelConfig:
    base = dict(d_model=64, n_heads=4, n_layers=2, vocab_size=97, embedding_size=128, max_sequence_length=32, init_device="cpu",
                flash_attention=False, include_bias=False, rope=True, alibi=False, attention_dropout=0.0, residual_dropout=0.0,
                embedding_dropout=0.0, eos_token_id=96, pad_token_id=95)
    base.update(kw)
    return ModelConfig(**base)


def make(**kw) -> OLMo:
    torch.manual_seed(0)
    m = OLMo(cfg(**kw))
    m.reset_parameters()
    return m.eval()


VARIANTS = {
    "olmo1": dict(layer_norm_type="default", layer_norm_with_affine=False),
    "olmo2": dict(layer_norm_type="rms", layer_norm_with_affine=True, attention_layer_norm=True, attention_layer_norm_with_affine=True,
                  norm_after=True, rope_theta=500000, init_fn="normal", init_cutoff_factor=3),
    "alibi": dict(alibi=True, rope=False),
    "learned_positions": dict(rope=False, alibi=False),
    "mqa": dict(multi_query_attention=True),
    "gqa": dict(n_kv_heads=2),
    "llama": dict(block_type="llama", layer_norm_type="rms"),
    "bias_tied_clip": dict(include_bias=True, weight_tying=True, clip_qkv=4.0, bias_for_layer_norm=True, layer_norm_with_affine=True),
    "gelu_wide": dict(activation_type="gelu", mlp_ratio=3),
    "relu_fullprec_rope": dict(activation_type="relu", rope_full_precision=False),
    "scaled_logits_embnorm": dict(scale_logits=True, embedding_layer_norm=True),
    "groups": dict(n_layers=4, block_group_size=2),
}


@pytest.mark.parametrize("name", sorted(VARIANTS))
def test_forward_backward_every_variant(name):
    m = make(**VARIANTS[name]).train()
    ids = torch.randint(0, 97, (3, 12))
    out = m(ids)
    assert out.logits.shape == (3, 12, 128) and out.attn_key_values is None
    loss = F.cross_entropy(out.logits.view(-1, 128), ids.view(-1))
    loss.backward()
    missing = [n for n, p in m.named_parameters() if p.grad is None]
    assert not missing, missing
    assert all(torch.isfinite(p.grad).all() for p in m.parameters())


@pytest.mark.parametrize("name", ["olmo1", "olmo2", "alibi", "gqa", "llama", "learned_positions"])
def test_kv_cache_matches_full_forward(name):
    m = make(**VARIANTS[name])
    ids = torch.randint(0, 97, (2, 10))
    with torch.no_grad():
        full = m(ids).logits
        first = m(ids[:, :6], use_cache=True)
        assert len(first.attn_key_values) == 2
        step_logits = [first.logits]
        past = first.attn_key_values
        for t in range(6, 10):
            out = m(ids[:, t : t + 1], past_key_values=past, use_cache=True)
            past = out.attn_key_values
            step_logits.append(out.logits)
        last_only = m(ids, last_logits_only=True).logits
    torch.testing.assert_close(torch.cat(step_logits, dim=1), full, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(last_only, full[:, -1:], rtol=1e-5, atol=1e-5)
    assert past[0][0].shape[-2] == 10


@pytest.mark.parametrize("name", ["olmo1", "alibi"])
def test_left_padding_with_mask_does_not_change_logits(name):
    m = make(**VARIANTS[name])
    a, b = torch.randint(0, 90, (1, 9)), torch.randint(0, 90, (1, 5))
    with torch.no_grad():
        alone = m(b).logits
        batch_ids = torch.cat([a, torch.cat([torch.full((1, 4), 95), b], dim=1)], dim=0)
        mask = torch.ones(2, 9)
        mask[1, :4] = 0
        both = m(batch_ids, attention_mask=mask).logits
    if name == "alibi":  # relative biases are position-shift invariant
        torch.testing.assert_close(both[1, 4:], alone[0], rtol=1e-4, atol=1e-4)
    else:  # rotary phases are relative too
        torch.testing.assert_close(both[1, 4:], alone[0], rtol=1e-3, atol=1e-3)


def test_attention_bias_forms_agree():
    m = make(**VARIANTS["olmo1"])
    ids = torch.randint(0, 97, (2, 8))
    causal_bool = torch.tril(torch.ones(8, 8, dtype=torch.bool)).view(1, 1, 8, 8)
    causal_float = torch.zeros(1, 1, 8, 8).masked_fill(~causal_bool, float("-inf"))
    with torch.no_grad():
        base = m(ids).logits
        torch.testing.assert_close(m(ids, attention_bias=causal_bool).logits, base, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(m(ids, attention_bias=causal_float).logits, base, rtol=1e-4, atol=1e-4)


def test_document_masking_equals_separate_documents():
    m = make(**VARIANTS["olmo2"])
    doc_a, doc_b = torch.randint(0, 90, (1, 5)), torch.randint(0, 90, (1, 7))
    packed = torch.cat([doc_a, doc_b], dim=1)
    with torch.no_grad():
        sep_b = m(doc_b).logits
        sep_a = m(doc_a).logits
        joint = m(packed, doc_lens=torch.tensor([[5, 7]]), max_doc_lens=[7]).logits
        leaky = m(packed).logits
    torch.testing.assert_close(joint[:, :5], sep_a, rtol=1e-4, atol=1e-4)
    # the second document restarts attention but keeps absolute rotary positions, which are relative in effect
    torch.testing.assert_close(joint[:, 5:], sep_b, rtol=1e-3, atol=1e-3)
    assert not torch.allclose(leaky[:, 5:], sep_b, rtol=1e-3, atol=1e-3)


def test_input_embeddings_and_hidden_states():
    m = make(**VARIANTS["olmo2"])
    ids = torch.randint(0, 97, (2, 6))
    with torch.no_grad():
        emb = m.transformer.wte(ids)
        a = m(ids, output_hidden_states=True)
        b = m(None, input_embeddings=emb)
    torch.testing.assert_close(a.logits, b.logits)
    assert len(a.hidden_states) == 3 and a.hidden_states[0].shape == (2, 6, 64)
    torch.testing.assert_close(m.output_projection(m.hidden_before_head(ids)), a.logits, rtol=1e-5, atol=1e-5)


def test_greedy_generate_matches_argmax_loop_and_beams_are_sorted():
    m = make(**VARIANTS["olmo2"])
    prompt = torch.randint(0, 90, (2, 5))
    out = m.generate(prompt, max_steps=6, beam_size=1)
    assert out.token_ids.shape[:2] == (2, 1)
    ids = prompt.clone()
    want = []
    alive = torch.ones(2, dtype=torch.bool)
    with torch.no_grad():
        for _ in range(out.token_ids.shape[-1]):
            nxt = m(ids).logits[:, -1].log_softmax(-1).argmax(-1)
            nxt = torch.where(alive, nxt, torch.full_like(nxt, 96))
            alive &= nxt != 96
            want.append(nxt)
            ids = torch.cat([ids, nxt[:, None]], dim=1)
    assert out.token_ids[:, 0].tolist() == torch.stack(want, dim=1).tolist()
    beams = m.generate(prompt, max_steps=4, beam_size=3)
    assert beams.token_ids.shape[:2] == (2, 3) and bool((beams.scores[:, :-1] >= beams.scores[:, 1:]).all())
    assert float(beams.scores[0, 0]) >= float(out.scores[0, 0]) - 1e-4 or beams.token_ids.shape[-1] != out.token_ids.shape[-1]
    mask = torch.ones_like(prompt)
    masked = m.generate(prompt, attention_mask=mask, max_steps=6, beam_size=1)
    assert masked.token_ids.tolist() == out.token_ids.tolist()


@pytest.mark.parametrize("strategy", list(ActivationCheckpointingStrategy))
def test_activation_checkpointing_keeps_gradients(strategy):
    ids = torch.randint(0, 97, (2, 8))

    def grads(strat):
        m = make(n_layers=4, **VARIANTS["olmo2"]).train()
        m.set_activation_checkpointing(strat)
        F.cross_entropy(m(ids).logits.view(-1, 128), ids.view(-1)).backward()
        return [p.grad.clone() for p in m.parameters()]

    for a, b in zip(grads(None), grads(strategy)):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


def test_layer_norms_match_torch():
    c = cfg(layer_norm_with_affine=True, bias_for_layer_norm=True, layer_norm_eps=1e-5)
    x = torch.randn(3, 5, 64)
    ln = LayerNorm(c)
    with torch.no_grad():
        ln.weight.uniform_(0.5, 1.5)
        ln.bias.uniform_(-0.5, 0.5)
    torch.testing.assert_close(ln(x), F.layer_norm(x, (64,), ln.weight, ln.bias, 1e-5))
    plain = LayerNorm(cfg(layer_norm_with_affine=False))
    assert plain.weight is None and plain.bias is None
    torch.testing.assert_close(plain(x), F.layer_norm(x, (64,), None, None, 1e-5))
    rms = RMSLayerNorm(cfg(layer_norm_with_affine=True, bias_for_layer_norm=False, layer_norm_eps=1e-6))
    with torch.no_grad():
        rms.weight.uniform_(0.5, 1.5)
    want = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * rms.weight
    torch.testing.assert_close(rms(x), want, rtol=1e-5, atol=1e-6)
    assert rms.bias is None


def test_block_groups_share_parameter_layout_with_flat_blocks():
    flat, grouped = make(n_layers=4), make(n_layers=4, block_group_size=2)
    assert isinstance(grouped.transformer.block_groups[0], OLMoBlockGroup) and len(grouped.transformer.block_groups) == 2
    assert sum(p.numel() for p in flat.parameters()) == sum(p.numel() for p in grouped.parameters())
    assert "transformer.block_groups.1.0.att_proj.weight" in grouped.state_dict()
    # grouped state re-keyed to the flat layout loads into the flat model and gives identical logits
    sd = {}
    for k, v in grouped.state_dict().items():
        if ".block_groups." in k:
            head, rest = k.split(".block_groups.")
            g, i, tail = rest.split(".", 2)
            k = f"{head}.blocks.{int(g) * 2 + int(i)}.{tail}"
        sd[k] = v
    flat.load_state_dict(sd)
    ids = torch.randint(0, 97, (2, 7))
    with torch.no_grad():
        torch.testing.assert_close(flat(ids).logits, grouped(ids).logits)
    assert [b.layer_id for b in grouped.all_blocks()] == [0, 1, 2, 3]


def test_block_classes_and_kv_widths():
    assert isinstance(make().transformer.blocks[0], OLMoSequentialBlock)
    assert isinstance(make(block_type="llama").transformer.blocks[0], OLMoLlamaBlock)
    gqa = make(n_kv_heads=2).transformer.blocks[0]
    assert gqa.att_proj.out_features == 64 + 2 * 2 * 16
    mqa = make(multi_query_attention=True).transformer.blocks[0]
    assert mqa.att_proj.out_features == 64 + 2 * 16
    swiglu = make(mlp_hidden_size=192).transformer.blocks[0]
    assert swiglu.ff_proj.out_features == 192 and swiglu.ff_out.in_features == 96


def _std(t):
    return float(t.detach().float().std())


@pytest.mark.parametrize("seed", [0, 1])
def test_init_normal_with_cutoff(seed):
    torch.manual_seed(seed)
    m = OLMo(cfg(d_model=256, n_heads=4, n_layers=2, init_fn="normal", init_std=0.02, init_cutoff_factor=3, layer_norm_with_affine=True))
    m.reset_parameters()
    for name, p in m.named_parameters():
        if name.endswith("norm.weight") or "ln_f" in name:
            assert bool((p == 1).all())
        elif p.dim() == 2:
            assert float(p.detach().abs().max()) <= 0.06 + 1e-6, name
            assert _std(p) == pytest.approx(0.02, rel=0.08), name


def test_init_mitchell_scales_with_width_and_depth():
    torch.manual_seed(0)
    d, L = 256, 4
    m = OLMo(cfg(d_model=d, n_heads=4, n_layers=L, init_fn="mitchell", vocab_size=997, embedding_size=1024, weight_tying=False))
    m.reset_parameters()
    assert _std(m.transformer.wte.weight) == pytest.approx(1 / math.sqrt(d), rel=0.08)
    assert _std(m.transformer.ff_out.weight) == pytest.approx(1 / math.sqrt(d), rel=0.08)
    for i, blk in enumerate(m.transformer.blocks):
        assert _std(blk.att_proj.weight) == pytest.approx(1 / math.sqrt(d), rel=0.08)
        assert _std(blk.attn_out.weight) == pytest.approx(1 / math.sqrt(2 * d * (i + 1)), rel=0.08)
        assert _std(blk.ff_out.weight) == pytest.approx(1 / math.sqrt(2 * blk.ff_out.in_features * (i + 1)), rel=0.08)


def test_init_full_megatron():
    torch.manual_seed(0)
    d, L, std = 256, 4, 0.006
    m = OLMo(cfg(d_model=d, n_heads=4, n_layers=L, init_fn=InitFnType.full_megatron, init_std=std, init_cutoff_factor=3, scale_emb_init=True,
                 vocab_size=997, embedding_size=1024, weight_tying=False))
    m.reset_parameters()
    assert _std(m.transformer.wte.weight) == pytest.approx(std * math.sqrt(d), rel=0.08)
    assert _std(m.transformer.ff_out.weight) == pytest.approx(1 / math.sqrt(d), rel=0.08)
    blk = m.transformer.blocks[1]
    assert _std(blk.att_proj.weight) == pytest.approx(std, rel=0.08)
    assert _std(blk.attn_out.weight) == pytest.approx(std / math.sqrt(2 * L), rel=0.08)
    assert _std(blk.ff_out.weight) == pytest.approx(std / math.sqrt(2 * L), rel=0.08)


def test_parameter_and_flop_accounting():
    m = make(n_layers=3, mlp_hidden_size=256)
    total = sum(p.numel() for p in m.parameters())
    assert m.num_params() == total
    assert m.num_params(include_embedding=False) == total - m.transformer.wte.weight.numel()
    c = m.config
    attn = c.n_layers * c.d_model * c.max_sequence_length
    assert m.num_fwd_flops == 2 * m.num_params(include_embedding=False) + 4 * attn
    assert m.num_bck_flops == 4 * m.num_params() + 8 * attn
    tied, untied = make(weight_tying=True), make(weight_tying=False)
    assert not hasattr(tied.transformer, "ff_out") and hasattr(untied.transformer, "ff_out")
    assert untied.num_params() - tied.num_params() == 128 * 64


def test_meta_device_and_compatibility_of_old_state_dicts():
    m = OLMo(cfg(init_device="meta"), init_params=False)
    assert all(p.is_meta for p in m.parameters())
    live = make(layer_norm_with_affine=True)
    sd = live.state_dict()
    old = dict(sd)
    # checkpoints older than the attn_norm/ff_norm split stored one ``norm`` per block
    for i in range(2):
        old[f"transformer.blocks.{i}.norm.weight"] = old.pop(f"transformer.blocks.{i}.attn_norm.weight")
        old.pop(f"transformer.blocks.{i}.ff_norm.weight")
    fixed, renamed = live._make_state_dict_compatible(old)
    assert set(fixed) == set(sd)
    torch.testing.assert_close(fixed["transformer.blocks.0.ff_norm.weight"], sd["transformer.blocks.0.attn_norm.weight"])
    assert "transformer.blocks.0.attn_norm.weight" in renamed or renamed
