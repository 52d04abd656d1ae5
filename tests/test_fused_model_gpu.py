"""The fused sm_100a training path against the portable fp32 autograd path on identical weights."""
import tempfile

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _cfg(precision: str, flavour: str = "olmo2", n_kv_heads=None, n_heads: int = 2, seq: int = 256):
    from olmo_b200.config import (
        DistributedStrategy, LayerNormType, ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig, SchedulerType, TrainConfig,
    )
    from olmo_b200.launch import derive_batch_sizes

    olmo2 = flavour == "olmo2"
    model = ModelConfig(
        d_model=256, n_heads=n_heads, n_kv_heads=n_kv_heads, n_layers=2, mlp_hidden_size=1024, weight_tying=False, rope=True,
        rope_theta=500000 if olmo2 else 10000, flash_attention=True, attention_dropout=0.0, residual_dropout=0.0,
        embedding_dropout=0.0, include_bias=False, layer_norm_type=LayerNormType.rms if olmo2 else LayerNormType.default,
        layer_norm_with_affine=olmo2, layer_norm_eps=1e-6 if olmo2 else 1e-5, bias_for_layer_norm=False,
        attention_layer_norm=olmo2, norm_after=olmo2, clip_qkv=None if olmo2 else 2.0, max_sequence_length=seq,
        vocab_size=500, embedding_size=512, eos_token_id=499, pad_token_id=499, init_device="meta", init_std=0.05,
    )
    cfg = TrainConfig(
        model=model, optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=1e-3, eps=1e-8, weight_decay=0.1),
        scheduler=SchedulerConfig(name=SchedulerType.constant), precision=precision, distributed_strategy=DistributedStrategy.single,
        global_train_batch_size=2, device_train_microbatch_size=2, max_grad_norm=1.0, save_folder=tempfile.mkdtemp(),
    )
    derive_batch_sizes(cfg, 1)
    return cfg


@pytest.mark.parametrize("flavour,n_kv", [("olmo2", None), ("olmo1", None)])
def test_fused_gradients_match_portable(flavour, n_kv):
    from olmo_b200 import ops
    from olmo_b200.launch import build_model_and_engine

    device = torch.device("cuda")
    fused = build_model_and_engine(_cfg("amp_bf16", flavour, n_kv), device).engine
    assert fused.fused
    oracle = build_model_and_engine(_cfg("fp32", flavour, n_kv), device, force_portable=True).engine
    assert not oracle.fused
    # identical weights: the bf16-rounded values of the fused engine
    state = {s.name: u.full[s.offset : s.offset + s.numel].view(s.shape).float() for u in fused.units for s in u.slots}
    oracle.load_full_model_state_dict(state)
    fused.load_full_model_state_dict(state)

    torch.manual_seed(1)
    ids = torch.randint(0, 500, (2, 256), device=device)
    labels = F.pad(ids[:, 1:], (0, 1), value=-100)
    labels[0, 10:20] = -100
    divisor, z_mult = float(ids.numel()), 1e-4

    fused.zero_grad()
    ce, z = fused.train_microbatch(ids, labels, divisor, z_mult=z_mult)
    ops.check_status()

    oracle.zero_grad()
    logits = oracle.model(ids).logits.float().view(-1, 512)
    ce_ref = F.cross_entropy(logits, labels.view(-1), ignore_index=-100, reduction="sum") / divisor
    lse = torch.logsumexp(logits, -1)
    z_ref = z_mult * (lse.square() * (labels.view(-1) != -100)).sum() / divisor
    (ce_ref + z_ref).backward()
    oracle.note_microbatch_backward()
    oracle.finish_grad_sync()

    assert abs(ce.item() - ce_ref.item()) < 2e-2 * abs(ce_ref.item())
    assert abs(z.item() - z_ref.item()) < 3e-2 * abs(z_ref.item()) + 1e-6
    for uf, uo in zip(fused.units, oracle.units):
        for s in uf.slots:
            so = uo.slot(s.name)
            g = uf.grad[s.offset : s.offset + s.numel]
            r = uo.grad[so.offset : so.offset + so.numel]
            scale = r.abs().max().item()
            err = (g - r).abs().max().item()
            assert err <= 0.1 * scale + 1e-7, f"{s.name}: max err {err} vs scale {scale}"
            rel = ((g - r).norm() / (r.norm() + 1e-12)).item()
            assert rel < 4e-2, f"{s.name}: relative error {rel}"


def test_fused_forward_matches_portable_module():
    """The autograd-visible fused block (used by ``OLMo.forward`` on CUDA) reproduces the portable logits."""
    from olmo_b200.models.olmo import OLMo

    cfg = _cfg("amp_bf16").model
    cfg.init_device = "cuda"
    torch.manual_seed(0)
    model = OLMo(cfg).eval()
    ids = torch.randint(0, 500, (2, 256), device="cuda")
    import os

    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused_logits = model(ids).logits.float()
        os.environ["OLMO_B200_KERNELS"] = "0"
        try:
            ref_logits = model(ids).logits.float()
        finally:
            os.environ.pop("OLMO_B200_KERNELS")
    err = (fused_logits - ref_logits).abs().max().item()
    assert err < 5e-2 * ref_logits.abs().max().item(), err


def test_train_steps_reduce_loss():
    import __graft_entry__ as entry

    entry.smoke()


@pytest.mark.parametrize("n_heads,T,doc_lens,max_doc_lens", [
    (2, 256, [[60, 130, 66, 0], [128, 100, 20, 8]], [130, 128]),   # head dim 128, whole tiles
    (4, 200, [[60, 100, 40, 0], [128, 50, 14, 8]], [100, 128]),    # head dim 64 and a ragged length: reached by zero padding
])
def test_fused_document_masking_matches_portable(n_heads, T, doc_lens, max_doc_lens):
    """Intra-document masking on the fused engine path (native attention kernels with per-token document starts)
    against the portable fp32 autograd path driven by ``doc_lens``."""
    from olmo_b200 import ops
    from olmo_b200.launch import build_model_and_engine
    from olmo_b200.ops.attention_native import doc_start_from_lengths

    device = torch.device("cuda")
    fused = build_model_and_engine(_cfg("amp_bf16", "olmo2", n_heads=n_heads, seq=T), device).engine
    oracle = build_model_and_engine(_cfg("fp32", "olmo2", n_heads=n_heads, seq=T), device, force_portable=True).engine
    assert fused.fused
    state = {s.name: u.full[s.offset : s.offset + s.numel].view(s.shape).float() for u in fused.units for s in u.slots}
    oracle.load_full_model_state_dict(state)
    fused.load_full_model_state_dict(state)

    torch.manual_seed(2)
    ids = torch.randint(0, 500, (2, T), device=device)
    labels = F.pad(ids[:, 1:], (0, 1), value=-100)
    doc_lens = torch.tensor(doc_lens, device=device)
    divisor = float(ids.numel())

    fused.zero_grad()
    ce, _ = fused.train_microbatch(ids, labels, divisor, z_mult=0.0, doc_start=doc_start_from_lengths(doc_lens, T))
    ops.check_status()
    fused.zero_grad()
    ce_plain, _ = fused.train_microbatch(ids, labels, divisor, z_mult=0.0)

    oracle.zero_grad()
    logits = oracle.model(ids, doc_lens=doc_lens, max_doc_lens=max_doc_lens).logits.float().view(-1, 512)
    ce_ref = F.cross_entropy(logits, labels.view(-1), ignore_index=-100, reduction="sum") / divisor
    ce_ref.backward()
    oracle.note_microbatch_backward()
    oracle.finish_grad_sync()

    assert abs(ce.item() - ce_ref.item()) < 2e-2 * abs(ce_ref.item())
    assert abs(ce_plain.item() - ce.item()) > 1e-4  # the mask changes the loss

    fused.zero_grad()
    fused.train_microbatch(ids, labels, divisor, z_mult=0.0, doc_start=doc_start_from_lengths(doc_lens, T))
    for uf, uo in zip(fused.units, oracle.units):
        for s in uf.slots:
            so = uo.slot(s.name)
            g = uf.grad[s.offset : s.offset + s.numel]
            r = uo.grad[so.offset : so.offset + so.numel]
            rel = ((g - r).norm() / (r.norm() + 1e-12)).item()
            assert rel < 5e-2, f"{s.name}: relative error {rel}"


@pytest.mark.parametrize("flavour", ["olmo2", "olmo1"])
def test_kept_activations_give_the_same_gradients_as_recomputed_ones(flavour):
    """The backward pass either recomputes the rotated q/k and the SwiGLU output or reads the copies the forward pass
    kept; both run the same kernels on the same inputs, so the loss is identical and the gradients agree up to the
    order of floating-point atomics."""
    from olmo_b200 import ops
    from olmo_b200.config import ActivationCheckpointingStrategy
    from olmo_b200.launch import build_model_and_engine

    device = torch.device("cuda")
    engine = build_model_and_engine(_cfg("amp_bf16", flavour), device).engine
    assert engine.fused
    torch.manual_seed(3)
    ids = torch.randint(0, 500, (2, 256), device=device)
    labels = F.pad(ids[:, 1:], (0, 1), value=-100)

    def grads(keep, ac=None):
        engine.keep_recomputable = keep
        engine.zero_grad()
        ce, _ = engine.train_microbatch(ids, labels, float(ids.numel()), z_mult=1e-4, ac_strategy=ac)
        ops.check_status()
        return ce.item(), {s.name: u.grad[s.offset : s.offset + s.numel].clone() for u in engine.units for s in u.slots}

    ce_a, recomputed = grads(False)
    ce_b, kept = grads(True)
    ce_c, checkpointed = grads(False, ActivationCheckpointingStrategy.whole_layer)
    assert ce_a == ce_b == ce_c
    for name, g in recomputed.items():
        for other in (kept, checkpointed):
            # dQ tiles and embedding rows are accumulated with floating-point atomics, whose order varies run to run
            rel = ((other[name] - g).norm() / (g.norm() + 1e-12)).item()
            assert rel < 1e-3, f"{name}: relative difference {rel}"
