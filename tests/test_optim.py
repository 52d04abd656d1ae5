"""Optimizers, gradient clipping / metrics, parameter groups and LR schedules (CPU)."""
import math

import pytest
import torch
import torch.nn as nn

from olmo_b200.config import ModelConfig, OptimizerConfig, OptimizerType, SchedulerConfig, SchedulerType, TrainConfig
from olmo_b200.models.olmo import OLMo
from olmo_b200.optim import (
    AdamW,
    BoltOnWarmupScheduler,
    ConstantScheduler,
    ConstantWithWarmupScheduler,
    CosLinearEnvelope,
    CosWithWarmup,
    InvSqrtWithWarmup,
    LinearWithWarmup,
    LionW,
    MaxScheduler,
    build_optimizer,
    build_scheduler,
    fix_optim_state_dict,
    get_param_groups,
)

BASE = dict(grad_clip_warmup_steps=None, grad_clip_warmup_factor=None, warmup_min_lr=None)


def tiny_config(**kw) -> TrainConfig:
    model = ModelConfig(d_model=32, n_heads=2, n_layers=2, vocab_size=64, embedding_size=64, max_sequence_length=16, init_device="cpu",
                        flash_attention=False, include_bias=False, layer_norm_with_affine=True, layer_norm_type="rms")
    return TrainConfig(model=model, **kw)


# ------------------------------------------------------------------------------------- schedules


def test_linear_schedule_golden_values():
    s = LinearWithWarmup(**BASE, warmup_steps=2000, alpha_f=0.1)
    lr, T = 1.0, 10_000
    assert s.get_lr(lr, 0, T) == pytest.approx(0.1)
    assert s.get_lr(lr, 2000, T) == pytest.approx(1.0)
    assert s.get_lr(lr, T, T) == pytest.approx(0.1)
    assert s.get_lr(lr, 3000, T) > s.get_lr(lr, 5000, T)
    assert s.get_lr(lr, 6000, T) == pytest.approx(1.0 - 0.9 * 0.5)
    assert s.get_lr(lr, 2 * T, T) == pytest.approx(0.1)


def test_bolt_on_warmup_golden_values():
    alpha = 0.1
    inner = LinearWithWarmup(**BASE, warmup_steps=1000, alpha_f=alpha)
    s = BoltOnWarmupScheduler.wrap(inner, 5000, 6000)
    T = 11_000
    assert inner.get_lr(1.0, 100, T) > 0.0
    assert s.get_lr(1.0, 100, T) == 0.0 and s.get_lr(1.0, 5000, T) == 0.0
    assert s.get_lr(1.0, 5500, T) == pytest.approx(0.25 * (1 + alpha))
    assert s.get_lr(1.0, 6000, T) == pytest.approx(0.5 * (1 + alpha))
    assert s.get_lr(1.0, 7000, T) == inner.get_lr(1.0, 7000, T)


def test_cosine_family_and_misc_schedules():
    T = 1000
    c = CosWithWarmup(**BASE, warmup_steps=100, alpha_f=0.1)
    assert c.get_lr(2.0, 100, T) == pytest.approx(2.0)
    assert c.get_lr(2.0, 550, T) == pytest.approx(0.2 + 1.8 * 0.5)
    assert c.get_lr(2.0, T, T) == pytest.approx(0.2)
    c_short = CosWithWarmup(**BASE, warmup_steps=100, alpha_f=0.1, t_max=500)
    assert c_short.get_lr(2.0, 500, T) == pytest.approx(0.2) and c_short.get_lr(2.0, 900, T) == pytest.approx(0.2)
    floor = CosWithWarmup(grad_clip_warmup_steps=None, grad_clip_warmup_factor=None, warmup_min_lr=0.0, warmup_steps=100)
    assert floor.get_lr(1.0, 0, T) == 0.0 and floor.get_lr(1.0, 50, T) == pytest.approx(0.5)

    env = CosLinearEnvelope(**BASE, warmup_steps=0, alpha_f=0.0)
    x = 0.25
    assert env.get_lr(1.0, 250, T) == pytest.approx((1 - x) * (1 + math.cos(math.pi * x)) / 2)
    assert env.get_lr(1.0, T, T) == 0.0

    inv = InvSqrtWithWarmup(**BASE, warmup_steps=100)
    assert inv.get_lr(1.0, 100, T) == pytest.approx(1.0) and inv.get_lr(1.0, 400, T) == pytest.approx(0.5)
    const = ConstantScheduler(**BASE)
    assert const.get_lr(0.3, 12345, T) == 0.3
    cw = ConstantWithWarmupScheduler(**BASE, warmup_steps=10)
    assert cw.get_lr(1.0, 5, T) == pytest.approx(0.1 + 0.9 * 0.5) and cw.get_lr(1.0, 500, T) == 1.0
    mx = MaxScheduler(**BASE, sched1=c, sched2=ConstantScheduler(**BASE))
    assert mx.get_lr(2.0, 900, T) == 2.0


def test_grad_clip_warmup_and_builder():
    s = LinearWithWarmup(grad_clip_warmup_steps=10, grad_clip_warmup_factor=5.0, warmup_min_lr=None, warmup_steps=10)
    assert s.get_max_grad_norm(1.0, 5, 100) == 5.0 and s.get_max_grad_norm(1.0, 11, 100) == 1.0
    assert s.get_max_grad_norm(None, 5, 100) is None
    assert s.get_max_grad_norm_ratio(0.5, 10, 100) == 2.5
    cfg = tiny_config(scheduler=SchedulerConfig(name=SchedulerType.cosine_with_warmup, t_warmup=7, alpha_f=0.2, t_max=70))
    built = build_scheduler(cfg)
    assert isinstance(built, CosWithWarmup) and built.warmup_steps == 7 and built.t_max == 70 and built.alpha_f == 0.2
    for name in SchedulerType:
        sub = SchedulerConfig(name=name, t_warmup=3)
        if name == SchedulerType.max_scheduler:
            continue
        assert build_scheduler(cfg, sub).get_lr(1.0, 50, 100) > 0


# ------------------------------------------------------------------------------------ optimisers


def paired_models(seed=0):
    torch.manual_seed(seed)
    a = nn.Sequential(nn.Linear(8, 16), nn.GELU(), nn.Linear(16, 4))
    b = nn.Sequential(nn.Linear(8, 16), nn.GELU(), nn.Linear(16, 4))
    b.load_state_dict(a.state_dict())
    return a, b


def test_adamw_matches_torch():
    ours_m, ref_m = paired_models()
    ours = AdamW(ours_m.parameters(), lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    ref = torch.optim.AdamW(ref_m.parameters(), lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(5):
        x = torch.randn(32, 8)
        for m, o in ((ours_m, ours), (ref_m, ref)):
            o.zero_grad()
            m(x).pow(2).mean().backward()
            o.step()
    for p, q in zip(ours_m.parameters(), ref_m.parameters()):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
    state = ours.get_state_for_param(next(ours_m.parameters()))
    assert set(state) >= {"exp_avg", "exp_avg_sq"}


def test_adamw_selective_updates_skip_zero_grad_rows():
    torch.manual_seed(0)
    emb = nn.Embedding(10, 4)
    opt = AdamW(emb.parameters(), lr=0.1, weight_decay=0.5, selective_updates=True)
    before = emb.weight.detach().clone()
    emb(torch.tensor([1, 3])).sum().backward()
    opt.step()
    changed = (emb.weight.detach() != before).any(dim=1)
    assert changed.tolist() == [i in (1, 3) for i in range(10)]


def test_lionw_update_rule_and_metrics():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(6, 3))
    opt = LionW([p], lr=0.01, betas=(0.9, 0.99), weight_decay=0.1, record_update_metrics=True)
    opt._collecting_metrics = True
    m = torch.zeros_like(p)
    want = p.detach().clone()
    for _ in range(3):
        g = torch.randn_like(p)
        p.grad = g.clone()
        opt.step()
        update = (0.9 * m + 0.1 * g).sign()
        want = want * (1 - 0.01 * 0.1) - 0.01 * update
        m = 0.99 * m + 0.01 * g
    torch.testing.assert_close(p.detach(), want, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(opt.state[p]["exp_avg"], m, rtol=1e-5, atol=1e-6)
    metrics = opt.get_post_step_metrics(nn.Module())
    assert 0.0 < float(metrics["update_cos_sim"]) <= 1.0


def test_param_groups_follow_decay_flags():
    cfg = tiny_config(optimizer=OptimizerConfig(decay_norm_and_bias=False, decay_embeddings=False))
    model = OLMo(cfg.model)
    groups = get_param_groups(cfg, model)
    assert len(groups) == 2 and groups[1]["weight_decay"] == 0.0
    decay, no_decay = set(groups[0]["param_names"]), set(groups[1]["param_names"])
    assert "transformer.wte.weight" in no_decay
    assert any(n.endswith("attn_norm.weight") for n in no_decay)
    assert any(n.endswith("att_proj.weight") for n in decay) and any(n.endswith("ff_out.weight") for n in decay)
    assert groups[0]["param_names"] == sorted(groups[0]["param_names"])
    assert decay | no_decay == {n for n, _ in model.named_parameters()}

    cfg.optimizer.decay_norm_and_bias = True
    cfg.optimizer.decay_embeddings = True
    groups = get_param_groups(cfg, model)
    assert len(groups) == 1 and len(groups[0]["params"]) == len(list(model.parameters()))


@pytest.mark.parametrize("name", [OptimizerType.adamw, OptimizerType.lionw])
def test_global_clipping_matches_torch_and_reports_metrics(name):
    torch.manual_seed(0)
    cfg = tiny_config(optimizer=OptimizerConfig(name=name, learning_rate=1e-3), max_grad_norm=0.5)
    model = OLMo(cfg.model)
    model.reset_parameters()
    opt = build_optimizer(cfg, model)
    ids = torch.randint(0, 64, (2, 16))
    logits = model(ids).logits
    torch.nn.functional.cross_entropy(logits.view(-1, logits.shape[-1]), ids.view(-1)).backward()
    ref_grads = [p.grad.detach().clone() for p in model.parameters()]
    total = torch.sqrt(sum(g.float().pow(2).sum() for g in ref_grads))
    metrics = opt.clip_grads_and_collect_metrics(global_step=100, collect_param_metrics=True, device=torch.device("cpu"))
    assert float(metrics["total_grad_norm"]) == pytest.approx(float(total), rel=1e-4)
    coef = min(1.0, 0.5 / (float(total) + 1e-6))
    for p, g in zip(model.parameters(), ref_grads):
        torch.testing.assert_close(p.grad, g * coef, rtol=1e-4, atol=1e-7)
    assert float(metrics["clipping_rate"]) == (1.0 if float(total) > 0.5 else 0.0)
    some = "transformer.blocks.0.att_proj.weight"
    for key in (f"grad/{some}.norm", f"param/{some}.norm", f"param/{some}.max", f"param/{some}.min", f"param/{some}.avg"):
        assert key in metrics, key
    slim = opt.clip_grads_and_collect_metrics(global_step=101, collect_param_metrics=False, device=torch.device("cpu"))
    assert "total_grad_norm" in slim and f"param/{some}.norm" not in slim


def test_adaptive_clipping_uses_running_norm():
    torch.manual_seed(0)
    p = nn.Parameter(torch.zeros(4))
    opt = AdamW([{"params": [p], "param_names": ["w"], "max_grad_norm_ratio": 2.0, "max_grad_norm": None, "sharded": False}], lr=0.1)
    p.grad = torch.full((4,), 0.5)  # norm 1
    opt.clip_grads_and_collect_metrics(global_step=2, device=torch.device("cpu"))
    torch.testing.assert_close(p.grad, torch.full((4,), 0.5))  # this step only seeds the average (steps 0 and 1 never do)
    p.grad = torch.full((4,), 5.0)  # norm 10 > 2 x running norm (1)
    opt.clip_grads_and_collect_metrics(global_step=3, device=torch.device("cpu"))
    assert float(p.grad.norm()) == pytest.approx(2.0, rel=1e-3)


def test_state_dict_upgrade_from_single_group():
    cfg = tiny_config(optimizer=OptimizerConfig(decay_norm_and_bias=False))
    model = OLMo(cfg.model)
    opt = build_optimizer(cfg, model)
    assert len(opt.param_groups) == 2
    n = sum(len(g["params"]) for g in opt.param_groups)
    old = {"state": {}, "param_groups": [{"lr": 1.0, "betas": (0.9, 0.95), "eps": 1e-8, "weight_decay": 0.1, "params": list(range(n))}]}
    fixed = fix_optim_state_dict(opt, old)
    assert len(fixed["param_groups"]) == 2 and fixed["param_groups"][1]["weight_decay"] == 0.0
    assert fixed["param_groups"][0]["param_names"] == opt.param_groups[0]["param_names"]
    assert sorted(fixed["param_groups"][0]["params"] + fixed["param_groups"][1]["params"]) == list(range(n))


def test_ten_step_trajectory_matches_torch_adamw_with_clip_grad_norm():
    """A whole training trajectory, not one update: ten steps of this package's AdamW with its own global clipping and
    a warm-up schedule against ``torch.optim.AdamW`` + ``clip_grad_norm_`` on a copy of the model with the same
    decay / no-decay groups (the comparison the reference makes in ``tests/grad_norm_test.py:226-262``)."""
    from copy import deepcopy

    torch.manual_seed(0)
    max_norm, steps = 1.0, 10
    cfg = tiny_config(optimizer=OptimizerConfig(name=OptimizerType.adamw, learning_rate=3e-3, weight_decay=0.1, decay_norm_and_bias=False,
                                                betas=(0.9, 0.95), eps=1e-8),
                      scheduler=SchedulerConfig(name=SchedulerType.linear_with_warmup, t_warmup=4, alpha_f=0.1, **BASE),
                      max_grad_norm=max_norm, max_duration=steps)
    ours = OLMo(cfg.model)
    ours.reset_parameters()
    ours.eval()  # dropout off: the two copies must see the same function
    theirs = deepcopy(ours)
    opt = build_optimizer(cfg, ours)
    sched = build_scheduler(cfg)
    by_name = dict(theirs.named_parameters())
    torch_opt = torch.optim.AdamW(
        [{"params": [by_name[n] for n in g["param_names"]], "weight_decay": g["weight_decay"]} for g in opt.param_groups],
        lr=cfg.optimizer.learning_rate, betas=(0.9, 0.95), eps=1e-8)

    def loss_of(model, ids):
        logits = model(ids).logits[:, :-1]
        return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))

    clipped = 0
    for step in range(1, steps + 1):
        ids = torch.randint(0, 64, (4, 16))
        lr = sched.get_lr(cfg.optimizer.learning_rate, step, steps)
        for group in opt.param_groups:
            group["lr"] = lr
            group["max_grad_norm"] = sched.get_max_grad_norm(max_norm, step, steps)
        for group in torch_opt.param_groups:
            group["lr"] = lr

        opt.zero_grad(set_to_none=True)
        a = loss_of(ours, ids)
        a.backward()
        metrics = opt.clip_grads_and_collect_metrics(global_step=step, device=torch.device("cpu"))
        opt.step()

        torch_opt.zero_grad(set_to_none=True)
        b = loss_of(theirs, ids)
        b.backward()
        norm = torch.nn.utils.clip_grad_norm_(theirs.parameters(), max_norm)
        torch_opt.step()

        clipped += int(float(norm) > max_norm)
        assert a.item() == pytest.approx(b.item(), rel=1e-5), step
        assert float(metrics["total_grad_norm"]) == pytest.approx(float(norm), rel=1e-4), step
        for (name, p), q in zip(ours.named_parameters(), theirs.parameters()):
            torch.testing.assert_close(p, q, rtol=2e-5, atol=2e-6, msg=lambda m: f"step {step}, {name}: {m}")
    assert clipped > 0  # the clipping branch was exercised, not only the pass-through


def test_schedule_shape_properties():
    """Property test of the warm-up + decay schedules: the rate never leaves [floor, peak] after warm-up, rises during
    warm-up, does not rise afterwards, reaches the peak at the end of warm-up and the floor at the horizon and beyond."""
    from hypothesis import given, settings
    from hypothesis import strategies as st

    @settings(max_examples=80, deadline=None)
    @given(kind=st.sampled_from(["cos", "linear"]), warmup=st.integers(0, 50), extra=st.integers(1, 200), alpha=st.floats(0.0, 1.0),
           peak=st.floats(1e-6, 1.0), use_t_max=st.booleans())
    def check(kind, warmup, extra, alpha, peak, use_t_max):
        horizon = warmup + extra
        cls = CosWithWarmup if kind == "cos" else LinearWithWarmup
        sched = cls(warmup_steps=warmup, alpha_f=alpha, t_max=horizon if use_t_max else None, **BASE)
        max_steps = horizon if not use_t_max else horizon + 37  # with t_max the trainer's own horizon must not matter
        rates = [sched.get_lr(peak, s, max_steps) for s in range(horizon + 5)]
        floor = peak * alpha
        tol = 1e-12 + 1e-9 * peak
        assert rates[warmup] == pytest.approx(peak, rel=1e-9)
        assert all(a <= b + tol for a, b in zip(rates[:warmup], rates[1 : warmup + 1]))  # warm-up rises
        assert all(a + tol >= b for a, b in zip(rates[warmup:], rates[warmup + 1 :]))  # decay never rises
        assert all(floor - tol <= r <= peak + tol for r in rates[warmup:])
        assert all(r == pytest.approx(floor, abs=tol) for r in rates[horizon:])
        assert all(0 <= r <= peak + tol for r in rates[:warmup])

    check()
