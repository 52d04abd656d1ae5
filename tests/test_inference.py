"""4-bit inference side product: packing, C++ CPU reference, GPTQ vs round-to-nearest, whole-model quantisation,
quantised checkpoint round trip, stdin/stdout predictor, and (on a GPU) the sm_100a kernels against the CPU reference."""
import io
import json

import pytest
import torch
import torch.nn as nn

from olmo_b200.config import ModelConfig, TokenizerConfig, TrainConfig
from olmo_b200.inference import QuantLinear, gptq_quantize_weight, pack_int4, quantize_model, unpack_int4
from olmo_b200.inference import cpu_ref
from olmo_b200.inference.efficiency import Predictor, load_quantized, run_quantization, stdio_predictor_wrapper
from olmo_b200.inference.quantize import quantized_state_summary
from olmo_b200.models.olmo import OLMo


def manual_dequant(layer: QuantLinear) -> torch.Tensor:
    q = unpack_int4(layer.qweight).float().reshape(layer.out_features, -1, layer.group)
    return ((q - layer.zeros.float().unsqueeze(-1)) * layer.scales.float().unsqueeze(-1)).reshape(layer.out_features, layer.in_features)


def test_pack_unpack_and_cpu_reference():
    torch.manual_seed(0)
    q = torch.randint(0, 16, (7, 128))
    packed = pack_int4(q)
    assert packed.dtype == torch.int32 and packed.shape == (7, 16)
    assert torch.equal(unpack_int4(packed).long(), q)
    assert int(packed[0, 0]) == int(sum(int(q[0, i]) << (4 * i) for i in range(8)) - (2**32 if q[0, 7] >= 8 else 0))

    lin = nn.Linear(128, 24, bias=True)
    layer = QuantLinear.from_linear_rtn(lin, group=32)
    W = manual_dequant(layer)
    torch.testing.assert_close(cpu_ref.dequant(layer.qweight, layer.scales.float(), layer.zeros, 32), W)
    x = torch.randn(3, 5, 128)
    want = x @ W.t() + layer.bias.float()
    torch.testing.assert_close(layer(x), want, rtol=1e-4, atol=1e-4)
    # 4-bit grid: the reconstruction error stays within one quantisation step of the weight's group (half a step of
    # rounding plus what the bf16-rounded scale clips at the ends of the range)
    step = layer.scales.float().repeat_interleave(32, dim=1)
    err = (W - lin.weight.detach()).abs()
    assert bool((err <= step + 1e-6).all()) and float((err <= 0.5 * step + 1e-6).float().mean()) > 0.9
    with pytest.raises(ValueError):
        cpu_ref.dequant(layer.qweight, layer.scales.float(), layer.zeros, 48)  # group does not divide K


def test_activation_order_permutation_is_applied_to_inputs():
    torch.manual_seed(1)
    q = torch.randint(0, 16, (8, 64))
    scales, zeros = torch.rand(8, 2) + 0.5, torch.randint(0, 16, (8, 2))
    perm = torch.randperm(64)
    layer = QuantLinear.from_quantized(q, scales, zeros, 32, perm=perm)
    W_stored = manual_dequant(layer)
    x = torch.randn(4, 64)
    torch.testing.assert_close(layer(x), x[:, perm] @ W_stored.t(), rtol=1e-4, atol=1e-4)


def test_gptq_beats_round_to_nearest_on_correlated_inputs():
    torch.manual_seed(0)
    lin = nn.Linear(256, 64, bias=False)
    X = torch.randn(4096, 256) @ (torch.randn(256, 256) * 0.1)
    H = X.t() @ X
    want = lin(X).detach()

    def rel(layer):
        return float((layer(X) - want).norm() / want.norm())

    rtn = QuantLinear.from_linear_rtn(lin, group=64)
    errs = {}
    for act_order in (False, True):
        Q, s, z, perm = gptq_quantize_weight(lin.weight, H, group=64, act_order=act_order)
        assert Q.min() >= 0 and Q.max() <= 15 and (perm is None) == (not act_order)
        errs[act_order] = rel(QuantLinear.from_quantized(Q, s, z, 64, perm=perm))
    assert errs[False] < rel(rtn) and errs[True] < rel(rtn)
    # dead input columns (never active) are handled
    H2 = H.clone()
    H2[5, :] = 0
    H2[:, 5] = 0
    Q, s, z, perm = gptq_quantize_weight(lin.weight, H2, group=64, act_order=True)
    assert torch.isfinite(s).all()


def tiny_model():
    torch.manual_seed(0)
    cfg = ModelConfig(d_model=128, n_heads=4, n_layers=2, mlp_hidden_size=512, vocab_size=96, embedding_size=128, max_sequence_length=64,
                      weight_tying=False, include_bias=False, rope=True, flash_attention=False, layer_norm_type="rms", layer_norm_with_affine=True,
                      attention_layer_norm=True, norm_after=True, eos_token_id=95, pad_token_id=94, init_device="cpu", init_std=0.08)
    m = OLMo(cfg)
    m.reset_parameters()
    return m.eval()


@pytest.mark.parametrize("method", ["rtn", "gptq"])
def test_quantize_whole_model_keeps_predictions_close(method):
    model = tiny_model()
    calib = [torch.randint(0, 94, (4, 32)) for _ in range(4)]
    ids = torch.randint(0, 94, (2, 24))
    with torch.no_grad():
        before = model(ids).logits.log_softmax(-1)
    report = quantize_model(model, calib, group=64, method=method)
    assert len(report) == 8 and all(0 <= v < 0.35 for v in report.values()), report
    assert all(isinstance(getattr(b, n), QuantLinear) for b in model.all_blocks() for n in ("att_proj", "attn_out", "ff_proj", "ff_out"))
    with torch.no_grad():
        after = model(ids).logits.log_softmax(-1)
    kl = float((before.exp() * (before - after)).sum(-1).mean())
    assert kl < 0.05, kl
    summary = quantized_state_summary(model)
    assert summary["quantized_bytes"] < 0.2 * (2 * (3 * 128 * 128 + 128 * 128 + 128 * 512 + 256 * 128) * 4)
    out = model.generate(ids, max_steps=3, beam_size=1)  # KV-cache decoding through the quantised layers
    assert out.token_ids.shape[:2] == (2, 1)


def test_quantised_checkpoint_round_trip_and_stdio_predictor(tmp_path):
    tokenizers = pytest.importorskip("tokenizers")
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit

    vocab = {f"t{i}": i for i in range(94)}
    vocab["<pad>"], vocab["<eos>"] = 94, 95
    tok = tokenizers.Tokenizer(WordLevel(vocab, unk_token="t0"))
    tok.pre_tokenizer = WhitespaceSplit()
    tok.add_special_tokens(["<pad>", "<eos>"])
    tok.save(str(tmp_path / "tok.json"))

    model = tiny_model()
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    TrainConfig(model=model.config, tokenizer=TokenizerConfig(identifier=str(tmp_path / "tok.json"))).save(ckpt / "config.yaml")
    torch.save(model.state_dict(), ckpt / "model.pt")
    out = run_quantization(str(ckpt), str(tmp_path / "q"), [torch.randint(0, 94, (2, 16))], group=64, method="gptq")
    loaded = load_quantized(str(out))
    ids = torch.randint(0, 94, (1, 12))
    reference = OLMo.from_checkpoint(str(ckpt))
    quantize_model(reference, [torch.randint(0, 94, (2, 16))], group=64, method="rtn")
    with torch.no_grad():
        a = loaded(ids).logits
    assert a.shape == (1, 12, 128) and torch.isfinite(a).all()
    assert any(isinstance(m, QuantLinear) and m.perm is not None for m in loaded.modules())

    from olmo_b200.tokenizer import Tokenizer

    predictor = Predictor(loaded, Tokenizer.from_checkpoint(str(out)), max_new_tokens=4)
    stdin = io.StringIO(json.dumps(["t1 t2 t3", "t4"]) + "\n\n" + json.dumps(["t5 t6"]) + "\n")
    stdout = io.StringIO()
    assert stdio_predictor_wrapper(predictor, stdin, stdout) == 2
    lines = [json.loads(x) for x in stdout.getvalue().splitlines()]
    assert len(lines) == 2 and len(lines[0]) == 2 and len(lines[1]) == 1 and all(isinstance(s, str) for s in lines[0])

    # stop strings cut a continuation; next-token predictions agree with the logits
    free = list(Predictor(loaded, predictor.tokenizer, max_new_tokens=4).predict(["t1 t2 t3"]))[0]
    words = free.split()
    if len(words) > 1:
        cut = list(Predictor(loaded, predictor.tokenizer, max_new_tokens=4, stop_sequences=[words[1]]).predict(["t1 t2 t3"]))[0]
        assert cut == words[0]
    picks, probs = predictor.next_token_predictions(["t1 t2 t3", "t4"], candidate_token_ids=[5, 6, 7, 8])
    with torch.no_grad():
        direct = loaded(torch.tensor([[1, 2, 3]])).logits[0, -1, [5, 6, 7, 8]]
    assert picks[0] == int(direct.argmax()) and len(probs) == 2 and abs(sum(probs[0]) - 1.0) > 0 and len(probs[0]) == 4


def _grad_case(act_order: bool, M: int = 5, N: int = 24, K: int = 64, G: int = 32):
    torch.manual_seed(3)
    q = torch.randint(0, 16, (N, K))
    scales = (torch.rand(N, K // G) * 0.2 + 0.05).to(torch.bfloat16).float()
    zeros = torch.randint(0, 16, (N, K // G))
    perm = torch.randperm(K) if act_order else None
    layer = QuantLinear.from_quantized(q, scales, zeros, G, perm=perm, bias=torch.randn(N))
    x = torch.randn(2, M, K)
    dy = torch.randn(2, M, N)
    w_stored = manual_dequant(layer)
    xr = x.clone().requires_grad_(True)
    cols = xr if perm is None else xr[..., perm]
    ((cols @ w_stored.t() + layer.bias) * dy).sum().backward()
    return layer, x, dy, xr.grad


@pytest.mark.parametrize("act_order", [False, True])
def test_input_gradient_through_quantised_weights_cpu(act_order):
    layer, x, dy, want = _grad_case(act_order)
    xg = x.clone().requires_grad_(True)
    y = layer(xg)
    assert y.requires_grad and y.shape == dy.shape
    (y * dy).sum().backward()
    torch.testing.assert_close(xg.grad, want, rtol=1e-4, atol=1e-4)
    with torch.no_grad():
        assert not layer(xg).requires_grad


@pytest.mark.gpu
@pytest.mark.parametrize("act_order", [False, True])
def test_input_gradient_through_quantised_weights_gpu(act_order):
    layer, x, dy, want = _grad_case(act_order, M=100, N=256, K=512, G=128)
    layer = layer.cuda()
    xg = x.cuda().to(torch.bfloat16).requires_grad_(True)
    (layer(xg) * dy.cuda().to(torch.bfloat16)).sum().backward()
    ref = want.to(torch.bfloat16).float()
    err = (xg.grad.float().cpu() - ref).abs().max().item()
    assert err <= 3e-2 * ref.abs().max().item() + 1e-3, err  # bf16 inputs, bf16 reconstructed weights, fp32 accumulation


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 64])
@pytest.mark.parametrize("act_order", [False, True])
def test_gpu_kernels_match_cpu_reference(M, act_order):
    torch.manual_seed(0)
    N, K, G = 384, 1024, 128
    q = torch.randint(0, 16, (N, K))
    scales = (torch.rand(N, K // G) * 0.02 + 0.005).to(torch.bfloat16).float()
    zeros = torch.randint(0, 16, (N, K // G))
    perm = torch.randperm(K) if act_order else None
    layer = QuantLinear.from_quantized(q, scales, zeros, G, perm=perm)
    x = torch.randn(M, K).to(torch.bfloat16)
    want = cpu_ref.matmul(x.float(), layer.qweight, layer.scales.float(), layer.zeros, G, layer.perm)
    import copy

    dev = copy.deepcopy(layer).to("cuda")  # Module.to moves in place; keep the host copy for the reference
    got = dev(x.cuda()).float().cpu()
    torch.testing.assert_close(got, want, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dev.dequantize().float().cpu(), cpu_ref.dequant(layer.qweight, layer.scales.float(), layer.zeros, G), rtol=1e-2, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [9, 32, 33, 100, 256])
@pytest.mark.parametrize("N,K,G", [(384, 1024, 128), (1152, 704, 64), (128, 4096, 128)])
def test_fused_dequant_tensor_core_gemm_matches_cpu_reference(M, N, K, G):
    """Decode-batch path (9..256 rows): dequantisation fused into a tcgen05 GEMM.  Checked against the C++ CPU int4
    reference and against the reconstruct-then-multiply path on the device; rows beyond M must stay untouched."""
    from olmo_b200 import ops

    torch.manual_seed(1)
    q = torch.randint(0, 16, (N, K))
    scales = (torch.rand(N, K // G) * 0.02 + 0.005).to(torch.bfloat16).float()
    zeros = torch.randint(0, 16, (N, K // G))
    layer = QuantLinear.from_quantized(q, scales, zeros, G)
    x = torch.randn(M, K).to(torch.bfloat16)
    want = cpu_ref.matmul(x.float(), layer.qweight, layer.scales.float(), layer.zeros, G, None)
    import copy

    dev = copy.deepcopy(layer).to("cuda")
    lib = ops.lib()
    assert lib.ob_w4a16_gemm_small_supported(M, N, K, G) == 1
    xd = x.cuda()
    sentinel = -7.0
    y = torch.full((M + 3, N), sentinel, dtype=torch.bfloat16, device="cuda")  # three guard rows
    ops.check(lib.ob_w4a16_gemm_small(ops.ptr(xd), ops.ptr(dev.qweight), ops.ptr(dev.scales), ops.ptr(dev.zeros), ops.ptr(y), None, M, N, K, G,
                                      1, ops.ptr(ops.status_tensor(xd.device)), ops.stream_ptr()), "ob_w4a16_gemm_small")
    ops.check_status()
    assert bool((y[M:] == sentinel).all())
    # the same product with K split over several CTAs that add into an fp32 buffer (guard rows again)
    k_blocks = K // 64
    for splits in sorted({2, max(1, k_blocks // 8), lib.ob_w4a16_gemm_small_splits(N, K)} - {1}):
        per = -(-k_blocks // splits)
        if -(-k_blocks // per) != splits:
            continue
        partial = torch.zeros(M + 3, N, dtype=torch.float32, device="cuda")
        partial[M:] = sentinel
        ops.check(lib.ob_w4a16_gemm_small(ops.ptr(xd), ops.ptr(dev.qweight), ops.ptr(dev.scales), ops.ptr(dev.zeros), None, ops.ptr(partial),
                                          M, N, K, G, splits, ops.ptr(ops.status_tensor(xd.device)), ops.stream_ptr()), "ob_w4a16_gemm_small")
        ops.check_status()
        assert bool((partial[M:] == sentinel).all())
        torch.testing.assert_close(partial[:M].cpu(), want, rtol=2e-2, atol=6e-2)
    torch.testing.assert_close(y[:M].float().cpu(), want, rtol=2e-2, atol=6e-2)  # outputs reach ±16: half a bf16 step is 0.03
    via_matrix = (xd.float() @ dev.dequantize().float().t()).cpu()
    torch.testing.assert_close(y[:M].float().cpu(), via_matrix, rtol=1e-2, atol=2e-2)
    # the module takes the same kernel for this batch size (with its own choice of K splits, hence not bit-identical)
    torch.testing.assert_close(dev(xd).float().cpu(), y[:M].float().cpu(), rtol=1e-2, atol=6e-2)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_bit_stream_packing_round_trips_and_cpu_layer_matches_dense(bits):
    from olmo_b200.inference.wna16 import BitsLinear, pack_bits, quantize_groups_bits, unpack_bits

    torch.manual_seed(bits)
    q = torch.randint(0, 2**bits, (5, 96))
    packed = pack_bits(q, bits)
    assert packed.shape == (5, 96 * bits // 32) and packed.dtype == torch.int32
    assert torch.equal(unpack_bits(packed, bits).long(), q)
    lin = torch.nn.Linear(128, 24, bias=True)
    layer = BitsLinear.from_linear_rtn(lin, bits, group=32)
    qq, scales, zeros = quantize_groups_bits(lin.weight.detach(), 32, bits)
    dense = ((qq.float().reshape(24, 4, 32) - zeros.unsqueeze(-1)) * scales.to(torch.bfloat16).float().unsqueeze(-1)).reshape(24, 128)
    torch.testing.assert_close(layer.dequantize(), dense, rtol=0, atol=1e-6)
    x = torch.randn(3, 128)
    torch.testing.assert_close(layer(x), x @ dense.t() + lin.bias, rtol=1e-4, atol=1e-4)
    if bits == 8:  # fine grids reproduce the dense layer closely
        assert (layer(x) - lin(x)).abs().max() < 0.05


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("rows", [1, 5, 8, 19, 100])
def test_bit_width_kernels_match_the_fp32_reference(bits, rows):
    """GEMV and reconstruct kernels for every width against the same layer evaluated with plain fp32 tensor ops."""
    from olmo_b200.inference.wna16 import BitsLinear

    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 384, bias=False)
    cpu_layer = BitsLinear.from_linear_rtn(lin, bits, group=128)
    gpu_layer = BitsLinear.from_linear_rtn(lin, bits, group=128).cuda()
    ref_w = cpu_layer.dequantize()
    got_w = gpu_layer.dequantize().float().cpu()
    assert (got_w - ref_w).abs().max() <= 2.0 ** -8 * ref_w.abs().max() + 1e-6  # bf16 rounding of the reconstructed weights
    x = torch.randn(rows, 512).to(torch.bfloat16)
    ref = x.float() @ ref_w.t()
    got = gpu_layer(x.cuda()).float().cpu()
    assert (got - ref).abs().max() <= 2e-2 * ref.abs().max() + 1e-3
