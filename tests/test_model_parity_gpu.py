"""The fused sm_100a model path against the PyTorch reference path of the same model (GPU)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from tensor_train_ing_b200.config import ModelConfig
from tensor_train_ing_b200.models.model import TensorLM


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def _grad_bound(name, err_ref):
    """Relative gradient error allowed for the fused path.  Weight matrices and norms: twice the
    bf16 reference path's error (at least 3 %).  Per-layer scalars whose gradient is one sum over a
    whole layer -- the attention kind parameters (coef, b: sums of dS over every visible token
    pair) and the spectral gains (gamma: <dW_eff, W> / sigma) -- cancel to small totals, so their
    relative error says little: measured on sandwich_rms / lower_degree_mix, coef 0.05-0.12 off fp64
    on both the module path and the kernel path; on spectral_rms / offset_square, the second
    layer's q1/k1 gamma (true value 5 % of the first layer's) 0.095 off on the PyTorch spectral path
    and 0.23 on the kernel path, 0.063 on the bf16 reference path.  They get three times the
    reference error, at least 25 %."""
    if name.endswith((".attn.coef", ".attn.b", ".gamma")):
        return max(3.0 * err_ref, 0.25)
    return max(2.0 * err_ref, 3e-2)


@pytest.mark.parametrize("kind", ["signed_product", "offset_square", "lower_degree_mix"])
@pytest.mark.parametrize("norm", ["pre_rms", "group_rms", "sandwich_rms", "spectral_rms"])
def test_fused_matches_reference(kind, norm):
    torch.manual_seed(0)
    cfg = ModelConfig(layers=2, d_model=256, heads=2, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                      padded_vocab=1024, attention=kind, normalization=norm, loss_chunk_tokens=256,
                      qk_init_scale=0.5)
    model = TensorLM(cfg).cuda()
    B, T = 2, 160
    idx = torch.randint(0, 1000, (B, T), device="cuda")
    docs = torch.zeros(B, T, dtype=torch.long, device="cuda")
    docs[:, 90:] = 1
    tgt = torch.roll(idx, -1, 1)
    tgt[:, -1] = -100
    _, loss, n = model(idx, docs, tgt, reduction="sum")
    loss.backward()
    grads = {k: p.grad.detach().clone() for k, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    ref_cfg = ModelConfig(**{**cfg.__dict__, "attention_backend": "reference"})
    ref = TensorLM(ref_cfg).cuda()
    ref.load_state_dict(model.state_dict())
    with torch.autocast("cuda", dtype=torch.bfloat16):
        _, loss_r, n_r = ref(idx, docs, tgt, reduction="sum")
    loss_r.backward()
    exact = TensorLM(ref_cfg).cuda().double()
    exact.load_state_dict(model.state_dict())
    _, loss_x, _ = exact(idx, docs, tgt, reduction="sum")
    loss_x.backward()
    assert int(n) == int(n_r)
    assert abs(loss.item() - loss_x.item()) / abs(loss_x.item()) < 1e-2
    ref_grads = dict(ref.named_parameters())
    for k, p in exact.named_parameters():
        if p.grad is None:
            continue
        # the fused bf16 path must be about as close to fp64 as the reference's own bf16 autocast path
        err_fused = rel(grads[k], p.grad)
        err_ref = rel(ref_grads[k].grad, p.grad)
        assert err_fused < _grad_bound(k, err_ref), (k, err_fused, err_ref)


@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_training_steps_follow_reference_path(optimizer):
    """Several optimizer updates through the engine: the fused path's loss trajectory tracks the
    PyTorch reference path of the same weights.  A stale bf16 weight cache (parameters updated
    without the GEMMs seeing it) would leave the fused loss flat while the reference one falls."""
    from tensor_train_ing_b200.config import Config, TrainConfig
    from tensor_train_ing_b200.engine import TrainEngine
    mcfg = ModelConfig(layers=2, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=500,
                       padded_vocab=512, loss_chunk_tokens=256)
    tcfg = TrainConfig(optimizer=optimizer, lr=3e-3 if optimizer == "adamw" else 0.02, aux_adamw_lr=3e-3,
                       grad_clip=1.0)
    losses = {}
    for name in ("fused", "reference"):
        torch.manual_seed(0)
        model = TensorLM(mcfg).cuda()
        if name == "reference":
            model._force_reference = True  # module-level PyTorch math, fp32
        eng = TrainEngine(Config(model=mcfg, train=tcfg), device="cuda", micro_batch=2, model=model)
        g = torch.Generator().manual_seed(1)
        idx = torch.randint(0, 500, (4, 128), generator=g)  # one batch, repeated: the loss must fall
        doc = torch.zeros_like(idx)
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -100
        out = []
        for _ in range(6):
            loss, count = eng.step(idx, doc, tgt)
            out.append(float(loss) / float(count))
        losses[name] = out
    f, r = losses["fused"], losses["reference"]
    assert r[-1] < 0.9 * r[0], r  # the test only means something if training moves the loss
    for a, b in zip(f, r):
        assert abs(a - b) < 3e-2 * abs(b), (f, r)


def _norm_modules(model, cls):
    return [m for m in model.modules() if isinstance(m, cls)]


@pytest.mark.parametrize("case", ["branch_rms", "lagged", "taper_warmup", "taper_frozen"])
def test_norm_variant_packages_match_reference(case):
    """The lagged, taper and branch-output norms on their fused kernels against the module path:
    loss, every gradient (as close to fp64 as the bf16 reference path), lagged and TaperNorm
    statistics, and the TaperNorm anchor term with its gradient."""
    from tensor_train_ing_b200.models.normalization import LaggedRMS, TaperRMS, taper_anchor_loss
    torch.manual_seed(0)
    norm = {"taper_warmup": "taper", "taper_frozen": "taper"}.get(case, case)
    final = {"lagged": "lagged", "taper": "taper"}.get(norm)  # the packages require their final norm
    extra = {"final_normalization": final} if final else {}
    cfg = ModelConfig(layers=2, d_model=256, heads=2, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                      padded_vocab=1024, attention="signed_product", normalization=norm, loss_chunk_tokens=256,
                      qk_init_scale=0.5, **extra)
    B, T = 2, 160
    idx = torch.randint(0, 1000, (B, T), device="cuda")
    docs = torch.zeros(B, T, dtype=torch.long, device="cuda")
    docs[:, 90:] = 1
    tgt = torch.roll(idx, -1, 1)
    tgt[:, -1] = -100
    valid = (tgt != -100).to(torch.float32)

    def prepare(model):
        with torch.no_grad():
            for i, m in enumerate(_norm_modules(model, LaggedRMS)):
                m.mean_sq.fill_(2.5 + i)
                m.calibrated.fill_(True)
                m.collecting = True
                m.set_valid_mask(valid)
            for i, m in enumerate(_norm_modules(model, TaperRMS)):
                m.set_valid_mask(valid)
                if case == "taper_warmup":
                    m.collecting = True
                else:
                    m.frozen.fill_(True)
                    m.gate.fill_(0.4)
                    m.c.fill_(0.8 + 0.05 * i)
                    m.s_tgt.fill_(1.3)
                    m.weight_tilde.copy_(1.1 * m.weight)  # idempotent: prepare runs after load_state_dict too
        return model

    def run(model, autocast):
        model.train()
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            _, loss, _ = model(idx, docs, tgt, reduction="sum")
        anchor = taper_anchor_loss(model)
        total = loss + (50.0 * anchor if anchor is not None else 0.0)
        total.backward()
        return loss.detach(), (anchor.detach() if anchor is not None else None)

    model = prepare(TensorLM(cfg).cuda())
    state = model.state_dict()
    loss, anchor = run(model, False)
    grads = {k: p.grad.detach().clone() for k, p in model.named_parameters() if p.grad is not None}
    ref_cfg = ModelConfig(**{**cfg.__dict__, "attention_backend": "reference"})
    ref = TensorLM(ref_cfg).cuda()
    ref.load_state_dict(state)
    prepare(ref)
    _, anchor_r = run(ref, True)
    exact = TensorLM(ref_cfg).cuda().double()
    exact.load_state_dict(state)
    prepare(exact)
    loss_x, anchor_x = run(exact, False)
    assert abs(loss.item() - loss_x.item()) / abs(loss_x.item()) < 1e-2
    if anchor_x is not None:
        # (r - s_tgt)^2 magnifies the bf16 paths' ~0.4 % activation error in the later layers: the
        # fused anchor must be as close to fp64 as the bf16 reference path's
        dev_ref = abs(anchor_r.item() - anchor_x.item())
        assert abs(anchor.item() - anchor_x.item()) < max(2.0 * dev_ref, 1e-3 * abs(anchor_x.item()))
    ref_grads = dict(ref.named_parameters())
    for k, p in exact.named_parameters():
        if p.grad is None:
            continue
        assert k in grads, k
        err_fused = rel(grads[k], p.grad)
        err_ref = rel(ref_grads[k].grad, p.grad)
        assert err_fused < _grad_bound(k, err_ref), (k, err_fused, err_ref)
    for fm, xm in zip(_norm_modules(model, LaggedRMS), _norm_modules(exact, LaggedRMS)):
        assert float(fm.acc_count) == float(xm.acc_count) > 0
        assert abs(float(fm.acc_sum) - float(xm.acc_sum)) <= 1e-3 * abs(float(xm.acc_sum))
    for fm, xm in zip(_norm_modules(model, TaperRMS), _norm_modules(exact, TaperRMS)):
        for name in ("acc_num", "acc_den", "acc_r", "acc_count"):
            a, b = float(getattr(fm, name)), float(getattr(xm, name))
            # activations of the later layers carry the bf16 path's rounding
            assert abs(a - b) <= 1e-3 * max(abs(b), 1e-12), (name, a, b)


@pytest.mark.parametrize("kind", ["signed_product", "offset_square"])
@pytest.mark.parametrize("dk", [64, 128])
def test_score_bounds_from_the_qkv_epilogue(kind, dk):
    """The per-head score bound max|q| max|k| / sqrt(dk) recorded by the fused path (row norms from
    the QKV GEMM's RoPE epilogue) agrees with the bound the reference path computes from its own
    bf16 q and k on the same weights."""
    from tensor_train_ing_b200.qk_clip import set_score_bound_recording
    torch.manual_seed(0)
    cfg = ModelConfig(layers=2, d_model=256, heads=2, d_key=dk, d_value=dk, d_mlp=512, vocab_size=1000,
                      padded_vocab=1024, attention=kind, qk_init_scale=0.5)
    model = TensorLM(cfg).cuda().eval()
    ref = TensorLM(ModelConfig(**{**cfg.__dict__, "attention_backend": "reference"})).cuda().eval()
    ref.load_state_dict(model.state_dict())
    idx = torch.randint(0, 1000, (2, 300), device="cuda")
    docs = torch.zeros(2, 300, dtype=torch.long, device="cuda")
    docs[:, 170:] = 1
    for m in (model, ref):
        set_score_bound_recording(m, True)
    with torch.no_grad():
        model(idx, docs)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            ref(idx, docs)
    for blk, rblk in zip(model.blocks, ref.blocks):
        got, want = blk.attn.last_score_bound, rblk.attn.last_score_bound
        assert set(got) == set(want) == ({"S1", "S2"} if kind == "signed_product" else {"S1"})
        for name in got:
            assert got[name].shape == (2,) and bool((got[name] > 0).all())
            torch.testing.assert_close(got[name], want[name].float(), rtol=2e-2, atol=1e-4)


def test_batch_score_bounds_and_clip_on_the_fused_path():
    """The trainer's batch-bound bookkeeping on CUDA: the update's maximum spans both micro-batches,
    the clip uses the last one's per-head bounds (2 layers x 2 factors x 2 heads over tau), and after
    the clip a re-run of that micro-batch records bounds at tau (the rescale multiplies each clipped
    head's scores by tau / bound; bf16 operands round the re-run's norms)."""
    from tensor_train_ing_b200.config import Config, TrainConfig
    from tensor_train_ing_b200.training_stability import BatchScoreBounds
    torch.manual_seed(0)
    mcfg = ModelConfig(layers=2, d_model=256, heads=2, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                       padded_vocab=1024, attention="signed_product", qk_init_scale=0.5)
    cfg = Config(model=mcfg, train=TrainConfig(qk_clip_source="batch_bound", qk_clip_tau=1e-3,
                                               qk_clip_every_steps=1), raw={})
    model = TensorLM(mcfg).cuda().eval()
    bounds = BatchScoreBounds(model, cfg)
    docs = torch.zeros(2, 256, dtype=torch.long, device="cuda")
    batches = [torch.randint(0, 1000, (2, 256), device="cuda") for _ in range(2)]
    bounds.begin_update()
    seen = []
    with torch.no_grad():
        for idx in batches:
            model(idx, docs)
            bounds.observe()
            seen.append(max(float(b.max()) for layer in bounds.last for b in layer.values()))
    assert bounds.finish_update() == pytest.approx(max(seen), rel=1e-6)
    report = bounds.clip(1e-3)
    assert report["clipped_heads"] == 8 and report["max_bound_before"] == pytest.approx(seen[-1], rel=1e-6)
    bounds.begin_update()
    with torch.no_grad():
        model(batches[-1], docs)
    bounds.observe()
    assert bounds.finish_update() <= 1e-3 * (1 + 2e-2)  # bf16 operands: the re-run's norms round


def test_selective_recompute_on_the_fused_path_keeps_every_gradient():
    """Activation checkpointing on the fused path: recomputing all, some or none of the blocks gives
    bit-identical gradients (the recomputed forward runs the same kernels on the same inputs)."""
    from tensor_train_ing_b200.config import ModelConfig
    from tensor_train_ing_b200.models.model import TensorLM
    cfg = ModelConfig(layers=3, d_model=256, heads=4, d_key=64, d_value=64, d_mlp=512, vocab_size=1000,
                      padded_vocab=1024, loss_chunk_tokens=512, activation_checkpointing=True)
    torch.manual_seed(0)
    model = TensorLM(cfg).cuda()
    g = torch.Generator().manual_seed(2)
    idx = torch.randint(0, 1000, (2, 256), generator=g).cuda()
    doc = torch.zeros_like(idx)
    doc[:, 100:] = 1
    tgt = torch.roll(idx, -1, 1)
    grads = []
    for recompute in (None, 2, 0):
        model.recompute_blocks = recompute
        model.zero_grad(set_to_none=True)
        assert model.recomputed_blocks() == (3 if recompute is None else recompute)
        _, loss, _ = model(idx, doc, tgt, reduction="sum")
        loss.backward()
        grads.append({n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None})
    torch.cuda.synchronize()
    for other in grads[1:]:
        assert other.keys() == grads[0].keys()
        for n in grads[0]:
            assert torch.equal(grads[0][n], other[n]), n
