"""The optimizer kernels against torch's optimizers on the same gradients (B200).

* FusedAdamW (one multi-tensor kernel per group, clip coefficient read on the device) against
  torch.optim.AdamW, three steps, with and without a gradient scale: parameters and both moments
  within rtol 1e-5 / atol 1e-6 (the same fp32 formulas; only operation order differs).
* Muon's fused path (prepare, normalize, tcgen05 Newton-Schulz, apply) against torch.optim.Muon,
  three steps on wide, tall and square matrices: momentum buffers within rtol 1e-6 (identical fp32
  lerps); parameters within 2 % of the accumulated update's norm (the Newton-Schulz GEMMs round
  bf16 products in another order than cuBLAS).
* FusedAdamW resumes a state saved by torch's non-fused AdamW (host step counters) and then
  matches torch's AdamW resumed from the same state.
* MuonAdamW writes the updated bf16 operand caches, which then equal a fresh conversion of the
  fp32 weights bit for bit.
"""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _grads(shapes, steps, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [[torch.randn(s, device="cuda", generator=g) for s in shapes] for _ in range(steps)]


@pytest.mark.parametrize("scaled", [False, True])
def test_fused_adamw_matches_torch_adamw(scaled):
    from tensor_train_ing_b200.optim import FusedAdamW
    shapes = [(257, 129), (4096,), (3,), (64, 64)]
    torch.manual_seed(0)
    base = [torch.randn(s, device="cuda") for s in shapes]
    ours = [b.clone().requires_grad_(True) for b in base]
    ref = [b.clone().requires_grad_(True) for b in base]
    groups = lambda ps: [{"params": ps[:2], "weight_decay": 0.1}, {"params": ps[2:], "weight_decay": 0.0}]
    opt = FusedAdamW(groups(ours), lr=3e-3, betas=(0.9, 0.95))
    topt = torch.optim.AdamW(groups(ref), lr=3e-3, betas=(0.9, 0.95), foreach=False)
    scale = torch.tensor([0.37], device="cuda") if scaled else None
    for grads in _grads(shapes, 3, seed=1):
        for p, q, g in zip(ours, ref, grads):
            p.grad = g.clone()
            q.grad = g * 0.37 if scaled else g.clone()
        opt.step(grad_scale=scale)
        topt.step()
    torch.cuda.synchronize()
    for p, q in zip(ours, ref):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
        for key in ("exp_avg", "exp_avg_sq"):
            torch.testing.assert_close(opt.state[p][key], topt.state[q][key], rtol=1e-5, atol=1e-7)
        assert float(opt.state[p]["step"]) == float(topt.state[q]["step"]) == 3.0
    # the state dict is torch AdamW's: it loads into a torch optimizer unchanged
    torch.optim.AdamW(groups([q.detach().clone().requires_grad_(True) for q in ref]), lr=3e-3).load_state_dict(
        opt.state_dict())


def test_fused_adamw_resumes_a_host_counter_adamw_state():
    """A state saved by torch's default (non-fused) AdamW keeps its step counters on the host; loaded
    into FusedAdamW they move to the device, and the next steps match torch's AdamW resumed from the
    same state."""
    from tensor_train_ing_b200.optim import FusedAdamW
    shapes = [(300, 70), (512,)]
    torch.manual_seed(3)
    base = [torch.randn(s, device="cuda") for s in shapes]
    first = [b.clone().requires_grad_(True) for b in base]
    donor = torch.optim.AdamW([{"params": first, "weight_decay": 0.1}], lr=2e-3, foreach=False)
    grads = _grads(shapes, 4, seed=7)
    for p, g in zip(first, grads[0]):
        p.grad = g.clone()
    donor.step()
    saved = donor.state_dict()
    assert all(st["step"].device.type == "cpu" for st in saved["state"].values())
    ours = [p.detach().clone().requires_grad_(True) for p in first]
    ref = [p.detach().clone().requires_grad_(True) for p in first]
    opt = FusedAdamW([{"params": ours, "weight_decay": 0.1}], lr=2e-3)
    # torch's loader keeps the given state tensors (no copy) where device and dtype already match, so
    # each optimizer loads its own copy instead of both updating the donor's moment tensors
    opt.load_state_dict(copy.deepcopy(saved))
    topt = torch.optim.AdamW([{"params": ref, "weight_decay": 0.1}], lr=2e-3, foreach=False)
    topt.load_state_dict(copy.deepcopy(saved))
    assert all(opt.state[p]["step"].is_cuda for p in ours) and opt.param_groups[0]["fused"] is True
    for step_grads in grads[1:]:
        for p, q, g in zip(ours, ref, step_grads):
            p.grad, q.grad = g.clone(), g.clone()
        opt.step()
        topt.step()
    torch.cuda.synchronize()
    for p, q in zip(ours, ref):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6)
        assert float(opt.state[p]["step"]) == float(topt.state[q]["step"]) == 4.0


@pytest.mark.parametrize("shape", [(256, 1024), (1024, 256), (512, 512)])
def test_fused_muon_matches_torch_muon(shape):
    from tensor_train_ing_b200.optim import Muon
    torch.manual_seed(0)
    p0 = torch.randn(shape, device="cuda") * 0.02
    ours = p0.clone().requires_grad_(True)
    ref = p0.clone().requires_grad_(True)
    kw = dict(lr=0.02, weight_decay=0.1, momentum=0.95, nesterov=True, adjust_lr_fn="match_rms_adamw")
    opt = Muon([ours], **kw)
    topt = torch.optim.Muon([ref], **kw)
    scale = torch.tensor([0.5], device="cuda")
    for (g,) in _grads([shape], 3, seed=2):
        ours.grad = g.clone()
        ref.grad = g * 0.5
        opt.step(grad_scale=scale)
        topt.step()
    torch.cuda.synchronize()
    torch.testing.assert_close(opt.state[ours]["momentum_buffer"], topt.state[ref]["momentum_buffer"],
                               rtol=1e-6, atol=1e-7)
    moved = (ref.detach() - p0).norm()
    assert float((ours.detach() - ref.detach()).norm() / moved) < 2e-2


def test_muon_adamw_writes_current_bf16_caches():
    from tensor_train_ing_b200.config import Config
    from tensor_train_ing_b200.engine import TrainEngine
    from tensor_train_ing_b200.ops.weights import cache_views
    cfg = Config.from_dict({"model": dict(vocab_size=512, padded_vocab=512, d_model=256, layers=2, heads=4, d_key=64,
                                          d_value=64, d_mlp=512, attention="signed_product", mlp="bilinear",
                                          loss_chunk_tokens=128),
                            "train": dict(optimizer="muon", lr=0.02, aux_adamw_lr=3e-3, grad_clip=1.0)})
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cuda", micro_batch=2)
    assert eng.optimizer.accepts_grad_scale
    idx = torch.randint(0, 512, (4, 128))
    for _ in range(2):
        eng.step(idx, torch.zeros_like(idx), torch.roll(idx, -1, 1))
    torch.cuda.synchronize()
    views, groups = cache_views(eng.model)
    assert groups, "the forward built bf16 operand caches"
    named = dict(eng.model.named_parameters())
    checked = 0
    for name, p in named.items():
        view = views.get(id(p))
        if view is not None:
            assert torch.equal(view, p.detach().to(torch.bfloat16)), name
            checked += 1
    assert checked >= 2 * 9
