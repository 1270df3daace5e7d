"""GPU parity of the training step's AdamW kernels.

* ``nvfp4b200_adamw_step`` (bf16 parameter, fp32 moments) and
  ``nvfp4b200_adamw_master_step`` (fp32 master copy) against the float32
  oracle (oracle/adamw_oracle.py): bit-exact m, v, master and bf16 parameter,
  over odd lengths (vector body + scalar tail), bf16 and fp32 gradients,
  weight decay and a gradient scale, several steps in a row.
* The master variant against torch.optim.AdamW on fp32 parameters, at a
  learning rate whose per-step change is below half a bf16 ulp of the
  weights: the master tracks torch (relative 1e-5) while the bf16-only
  update leaves the weights where they started.
"""
import numpy as np
import pytest
import torch

from oracle import adamw_oracle, nvfp4_oracle as orc

pytestmark = pytest.mark.gpu
HP = dict(lr=3e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("n", [1, 7, 8, 1001, 65536 + 13])
@pytest.mark.parametrize("grad_dtype", [torch.bfloat16, torch.float32])
def test_adamw_bf16_param_bit_exact(pkg, n, grad_dtype):
    gen = torch.Generator(device="cuda").manual_seed(n)
    p = torch.randn(n, device="cuda", generator=gen).to(torch.bfloat16)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    op, om, ov = bits(p), f32(m), f32(v)
    for step in range(1, 4):
        g = (torch.randn(n, device="cuda", generator=gen) * 0.1).to(grad_dtype)
        pkg.ops.adamw_step(p, g, m, v, step=step, grad_scale=0.5, **HP)
        gh = bits(g) if grad_dtype == torch.bfloat16 else f32(g)
        op, om, ov = adamw_oracle.adamw_bf16(op, gh, om, ov, step=step, grad_scale=0.5, **HP)
        torch.cuda.synchronize()
        assert np.array_equal(f32(m).view(np.uint32), om.view(np.uint32)), step
        assert np.array_equal(f32(v).view(np.uint32), ov.view(np.uint32)), step
        assert np.array_equal(bits(p), op), step


@pytest.mark.parametrize("n", [1, 7, 8, 1001, 65536 + 13])
@pytest.mark.parametrize("grad_dtype", [torch.bfloat16, torch.float32])
def test_adamw_master_bit_exact(pkg, n, grad_dtype):
    gen = torch.Generator(device="cuda").manual_seed(100 + n)
    w = torch.randn(n, device="cuda", generator=gen)
    p = w.to(torch.bfloat16)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    ow, om, ov = f32(w), f32(m), f32(v)
    for step in range(1, 4):
        g = (torch.randn(n, device="cuda", generator=gen) * 0.1).to(grad_dtype)
        pkg.ops.adamw_master_step(p, w, g, m, v, step=step, grad_scale=0.25, **HP)
        gh = bits(g) if grad_dtype == torch.bfloat16 else f32(g)
        ow, om, ov, op = adamw_oracle.adamw_master(ow, gh, om, ov, step=step, grad_scale=0.25, **HP)
        torch.cuda.synchronize()
        assert np.array_equal(f32(w).view(np.uint32), ow.view(np.uint32)), step
        assert np.array_equal(f32(m).view(np.uint32), om.view(np.uint32)), step
        assert np.array_equal(f32(v).view(np.uint32), ov.view(np.uint32)), step
        assert np.array_equal(bits(p), op), step


def test_adamw_master_tracks_torch_adamw_below_bf16_resolution(pkg):
    """lr = 1e-4 on weights in [1, 1.5]: one AdamW step (~1e-4) is far
    below half a bf16 ulp (2^-8 in [1, 2)).  The master update must follow
    torch.optim.AdamW on fp32 parameters; the bf16-only update cannot move."""
    n = 4096 + 5
    hp = dict(lr=1e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.0)
    gen = torch.Generator(device="cuda").manual_seed(7)
    w0 = (1.0 + 0.5 * torch.rand(n, device="cuda", generator=gen)).to(torch.bfloat16).float()
    ref = w0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=hp["lr"], betas=(hp["beta1"], hp["beta2"]), eps=hp["eps"],
                            weight_decay=hp["weight_decay"])
    w = w0.clone()
    p = w0.to(torch.bfloat16)
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    p_plain = w0.to(torch.bfloat16)
    m2, v2 = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    bias = torch.randn(n, device="cuda", generator=gen)        # a consistent gradient direction
    for step in range(1, 81):
        g = bias + 0.1 * torch.randn(n, device="cuda", generator=gen)
        ref.grad = g.clone()
        opt.step()
        pkg.ops.adamw_master_step(p, w, g, m, v, step=step, **hp)
        pkg.ops.adamw_step(p_plain, g, m2, v2, step=step, **hp)
    torch.cuda.synchronize()
    moved = (ref.detach() - w0).abs()
    assert moved.max().item() > 6e-3                          # torch moved the weights by ~80 lr
    err = (w - ref.detach()).abs() / ref.detach().abs()
    assert err.max().item() < 1e-5
    assert torch.equal(p.view(torch.int16), w.to(torch.bfloat16).view(torch.int16))
    assert (p.float() != w0).any()                           # the accumulated change reached bf16
    assert torch.equal(p_plain.float(), w0)                  # each bf16-only step was rounded away


def test_trainer_keeps_master_weights(pkg):
    """The stack trainer's default AdamW keeps fp32 masters: after a step the
    bf16 parameters equal the masters rounded to bf16."""
    import importlib
    mlp = importlib.import_module("nvfp4_b200.mlp")
    t, d, f = 256, 256, 512
    gen = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(t, d, device="cuda", generator=gen).to(torch.bfloat16)
    dy = (1e-3 * torch.randn(t, d, device="cuda", generator=gen)).to(torch.bfloat16)
    tr = mlp.NVFP4MLPStackTrainer(1, d, f, seed=3, micro_tokens=256, max_local_tokens=t)
    b = tr.blocks[0]
    assert b.master is not None and b.master.dtype == torch.float32
    tr.step(x, dy)
    tr.step(x, dy)
    torch.cuda.synchronize()
    assert torch.equal(b.param.view(torch.int16), b.master.to(torch.bfloat16).view(torch.int16))
    # the next step's weight global scales come from the update's amax: exactly the weights' own
    assert torch.equal(tr.w_g[0, 0:1], pkg.ops.global_scale(b.w_gu))
    assert torch.equal(tr.w_g[0, 1:2], pkg.ops.global_scale(b.w_down))
    assert pkg.ops.device_error() == 0


def test_adamw_master_amax_and_scale_from_amax(pkg):
    """The master kernel's amax output equals the max |bf16 parameter| it
    wrote (odd length: vector body and scalar tail, the maximum in the tail),
    and nvfp4b200_global_scale_from_amax reproduces nvfp4b200_global_scale."""
    n = 1000 + 3
    gen = torch.Generator(device="cuda").manual_seed(33)
    w = torch.randn(n, device="cuda", generator=gen)
    w[-2] = -7.5
    p = w.to(torch.bfloat16)
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    g = (0.1 * torch.randn(n, device="cuda", generator=gen)).to(torch.bfloat16)
    amax = torch.zeros(1, device="cuda", dtype=torch.int32)
    pkg.ops.adamw_master_step(p, w, g, m, v, step=1, amax_bits=amax, **HP)
    torch.cuda.synchronize()
    assert amax.view(torch.float32).item() == p.float().abs().max().item()
    gs = pkg.ops.global_scale_from_amax(torch.stack([amax[0], torch.zeros_like(amax[0])]))
    assert gs[0].item() == pkg.ops.global_scale(p).item() and gs[1].item() == 1.0
