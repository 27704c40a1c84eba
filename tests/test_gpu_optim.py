"""GPU parity of the one-launch AdamW (csrc/optim.cu, naylis_b200.optim) with
torch.optim.AdamW, the reference's optimizer, on the same parameters and
gradients: parameters and both moments within fp32 rounding after several
steps (torch forms m by lerp and divides by the bias-corrected root; the kernel
uses FMAs and a reciprocal), shapes with chunk tails and unaligned lengths, a
parameter without a gradient left alone; and the bf16 copy written in the same
pass equal to the updated parameter rounded to bf16."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_adamw_matches_torch_and_writes_bf16_copies():
    from naylis_b200 import optim, trunk
    torch.manual_seed(11)
    dev = torch.device("cuda")
    shapes = [(1024, 1024), (3, 5), (65537,), (7,), (130, 1000)]
    ours = [torch.nn.Parameter(torch.randn(s, device=dev)) for s in shapes]
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ours]
    skip = torch.nn.Parameter(torch.randn(9, device=dev))
    kw = dict(lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    opt = optim.AdamW(ours + [skip], **kw)
    ropt = torch.optim.AdamW(ref, foreach=False, **kw)
    trunk._bf16_weights([ours[0]])          # register bf16 rows for the first parameter
    skip0 = skip.detach().clone()
    for _ in range(4):
        for p, q in zip(ours, ref):
            g = torch.randn_like(p)
            p.grad = g.clone()
            q.grad = g.clone()
        opt.step()
        ropt.step()
    sd = opt.state_dict()
    assert all(int(v["step"]) == 4 for v in sd["state"].values())
    for p, q in zip(ours, ref):
        assert torch.allclose(p, q, rtol=1e-5, atol=1e-6)
        sp, sq = opt.state[p], ropt.state[q]
        assert torch.allclose(sp["exp_avg"], sq["exp_avg"], rtol=1e-5, atol=1e-7)
        assert torch.allclose(sp["exp_avg_sq"], sq["exp_avg_sq"], rtol=1e-5, atol=1e-9)
        assert int(sp["step"]) == 4
    assert torch.equal(skip, skip0) and skip not in opt.state
    assert torch.equal(trunk.bf16_copy(ours[0]), ours[0].detach().bfloat16())
    # the copy is fresh: the projection reuses it without recasting
    buf = trunk._bf16_weights([ours[0]])
    assert torch.equal(buf, ours[0].detach().bfloat16())
