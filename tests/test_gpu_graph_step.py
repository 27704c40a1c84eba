"""The decoder's training step replayed as one CUDA graph
(naylis_b200.graph_step.GraphedTrainStep) against the same step launched eagerly:
a small Naylis decoder on the bf16 kernel path, Gumbel noise off, the package's
AdamW after each step. The first step's loss is identical bit for bit (same
kernels on the same inputs) and its gradients agree within 2e-2 of their largest
magnitude (the read's dK / dV and the router's dW are fp32 atomic sums); the
losses of later steps, on weights updated from those gradients, within 1e-3.
New token ids given to step() are used, and every .grad is its bucket slot."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(dev):
    from naylis_b200.decoder import NaylisConfig, NaylisForCausalLM
    cfg = NaylisConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, mem_size=512, mom_block_size=128, mom_top_blocks=2,
                       mom_router_rank=32)
    torch.manual_seed(0)
    model = NaylisForCausalLM(cfg)
    for m in model.mom_layers():
        m.noise_scale = 0.0
        with torch.no_grad():
            m.mom_scale.fill_(0.5)
    return model.to(dev).train()


def test_graphed_step_equals_eager_step():
    from naylis_b200.data_parallel import GradAllReduce
    from naylis_b200.graph_step import GraphedTrainStep
    from naylis_b200.optim import AdamW
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    batches = [torch.randint(0, 512, (2, 256), device=dev, generator=g) for _ in range(3)]

    model = _model(dev)
    dp = GradAllReduce(model)
    opt = AdamW(model.parameters(), lr=1e-3)
    eager_losses, eager_grads = [], None
    for i, ids in enumerate(batches):
        dp.zero_grad()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids, labels=ids)
        loss.backward()
        dp.finish()
        if i == 0:
            eager_grads = {n: p.grad.clone() for n, p in model.named_parameters()}
        opt.step()
        eager_losses.append(float(loss.detach()))
    dp.remove()

    model_g = _model(dev)
    dp_g = GradAllReduce(model_g)
    opt_g = AdamW(model_g.parameters(), lr=1e-3)
    gstep = GraphedTrainStep(model_g, dp_g, batches[0])
    assert gstep.kernels_per_replay > 0
    graph_losses = []
    for i, ids in enumerate(batches):
        loss = gstep.step(ids)
        if i == 0:
            for n, p in model_g.named_parameters():
                want = eager_grads[n]
                err = float((p.grad - want).abs().max())
                assert err <= 2e-2 * float(want.abs().max()) + 1e-12, (n, err)
        opt_g.step()
        graph_losses.append(float(loss))
    assert graph_losses[0] == eager_losses[0]
    for a, b in zip(graph_losses[1:], eager_losses[1:]):
        assert abs(a - b) <= 1e-3 * abs(b), (graph_losses, eager_losses)
    flat = [(b.data_ptr(), b.data_ptr() + 4 * b.numel()) for b in dp_g.flat]
    assert all(any(lo <= p.grad.data_ptr() < hi for lo, hi in flat) for p in model_g.parameters())
    dp_g.remove()
