"""Data-parallel decoder training on 2 GPUs over NCCL (naylis_b200.data_parallel):
each rank runs a small Naylis decoder on its own sequence with the bf16 kernel
path, the projections' weight gradients written straight into the bucket slots,
and the bucket all-reduces launched from the backward's hooks. After finish()
both ranks hold the same gradients, equal to the mean of the two sequences'
gradients computed one after the other in a single process (within 2e-2 of the
largest magnitude: the read's dK / dV are fp32 atomic sums, so two runs differ
in the last bf16 bits). The same holds for the step replayed as one CUDA graph
(graph_step.GraphedTrainStep) with the buckets exchanged after each replay.
Skipped with fewer than 2 GPUs.
"""
import datetime
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu
S = 256


def _model():
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
    return model


def _ids():
    return torch.randint(0, 512, (2, S), generator=torch.Generator().manual_seed(3))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        sys.path.insert(0, ROOT)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from naylis_b200.data_parallel import GradAllReduce
        model = _model().to(dev).train()
        dp = GradAllReduce(model, bucket_mb=0.5)
        ids = _ids()[rank:rank + 1].to(dev)
        for _ in range(2):          # the second step re-arms the slots after zero_grad
            dp.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = model(ids, labels=ids)
            loss.backward()
            dp.finish()
        torch.cuda.synchronize()
        eager = {n: p.grad.float().cpu().numpy() for n, p in model.named_parameters()}
        dp.remove()
        # the same step replayed as one CUDA graph, the buckets exchanged after the replay
        from naylis_b200.graph_step import GraphedTrainStep
        model_g = _model().to(dev).train()
        dp_g = GradAllReduce(model_g, bucket_mb=0.5, overlap=False)
        gstep = GraphedTrainStep(model_g, dp_g, ids)
        for _ in range(2):
            gstep.step(ids)
        torch.cuda.synchronize()
        graphed = {n: p.grad.float().cpu().numpy() for n, p in model_g.named_parameters()}
        q.put((rank, {"eager": eager, "graphed": graphed}))
        dist.barrier()
        del gstep
        dp_g.remove()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_decoder_data_parallel_on_two_gpus_equals_mean_gradient():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out = q.get(timeout=240)
        res[rank] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert isinstance(res[r], dict), res[r]

    dev = torch.device("cuda", 0)
    model = _model().to(dev).train()
    ids = _ids().to(dev)
    per_seq = []
    for r in range(world):
        for p in model.parameters():
            p.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids[r:r + 1], labels=ids[r:r + 1])
        loss.backward()
        per_seq.append({n: p.grad.float().cpu().numpy() for n, p in model.named_parameters()})
    for mode in ("eager", "graphed"):
        for n in per_seq[0]:
            want = (per_seq[0][n] + per_seq[1][n]) / 2
            got = res[0][mode][n]
            assert np.array_equal(got, res[1][mode][n]), (mode, n)
            err = float(np.abs(got - want).max())
            assert err <= 2e-2 * float(np.abs(want).max()) + 1e-12, (mode, n, err)
