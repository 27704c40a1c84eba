"""The sequence-sharded router on 2 GPUs over NCCL: each rank routes its rows
of the sequence (unequal lengths) and the concatenated outputs equal the
single-call router on the whole sequence bit for bit, with certified columns
(one all-gather) and with columns that fail the certificate (the rank-order
chain of point-to-point carries). Skipped with fewer than 2 GPUs.
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
SIZES = [700, 324]


def _inputs(extreme):
    g = torch.Generator().manual_seed(17)
    x = torch.randn(2, sum(SIZES), 512, generator=g)
    if extreme:
        x[0, 17, 5] = 1e-30
        x[1, :, 77] *= 1e30
    return (x.to(torch.bfloat16), torch.randn(32, 512, generator=g) * 0.02,
            torch.randn(8, 32, generator=g) * 0.2, torch.randn(2, sum(SIZES), 8, generator=g))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, scan_mode, extreme):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        sys.path.insert(0, ROOT)
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from naylis_b200.sequence_parallel import route_sequence_sharded
        x, w_down, w_up, noise = _inputs(extreme)
        t0 = sum(SIZES[:rank])
        sl = slice(t0, t0 + SIZES[rank])
        dev = torch.device("cuda", rank)
        probs, idx, gates = route_sequence_sharded(
            x[:, sl].to(dev), w_down.to(dev), w_up.to(dev), 2, noise[:, sl].to(dev), t_base=t0,
            compute_dtype=torch.bfloat16, scan_mode=scan_mode)
        torch.cuda.synchronize()
        q.put((rank, {"probs": probs.cpu().numpy(), "idx": idx.cpu().numpy(), "gates": gates.cpu().numpy()}))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("scan_mode,extreme", [("fp64", False), ("fp64", True), ("fp32", False)])
def test_sharded_router_on_two_gpus_equals_whole_sequence(scan_mode, extreme):
    from naylis_b200 import mom_kernels as mk
    world = len(SIZES)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, scan_mode, extreme)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out = q.get(timeout=180)
        res[rank] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
    x, w_down, w_up, noise = _inputs(extreme)
    probs, idx, gates = mk.mom_route(x.cuda(), w_down.cuda(), w_up.cuda(), 2, noise.cuda(),
                                     compute_dtype=torch.bfloat16, scan_mode=scan_mode)
    whole = {"probs": probs.cpu().numpy(), "idx": idx.cpu().numpy(), "gates": gates.cpu().numpy()}
    for k in whole:
        got = np.concatenate([res[r][k] for r in range(world)], 1)
        assert np.array_equal(got, whole[k]), k
