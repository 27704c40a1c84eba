"""The exchange of the sequence-sharded router (naylis_b200.sequence_parallel)
on gloo process groups on CPU: 4 ranks holding unequal row ranges (one empty).

The per-shard compute is a numpy stand-in with the kernels' arithmetic (exact
fp64 totals and certificate, sequential fp64 / fp32 walks from the carry, the
oracle's router head); what is under test is the exchange: the all-gather
order, each rank's carry, the branch every rank takes, and the rank-order
chain for columns that fail the certificate and for the fp32 scan. The prefix
mean of the shards, concatenated, must equal the oracle's whole-sequence
prefix mean bit for bit, and the top-k indices must match.
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

f32, f64 = np.float32, np.float64
SIZES = [40, 0, 1, 23]
B, D, R, NB, TOP = 2, 16, 4, 6, 2


def _inputs(extreme):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((B, sum(SIZES), D)).astype(f32)
    if extreme:
        x[0, 11, 3] = 1e-30
        x[1, :, 9] *= 1e30
    w_down = (rng.standard_normal((R, D)) * 0.3).astype(f32)
    w_up = (rng.standard_normal((NB, R)) * 0.5).astype(f32)
    return x, w_down, w_up


def _numpy_ops(w_down, w_up):
    import mom_oracle as O
    from naylis_b200.sequence_parallel import ShardOps

    class NumpyShardOps(ShardOps):
        def __init__(self):
            self.h = None

        def stats(self, x):
            a = x.numpy().astype(f64)
            tot = a.sum(1)
            bound = np.abs(a).sum(1) * (1 + 2.0 ** -40)
            mag = np.abs(x.numpy())
            mag = np.where(mag > 0, mag, np.inf).min(1) if a.shape[1] else np.full((B, D), np.inf)
            em = np.where(np.isfinite(mag), np.frexp(mag.astype(f64))[1] - 24, 1 << 20).astype(f64)
            return torch.from_numpy(np.stack([tot, bound, em]))

        def carry(self, stats_all, world, rank):
            s = stats_all.numpy()
            run = np.zeros((B, D), f64)
            for j in range(rank):
                run = run + s[j, 0]
            bound = s[:, 1].sum(0) * (1 + 2.0 ** -40)
            em = s[:, 2].min(0)
            cert = (em == (1 << 20)) | ((em > -1000) & (bound < np.ldexp(1.0, (52 + em).astype(int))))
            return torch.from_numpy(np.stack([run, cert.astype(f64)])), int((~cert).sum())

        def zero_carry(self, x, scan_mode):
            return torch.zeros((B, D), dtype=torch.float32)

        def route(self, x, t_base, carry_in, want_carry_out, scan_mode):
            a = x.numpy().astype(f32)
            S = a.shape[1]
            h = np.empty((B, S, D), f32)
            c = carry_in.numpy()
            run = (c[0] if scan_mode == "fp64" else c).copy()
            for t in range(S):
                if scan_mode == "fp64":
                    run = run + a[:, t].astype(f64)
                    h[:, t] = run.astype(f32) / f32(t_base + t + 1)
                else:
                    run = (run + a[:, t]).astype(f32)
                    h[:, t] = run / f32(t_base + t + 1)
            self.h = h
            z = O.linear(h, w_down, "f32")
            act = O.round_to(np.tanh(z.astype(f64)), "f32")
            logits = O.linear(act, w_up, "f32").astype(f32)
            probs = O.softmax64(logits).astype(f32)
            idx, vals = O.topk_cuda_order(logits, TOP)
            gates = O.softmax64(vals).astype(f32)
            out = None
            if want_carry_out:
                out = torch.from_numpy(np.stack([run, c[1]]) if scan_mode == "fp64" else run.astype(f32))
            return torch.from_numpy(probs), torch.from_numpy(idx), torch.from_numpy(gates), out

    return NumpyShardOps()


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
        sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from naylis_b200.sequence_parallel import route_sequence_sharded
        x, w_down, w_up = _inputs(extreme)
        t0 = sum(SIZES[:rank])
        xs = torch.from_numpy(x[:, t0:t0 + SIZES[rank]].copy())
        ops = _numpy_ops(w_down, w_up)
        calls = []
        orig = ops.route
        ops.route = lambda *a, **k: (calls.append(a[3]), orig(*a, **k))[1]
        probs, idx, gates = route_sequence_sharded(xs, group=None, t_base=t0, scan_mode=scan_mode, ops=ops)
        q.put((rank, {"h": ops.h, "idx": idx.numpy(), "chained": calls[0]}))   # wants a carry_out
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("scan_mode,extreme", [("fp64", False), ("fp64", True), ("fp32", False)])
def test_sharded_router_exchange_equals_whole_sequence(scan_mode, extreme):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import mom_oracle as O
    world = len(SIZES)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, scan_mode, extreme)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, out = q.get(timeout=120)
        res[rank] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
    x, w_down, w_up = _inputs(extreme)
    rt = O.router_forward(x, w_down, w_up, TOP, "f32", scan_mode=scan_mode)
    h = np.concatenate([res[r]["h"] for r in range(world)], 1)
    assert np.array_equal(h, rt["h"])
    idx = np.concatenate([res[r]["idx"] for r in range(world)], 1)
    assert np.array_equal(idx, rt["top_idx"])
    # in a chain every rank but the last hands its end state on
    chain = extreme or scan_mode == "fp32"
    assert [res[r]["chained"] for r in range(world)] == [chain] * (world - 1) + [False]


def test_sharded_router_rejects_bad_calls_before_any_exchange():
    """Argument errors are raised on the host before any collective runs (a
    single gloo rank, so nothing could hang on a missing peer)."""
    import torch.distributed as dist
    from naylis_b200.sequence_parallel import route_sequence_sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=30))
    try:
        x = torch.zeros(1, 4, 16)
        with pytest.raises(RuntimeError, match="scan_mode"):
            route_sequence_sharded(x, torch.zeros(4, 16), torch.zeros(6, 4), 2, scan_mode="fp16")
        with pytest.raises(RuntimeError, match="CUDA"):
            route_sequence_sharded(x, torch.zeros(4, 16), torch.zeros(6, 4), 2)
    finally:
        dist.destroy_process_group()
