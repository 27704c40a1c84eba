"""Data-parallel gradient exchange (naylis_b200.data_parallel.GradAllReduce)
on world_size-2 gloo process groups on CPU.

* the bucketed, hook-driven all-reduce of a module with a shared bank, each
  rank on its own shard of the batch, equals the single-process full-batch
  gradient (mean loss, so the average over ranks is exact up to rounding);
* parameters that get no gradient in a step do not stall the exchange;
* with overlap=False (a backward captured in a CUDA graph) finish() alone
  exchanges every bucket, step after step;
* gradient accumulation: micro-batches under no_sync() then one exchange give
  the full-batch gradient, and a second backward before finish() without
  no_sync() raises;
* failure detection on the host: a rank that dies before the collective makes
  the survivor's next exchange fail within the process-group timeout.
"""
import contextlib
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _Net(torch.nn.Module):
    """A stand-in with the parameter structure the exchange has to get right in
    the MoM model: one bank (M) read by two consumers, so autograd sums its
    gradient before the hook fires; a router-like linear; a parameter that
    never receives a gradient."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(32, 32, bias=False)
        self.b = torch.nn.Linear(32, 32, bias=False)
        self.router = torch.nn.Linear(32, 8, bias=False)
        self.M = torch.nn.Parameter(torch.randn(8, 32))
        self.unused = torch.nn.Parameter(torch.zeros(3))

    def forward(self, x):
        h = torch.tanh(self.a(x)) @ self.M.t()
        g = torch.softmax(self.router(x), -1)
        return self.b(x) + (h * g) @ self.M


def _build(seed=0):
    torch.manual_seed(seed)
    return _Net()


def _data():
    g = torch.Generator().manual_seed(123)
    return torch.randn(4, 24, 32, generator=g)


def _loss(holder, x, parts=1):
    return (holder(x).float() ** 2).mean() / parts


def _worker(rank, world, port, q, mode):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import sys
        sys.path.insert(0, ROOT)
        timeout = datetime.timedelta(seconds=10 if mode == "fault" else 60)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timeout)
        from naylis_b200.data_parallel import GradAllReduce
        holder = _build()
        # tiny buckets: several in flight; "deferred": no collective in the
        # hooks, finish() exchanges everything (the CUDA-graph replay pattern)
        dp = GradAllReduce(holder, bucket_mb=0.001, overlap=(mode != "deferred"))
        x = _data()
        shard = x.chunk(world, dim=0)[rank]
        if mode == "fault":
            # step 1 completes on both ranks; rank 1 then dies before step 2
            dp.zero_grad()
            _loss(holder, shard).backward()
            dp.finish()
            if rank == 1:
                os._exit(3)
            dp.zero_grad()
            try:
                _loss(holder, shard).backward()   # bucket all-reduces start in the hooks
                dp.finish()
                q.put((rank, "no error"))
            except Exception as e:  # the survivor must see the failure, not hang
                q.put((rank, f"error: {type(e).__name__}"))
            q.close()
            q.join_thread()       # flush the queue before the hard exit
            os._exit(0)
        if mode in ("accum", "misuse"):
            # two micro-batches per step: the first inside no_sync (hooks only
            # accumulate), the second exchanges; "misuse" leaves no_sync out
            for it in range(2):
                dp.zero_grad()
                halves = shard.chunk(2, dim=0)
                ctx = dp.no_sync() if mode == "accum" else contextlib.nullcontext()
                with ctx:
                    _loss(holder, halves[0], 2).backward()
                try:
                    _loss(holder, halves[1], 2).backward()
                except RuntimeError as e:
                    q.put((rank, f"error: {e}"))
                    dist.destroy_process_group()
                    return
                dp.finish()
            grads = {n: p.grad.detach().numpy().copy() for n, p in holder.named_parameters()}
            q.put((rank, {"grads": grads, "nbuckets": len(dp.buckets)}))
            dist.barrier()
            dist.destroy_process_group()
            return
        for it in range(2):   # two steps: zero_grad re-arms the hooks and views
            if mode == "deferred" and it > 0:
                # a graph replay zeroes the buckets on the device and runs no
                # Python hook or zero_grad; finish() alone must exchange all
                for buf in dp.flat:
                    buf.zero_()
            else:
                dp.zero_grad()
            _loss(holder, shard).backward()
            dp.finish()
        # numpy copies travel by value; torch tensors would be shared through file
        # descriptors that vanish when this process exits before the parent reads them
        grads = {n: p.grad.detach().numpy().copy() for n, p in holder.named_parameters()}
        q.put((rank, {"grads": grads, "nbuckets": len(dp.buckets)}))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc()))


def _spawn(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    expected = world if mode != "fault" else 1
    for _ in range(expected):
        rank, res = q.get(timeout=120)
        results[rank] = res
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("mode", ["ok", "deferred"])
def test_grad_allreduce_equals_full_batch_gradient(mode):
    world = 2
    res = _spawn(world, mode)
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
    assert res[0]["nbuckets"] > 2
    holder = _build()
    for p in holder.parameters():
        p.grad = None
    _loss(holder, _data()).backward()
    for n, p in holder.named_parameters():
        ref = p.grad if p.grad is not None else torch.zeros_like(p)
        for r in range(world):
            got = torch.from_numpy(res[r]["grads"][n])
            assert torch.allclose(got, ref, rtol=1e-4, atol=1e-6), (n, (got - ref).abs().max())
    # the shared bank gets its gradient once, summed over all uses, then averaged
    assert float(abs(res[0]["grads"]["M"]).sum()) > 0
    assert torch.equal(torch.from_numpy(res[0]["grads"]["unused"]), torch.zeros(3))


def test_gradient_accumulation_under_no_sync_equals_full_batch_gradient():
    """Two micro-batches per rank per step, the first inside no_sync(): the
    exchanged gradient is the full batch's (the reference's grad_accum)."""
    res = _spawn(2, "accum")
    holder = _build()
    _loss(holder, _data()).backward()
    for n, p in holder.named_parameters():
        ref = p.grad if p.grad is not None else torch.zeros_like(p)
        for r in range(2):
            assert isinstance(res[r], dict), res[r]
            got = torch.from_numpy(res[r]["grads"][n])
            assert torch.allclose(got, ref, rtol=1e-4, atol=1e-6), (n, (got - ref).abs().max())


def test_second_backward_before_finish_raises():
    """Without no_sync(), a second backward would add into buckets already being
    exchanged: it must raise instead of returning wrong gradients."""
    res = _spawn(2, "misuse")
    for r in range(2):
        assert str(res[r]).startswith("error") and "no_sync" in str(res[r]), res[r]


def test_rank_failure_is_detected_on_the_host():
    res = _spawn(2, "fault")
    assert 0 in res
    assert str(res[0]).startswith("error"), res[0]


@pytest.mark.parametrize("bucket_mb", [0.001, 64.0])
def test_single_process_is_a_plain_backward(bucket_mb):
    from naylis_b200.data_parallel import GradAllReduce
    holder = _build()
    dp = GradAllReduce(holder, bucket_mb=bucket_mb)
    dp.zero_grad()
    _loss(holder, _data()).backward()
    dp.finish()
    got = {n: p.grad.clone() for n, p in holder.named_parameters()}
    ref_h = _build()
    _loss(ref_h, _data()).backward()
    for n, p in ref_h.named_parameters():
        ref = p.grad if p.grad is not None else torch.zeros_like(p)
        assert torch.allclose(got[n], ref, rtol=1e-6, atol=1e-7), n
