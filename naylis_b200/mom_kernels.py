"""The ``mom_kernels`` door of the sm_100a backend.

Mirrors the reference's dispatch door (mom_kernels/__init__.py:37-117: same
function names, arguments and fail-loud behaviour) for one new mode,
``"sm100"``: the gated memory read and the fused causal router run as
hand-written CUDA kernels for B200 through ``libnaylis_mom.so``. There is no
fallback inside this mode — a missing library, a non-sm_100 device or an
unsupported shape raises.

Added entry, not in the reference door: ``mom_route`` (the reference's router
is inline in model.py:178-220; the fused router kernel replaces it).
"""
from __future__ import annotations

import torch

from . import _lib

MODE = "sm100"
_ANNOUNCED = {"backend": None}


def _device_type(device) -> str:
    if isinstance(device, torch.device):
        return device.type
    return str(device).split(":")[0].lower()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _device_ok(device) -> None:
    idx = device.index if isinstance(device, torch.device) and device.index is not None \
        else torch.cuda.current_device()
    _lib.call("mom_device_check", idx)


def preflight(device_type: str) -> None:
    """Fail fast at startup if ``device_type`` cannot run the sm100 backend
    (reference: mom_kernels/__init__.py:37-53)."""
    if device_type != "cuda":
        raise RuntimeError(
            f"use_kernel=true with the sm100 backend requires a CUDA B200 (sm_100) device; "
            f"this process resolved to {device_type!r}. Set use_kernel=false (eager SDPA, "
            f"the parity reference) or run on the accelerator.")
    if not torch.cuda.is_available():
        raise RuntimeError("use_kernel=true (sm100): CUDA is not available in this process.")
    _lib.load()
    _device_ok(torch.device("cuda", torch.cuda.current_device()))


def _read_dtype(dtype):
    """The dtype the read's activations will have. The reference resolves with
    the dtype of the layer input x (model.py:164-165), which is fp32 under
    bf16 autocast (the residual stream keeps the fp32 master dtype); the q
    projection then runs in bf16, so the read gets bf16 activations."""
    if dtype == torch.float32 and torch.is_autocast_enabled("cuda") \
            and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        return torch.bfloat16
    return dtype


def resolve_mode(device, dtype, *, head_dim=None) -> str:
    """Pick the kernel backend and check its contract (reference:
    mom_kernels/__init__.py:56-84). Only ``"sm100"`` is served here: bf16
    activations (bf16 tensors, or fp32 ones inside a CUDA bf16 autocast
    region, which the read receives as bf16), fp32 activations outside
    autocast (the fp32 read), and head_dim 64 or 128 on an sm_100 device;
    anything else raises instead of falling back."""
    device_type = _device_type(device)
    if device_type != "cuda":
        raise RuntimeError(
            f"use_kernel=true: no sm100 kernel backend for device {device_type!r} "
            f"(the sm100 backend runs on CUDA B200 only).")
    dtype = _read_dtype(dtype)
    if dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(
            f"use_kernel=true (sm100) requires bf16 activations (the repo AMP dtype) or fp32 "
            f"(the fp32 read); fp16 is unsupported; got {dtype}.")
    if head_dim is not None:
        if head_dim > 128 or head_dim & (head_dim - 1) != 0:
            raise RuntimeError(
                f"use_kernel=true (sm100): head_dim {head_dim} must be a power of two <= 128.")
        if dtype == torch.bfloat16 and head_dim not in (64, 128):
            raise RuntimeError(
                f"use_kernel=true (sm100): the bf16 read kernels implement head_dim 64 and 128; "
                f"got {head_dim}.")
        if dtype == torch.float32 and head_dim not in (16, 32, 64, 128):
            raise RuntimeError(
                f"use_kernel=true (sm100): the fp32 read implements head_dim 16, 32, 64 and 128; "
                f"got {head_dim}.")
    _lib.load()
    dev = torch.device(device) if not isinstance(device, torch.device) else device
    if torch.cuda.is_available():
        _device_ok(dev)
    else:
        raise RuntimeError("use_kernel=true (sm100): CUDA is not available in this process.")
    return MODE


def announce(backend: str) -> None:
    """Print the backend banner once per process (reference: :105-117)."""
    if _ANNOUNCED["backend"] != backend:
        _ANNOUNCED["backend"] = backend
        if backend == MODE:
            print("[MoM] use_kernel=true -> backend 'sm100': routing-set bucketing, "
                  "read over the selected blocks only (hand-written sm_100a kernels), "
                  "fused exact-prefix-scan router.")


# ====================================================================== read
class _MomReadFunction(torch.autograd.Function):
    """Autograd of the sm100 read: saves q, k, v, out, the fp32 log-sum-exp,
    the routing plan and q in plan row order (reference:
    mom_kernels/triton_gpu.py:323-409)."""

    @staticmethod
    def forward(ctx, q_sh, k, v, top_idx, log_gates, num_blocks, block_size):
        B, S, H, hd = q_sh.shape
        L = k.shape[0]
        N, top = B * S, top_idx.shape[-1]
        dev = q_sh.device
        st = _stream(dev)
        idx = top_idx.reshape(N, top)
        if idx.dtype not in (torch.int64, torch.int32):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
        lg = log_gates.reshape(N, top).to(torch.float32).contiguous()
        plan = torch.empty(_lib.load().mom_plan_size(N, num_blocks, top), dtype=torch.uint8, device=dev)
        _lib.call("mom_bucket", idx.data_ptr(), _lib.I64 if idx.dtype == torch.int64 else _lib.I32,
                  lg.data_ptr(), N, num_blocks, top, plan.data_ptr(), plan.numel(), st)
        out = torch.empty_like(q_sh)
        lse = torch.empty((H, N), dtype=torch.float32, device=dev)
        # q in routing-plan row order, filled by the forward and read again by the backward
        q_rows = torch.empty((N, H * hd), dtype=q_sh.dtype, device=dev)
        _lib.call("mom_read_fwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.BF16, B, S, H, hd,
                  num_blocks, block_size, top, plan.data_ptr(), out.data_ptr(), lse.data_ptr(),
                  q_rows.data_ptr(), st)
        ctx.save_for_backward(q_sh, k, v, out, lse, plan, q_rows)
        ctx.meta = (num_blocks, block_size, top, L)
        return out

    @staticmethod
    def backward(ctx, dout):
        q_sh, k, v, out, lse, plan, q_rows = ctx.saved_tensors
        num_blocks, block_size, top, L = ctx.meta
        B, S, H, hd = q_sh.shape
        N = B * S
        dev = q_sh.device
        st = _stream(dev)
        dout = dout.to(torch.bfloat16).contiguous()
        dq = torch.empty_like(q_sh)
        dk = torch.empty((L, H * hd), dtype=torch.float32, device=dev)
        dv = torch.empty_like(dk)
        dlg = torch.empty((B, S, top), dtype=torch.float32, device=dev)
        ws = torch.empty(_lib.load().mom_read_bwd_workspace_size(B, S, H, hd), dtype=torch.uint8, device=dev)
        _lib.call("mom_read_bwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                  dout.data_ptr(), lse.data_ptr(), _lib.BF16, B, S, H, hd, num_blocks, block_size,
                  top, plan.data_ptr(), q_rows.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                  dlg.data_ptr(), ws.data_ptr(), ws.numel(), st)
        return (dq, *_kv_grads(dk, dv, k.dtype), None, dlg, None, None)


def _kv_grads(dk, dv, dtype):
    """dK, dV (fp32) cast to the bank's dtype (bf16 here), written side by side into
    one (L, 2n) buffer by one kernel (csrc/scale.cu, kv_pack) and returned as its
    two halves, so the bank projection's backward (trunk.bank_kv) reads [dK | dV]
    without another copy."""
    L, n = dk.shape
    both = torch.empty(L, 2 * n, dtype=dtype, device=dk.device)
    if dtype != torch.bfloat16:
        raise RuntimeError(f"sm100 mom_read backward: bf16 bank expected, got {dtype}")
    _lib.call("mom_kv_pack_bf16", dk.data_ptr(), dv.data_ptr(), L, n, both.data_ptr(), _stream(dk.device))
    return both[:, :n], both[:, n:]


class _MomReadSplitFunction(torch.autograd.Function):
    """The same read for top-k routing with more block sets than the set
    bucketing holds (``mom_plan_size`` is 0: top-4 of 32 blocks): every
    (token, k) pair is a row of a top-1 plan, and each token's rows are
    combined by their log-sum-exp (csrc/split.cu). Saves q, k, v, out, the
    rows' lse and softmax shares, the plan and q in plan order."""

    @staticmethod
    def forward(ctx, q_sh, k, v, top_idx, log_gates, num_blocks, block_size):
        B, S, H, hd = q_sh.shape
        L = k.shape[0]
        N, top = B * S, top_idx.shape[-1]
        M = N * top
        dev = q_sh.device
        st = _stream(dev)
        lib = _lib.load()
        idx = top_idx.reshape(N, top)
        if idx.dtype not in (torch.int64, torch.int32):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
        lg = log_gates.reshape(N, top).to(torch.float32).contiguous()
        plan = torch.empty(lib.mom_plan_split_size(N, num_blocks, top), dtype=torch.uint8, device=dev)
        idt = _lib.I64 if idx.dtype == torch.int64 else _lib.I32
        _lib.call("mom_bucket_split", idx.data_ptr(), idt, lg.data_ptr(), N, num_blocks, top, plan.data_ptr(),
                  plan.numel(), st)
        out = torch.empty_like(q_sh)
        lse_rows = torch.empty((H, M), dtype=torch.float32, device=dev)
        weights = torch.empty((M, H), dtype=torch.float32, device=dev)
        q_rows = torch.empty((M, H * hd), dtype=q_sh.dtype, device=dev)
        ws = torch.empty(lib.mom_read_split_fwd_workspace_size(B, S, H, hd, top), dtype=torch.uint8, device=dev)
        _lib.call("mom_read_split_fwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.BF16, B, S, H, hd,
                  num_blocks, block_size, top, idx.data_ptr(), idt, plan.data_ptr(), out.data_ptr(),
                  lse_rows.data_ptr(), weights.data_ptr(), q_rows.data_ptr(), ws.data_ptr(), ws.numel(), st)
        ctx.save_for_backward(q_sh, k, v, out, lse_rows, weights, idx, plan, q_rows)
        ctx.meta = (num_blocks, block_size, top, L, idt)
        return out

    @staticmethod
    def backward(ctx, dout):
        q_sh, k, v, out, lse_rows, weights, idx, plan, q_rows = ctx.saved_tensors
        num_blocks, block_size, top, L, idt = ctx.meta
        B, S, H, hd = q_sh.shape
        dev = q_sh.device
        st = _stream(dev)
        dout = dout.to(torch.bfloat16).contiguous()
        dq = torch.empty_like(q_sh)
        dk = torch.empty((L, H * hd), dtype=torch.float32, device=dev)
        dv = torch.empty_like(dk)
        dlg = torch.empty((B, S, top), dtype=torch.float32, device=dev)
        ws = torch.empty(_lib.load().mom_read_split_bwd_workspace_size(B, S, H, hd, top), dtype=torch.uint8,
                         device=dev)
        _lib.call("mom_read_split_bwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                  dout.data_ptr(), lse_rows.data_ptr(), weights.data_ptr(), _lib.BF16, B, S, H, hd, num_blocks,
                  block_size, top, idx.data_ptr(), idt, plan.data_ptr(), q_rows.data_ptr(), dq.data_ptr(),
                  dk.data_ptr(), dv.data_ptr(), dlg.data_ptr(), ws.data_ptr(), ws.numel(), st)
        return (dq, *_kv_grads(dk, dv, k.dtype), None, dlg, None, None)


class _MomReadF32Function(torch.autograd.Function):
    """The read for fp32 activations (csrc/read_f32.cu): fp32 FMA throughout, the
    reference's fp32 results to ~1e-6. Runs on the block-split plan for any top;
    saves q, k, v, out, the token-order log-sum-exp, the routing ids and the plan."""

    @staticmethod
    def forward(ctx, q_sh, k, v, top_idx, log_gates, num_blocks, block_size):
        B, S, H, hd = q_sh.shape
        N, top = B * S, top_idx.shape[-1]
        dev = q_sh.device
        st = _stream(dev)
        lib = _lib.load()
        idx = top_idx.reshape(N, top)
        if idx.dtype not in (torch.int64, torch.int32):
            idx = idx.to(torch.int64)
        idx = idx.contiguous()
        idt = _lib.I64 if idx.dtype == torch.int64 else _lib.I32
        lg = log_gates.reshape(N, top).to(torch.float32).contiguous()
        plan = torch.empty(lib.mom_plan_split_size(N, num_blocks, top), dtype=torch.uint8, device=dev)
        _lib.call("mom_bucket_split", idx.data_ptr(), idt, lg.data_ptr(), N, num_blocks, top, plan.data_ptr(),
                  plan.numel(), st)
        out = torch.empty_like(q_sh)
        lse = torch.empty((N, H), dtype=torch.float32, device=dev)
        ws = torch.empty(lib.mom_read_f32_workspace_size(B, S, H, hd, top), dtype=torch.uint8, device=dev)
        _lib.call("mom_read_f32_fwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), B, S, H, hd, num_blocks,
                  block_size, top, idx.data_ptr(), idt, plan.data_ptr(), out.data_ptr(), lse.data_ptr(),
                  ws.data_ptr(), ws.numel(), st)
        ctx.save_for_backward(q_sh, k, v, out, lse, idx, plan)
        ctx.meta = (num_blocks, block_size, top, idt)
        return out

    @staticmethod
    def backward(ctx, dout):
        q_sh, k, v, out, lse, idx, plan = ctx.saved_tensors
        num_blocks, block_size, top, idt = ctx.meta
        B, S, H, hd = q_sh.shape
        dev = q_sh.device
        st = _stream(dev)
        lib = _lib.load()
        dout = dout.to(torch.float32).contiguous()
        dq = torch.empty_like(q_sh)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        dlg = torch.empty((B, S, top), dtype=torch.float32, device=dev)
        ws = torch.empty(lib.mom_read_f32_workspace_size(B, S, H, hd, top), dtype=torch.uint8, device=dev)
        _lib.call("mom_read_f32_bwd", q_sh.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
                  lse.data_ptr(), B, S, H, hd, num_blocks, block_size, top, idx.data_ptr(), idt, plan.data_ptr(),
                  dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dlg.data_ptr(), ws.data_ptr(), ws.numel(), st)
        return dq, dk, dv, None, dlg, None, None


def _check_read_args(q_sh, k, v, top_idx, top_gates, num_blocks, block_size, mode):
    if mode != MODE:
        raise RuntimeError(f"unknown kernel mode {mode!r} (this door serves {MODE!r})")
    if k.dim() != 2 or v.dim() != 2:
        raise RuntimeError("sm100 mom_read: shared K/V (L, D) only, got batched inputs")
    if not (q_sh.dtype == k.dtype == v.dtype) or q_sh.dtype not in (torch.bfloat16, torch.float32):
        raise RuntimeError(f"sm100 mom_read requires bf16 (or all-fp32) activations, got q {q_sh.dtype}, "
                           f"k {k.dtype}, v {v.dtype}")
    if not q_sh.is_cuda:
        raise RuntimeError("sm100 mom_read: tensors must be on a CUDA device")
    if k.shape[0] != num_blocks * block_size:
        raise RuntimeError(
            f"sm100 mom_read: bank is {k.shape[0]} slots but num_blocks ({num_blocks}) x "
            f"block_size ({block_size}) disagrees")
    B, S, H, hd = q_sh.shape
    if k.shape[1] != H * hd or v.shape != k.shape:
        raise RuntimeError(f"sm100 mom_read: k/v must be (L, {H * hd}), got {tuple(k.shape)}, {tuple(v.shape)}")
    if top_idx.shape != top_gates.shape or top_idx.shape[:2] != (B, S):
        raise RuntimeError("sm100 mom_read: top_idx / top_gates must be (B, S, top)")


def _read_apply(q_sh, k, v, top_idx, log_gates, num_blocks, block_size):
    B, S = q_sh.shape[:2]
    top = top_idx.shape[-1]
    if q_sh.dtype == torch.float32:
        fn = _MomReadF32Function
    # routing sets beyond what the set bucketing holds: the block-split read
    elif _lib.load().mom_plan_size(B * S, int(num_blocks), top):
        fn = _MomReadFunction
    else:
        fn = _MomReadSplitFunction
    return fn.apply(q_sh.contiguous(), k.contiguous(), v.contiguous(), top_idx, log_gates, int(num_blocks),
                    int(block_size))


def mom_read_log_gates(q_sh, k, v, top_idx, log_gates, *, num_blocks, block_size, mode: str = MODE):
    """``mom_read`` taking log(max(gates, 1e-9)) directly (fp32, (B, S, top)),
    e.g. the fourth output of ``mom_route_log_gates``; the gradient is returned
    for log_gates. Not in the reference door (its mom_read takes the gates)."""
    _check_read_args(q_sh, k, v, top_idx, log_gates, num_blocks, block_size, mode)
    return _read_apply(q_sh, k, v, top_idx, log_gates.float(), num_blocks, block_size)


def mom_read(q_sh, k, v, top_idx, top_gates, *, num_blocks, block_size, mode: str = MODE):
    """MoM memory read with the per-token gate bias (reference door:
    mom_kernels/__init__.py:87-102; contract of mom_kernels/triton_gpu.py:412-439).

    q_sh (B, S, H, hd) bf16; shared k, v (L, H*hd) bf16 with L = num_blocks *
    block_size; top_idx (B, S, top) block ids; top_gates (B, S, top) fp32
    softmax gates. Returns (B, S, H, hd). With q, k, v all fp32 the read runs
    in fp32 (csrc/read_f32.cu) and returns fp32. Gradients reach q, k, v and the
    gates (through log(clamp_min(g, 1e-9)), as the reference bias does).
    """
    _check_read_args(q_sh, k, v, top_idx, top_gates, num_blocks, block_size, mode)
    log_gates = top_gates.clamp_min(1e-9).log().float()
    return _read_apply(q_sh, k, v, top_idx, log_gates, num_blocks, block_size)


# ====================================================================== router
def _compute_dtype(w: torch.Tensor) -> torch.dtype:
    """The dtype the router linears run in: autocast's dtype when enabled."""
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return w.dtype


def _dt_code(dtype) -> int:
    if dtype == torch.float32:
        return _lib.F32
    if dtype == torch.bfloat16:
        return _lib.BF16
    raise RuntimeError(f"sm100 router: unsupported dtype {dtype} (fp32 or bf16)")


class _MomRouteFunction(torch.autograd.Function):
    """Fused causal router (reference: model.py:178-220). Outputs router_probs,
    top_idx (no gradient) and top_gates; the backward returns dx, dW_down and
    dW_up (the reverse prefix scan runs in rank-r space)."""

    @staticmethod
    def forward(ctx, x, w_down, w_up, noise, top, compute_dtype, scan_mode, x_lowp=None):
        B, S, d = x.shape
        r, nb = w_down.shape[0], w_up.shape[0]
        dev = x.device
        st = _stream(dev)
        x_c = x.contiguous()
        wd = w_down.detach().to(compute_dtype).contiguous()
        wu = w_up.detach().to(compute_dtype).contiguous()
        probs = torch.empty((B, S, nb), dtype=torch.float32, device=dev)
        top_idx = torch.empty((B, S, top), dtype=torch.int64, device=dev)
        gates = torch.empty((B, S, top), dtype=torch.float32, device=dev)
        log_gates = torch.empty((B, S, top), dtype=torch.float32, device=dev)
        act = torch.empty((B, S, r), dtype=compute_dtype, device=dev)
        cd = _dt_code(compute_dtype)
        ws = torch.empty(_lib.load().mom_route_workspace_size(B, S, d, r, nb, cd), dtype=torch.uint8, device=dev)
        nz = None
        if noise is not None:
            nz = noise.to(torch.float32).contiguous()
        _lib.call("mom_route_fwd", x_c.data_ptr(), _dt_code(x.dtype), B, S, d, wd.data_ptr(),
                  wu.data_ptr(), cd, r, nb, top, _ptr(nz), _lib.SCAN_MODES[scan_mode],
                  probs.data_ptr(), top_idx.data_ptr(), _lib.I64, gates.data_ptr(), log_gates.data_ptr(),
                  act.data_ptr(), ws.data_ptr(), ws.numel(), st)
        # the backward reads x only as its bf16 rounding (dW_down = u^T bf16(x)): a caller
        # that already holds bf16(x) (x_lowp) saves the fp32 read of x there
        ctx.save_for_backward(x_c if x_lowp is None else x_lowp.contiguous(), wd, wu, probs, top_idx, gates, act)
        ctx.meta = (top, cd, w_down.dtype, w_up.dtype, x.dtype)
        ctx.mark_non_differentiable(top_idx)
        # outputs without a consumer (top_idx; gates when the read takes log_gates) reach the
        # backward as None instead of zero-filled tensors
        ctx.set_materialize_grads(False)
        return probs, top_idx, gates, log_gates

    @staticmethod
    def backward(ctx, dprobs, _didx, dgates, dlog_gates):
        x, wd, wu, probs, top_idx, gates, act = ctx.saved_tensors
        top, cd, wd_dtype, wu_dtype, x_dtype = ctx.meta
        B, S, d = x.shape
        r, nb = wd.shape[0], wu.shape[0]
        dev = x.device
        st = _stream(dev)
        dp = None if dprobs is None else dprobs.to(torch.float32).contiguous()
        dg = None if dgates is None else dgates.to(torch.float32).contiguous()
        dlg = None if dlog_gates is None else dlog_gates.to(torch.float32).contiguous()
        dx = torch.empty(x.shape, dtype=x_dtype, device=dev)
        dw_down = torch.empty((r, d), dtype=torch.float32, device=dev)
        dw_up = torch.empty((nb, r), dtype=torch.float32, device=dev)
        ws = torch.empty(_lib.load().mom_route_bwd_workspace_size(B, S, d, r, nb), dtype=torch.uint8, device=dev)
        _lib.call("mom_route_bwd", x.data_ptr(), _dt_code(x.dtype), B, S, d, wd.data_ptr(),
                  wu.data_ptr(), cd, r, nb, top, probs.data_ptr(), top_idx.data_ptr(), _lib.I64,
                  gates.data_ptr(), act.data_ptr(), _ptr(dlg), _ptr(dg), _ptr(dp), dx.data_ptr(),
                  _dt_code(x_dtype), 0, dw_down.data_ptr(), dw_up.data_ptr(), ws.data_ptr(),
                  ws.numel(), st)
        return dx, dw_down.to(wd_dtype), dw_up.to(wu_dtype), None, None, None, None, None


def mom_route(x, w_down, w_up, top_blocks: int, noise=None, *, compute_dtype=None,
              scan_mode: str = "fp32"):
    """Fused causal router: returns (router_probs, top_idx, top_gates).

    x (B, S, d) fp32/bf16 on CUDA; w_down (r, d) and w_up (nb, r) are the
    router_down / router_up weights (any float dtype; they are cast to the
    compute dtype — autocast's when enabled, as nn.Linear would be). noise
    (B, S, nb): the already-scaled Gumbel noise added before top-k, or None.
    scan_mode "fp32" (default) reproduces torch's CUDA cumsum bit for bit — what
    the reference's eager router computes on the same GPU — and "fp64" its
    CPU cumsum.
    """
    if not x.is_cuda:
        raise RuntimeError("sm100 mom_route: x must be on a CUDA device")
    if x.dim() != 3 or w_down.dim() != 2 or w_up.dim() != 2 or w_down.shape[1] != x.shape[2] \
            or w_up.shape[1] != w_down.shape[0]:
        raise RuntimeError(
            f"sm100 mom_route: shapes x {tuple(x.shape)}, w_down {tuple(w_down.shape)}, "
            f"w_up {tuple(w_up.shape)} disagree")
    if scan_mode not in _lib.SCAN_MODES:
        raise RuntimeError(f"sm100 mom_route: scan_mode must be one of {sorted(_lib.SCAN_MODES)}")
    cd = compute_dtype or _compute_dtype(w_down)
    probs, idx, gates, _ = _MomRouteFunction.apply(x, w_down, w_up, noise, int(top_blocks), cd, scan_mode)
    return probs, idx, gates


def mom_route_log_gates(x, w_down, w_up, top_blocks: int, noise=None, *, compute_dtype=None,
                        scan_mode: str = "fp32", x_lowp=None):
    """``mom_route`` that also returns log(max(top_gates, 1e-9)) as a fourth,
    differentiable output, computed by the router kernel; its gradient goes
    into the router backward directly (the kernel applies the clamp / log
    derivative). For callers that feed the read with log-gates
    (``mom_read_log_gates``), as the MoM layer does: the same values as the
    reference's bias (mom_kernels/reference.py:14-29) without the torch
    clamp / log ops and their backward.

    x_lowp: optionally x rounded to bf16 (round to nearest even), when the
    caller has it already; the backward then reads it instead of x, with the
    same results (it uses x only in that rounding) and half the bytes."""
    if not x.is_cuda:
        raise RuntimeError("sm100 mom_route: x must be on a CUDA device")
    if scan_mode not in _lib.SCAN_MODES:
        raise RuntimeError(f"sm100 mom_route: scan_mode must be one of {sorted(_lib.SCAN_MODES)}")
    if x_lowp is not None and (x_lowp.shape != x.shape or x_lowp.dtype != torch.bfloat16):
        raise RuntimeError("sm100 mom_route: x_lowp must be x's shape in bf16")
    cd = compute_dtype or _compute_dtype(w_down)
    return _MomRouteFunction.apply(x, w_down, w_up, noise, int(top_blocks), cd, scan_mode, x_lowp)


class _MomScaleFunction(torch.autograd.Function):
    """y = mom_scale * o with the reference's dtype promotion (model.py:239):
    fp32 result from a bf16 o; the backward is one fused pass."""

    @staticmethod
    def forward(ctx, o, scale):
        oc = o.contiguous()
        sc = scale.detach().to(torch.float32).contiguous()
        y = torch.empty(oc.shape, dtype=torch.float32, device=oc.device)
        _lib.call("mom_scale_fwd", oc.data_ptr(), _dt_code(oc.dtype), oc.numel(), sc.data_ptr(),
                  y.data_ptr(), _stream(oc.device))
        ctx.save_for_backward(oc, sc)
        ctx.scale_dtype = scale.dtype
        return y

    @staticmethod
    def backward(ctx, g):
        oc, sc = ctx.saved_tensors
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        g = g.contiguous()
        d_o = torch.empty_like(oc)
        d_s = torch.empty(1, dtype=torch.float32, device=oc.device)
        _lib.call("mom_scale_bwd", g.data_ptr(), _dt_code(g.dtype), oc.data_ptr(), _dt_code(oc.dtype),
                  oc.numel(), sc.data_ptr(), d_o.data_ptr(), d_s.data_ptr(), _stream(oc.device))
        return d_o, d_s.to(ctx.scale_dtype)


def mom_scale(o, scale):
    """``scale * o`` for the layer output (scale: the (1,) mom_scale parameter)."""
    if not o.is_cuda:
        raise RuntimeError("sm100 mom_scale: o must be on a CUDA device")
    if scale.numel() != 1:
        raise RuntimeError("sm100 mom_scale: scale must hold one element")
    return _MomScaleFunction.apply(o, scale)


class _RouterAuxFunction(torch.autograd.Function):
    """The load-balancing aux loss of one MoM layer and its router logs
    (reference: model.py:476-517) in one deterministic kernel. Returns the
    (3 + nb,) buffer [aux, entropy, dead_frac, frac_0 ..]; only aux carries a
    gradient: d aux / d probs[t, e] = nb * frac_e / N."""

    @staticmethod
    def forward(ctx, probs, top_idx, nb):
        p = probs.detach().to(torch.float32).contiguous()
        idx = top_idx.contiguous()
        N = p.numel() // nb
        out = torch.empty(3 + nb, dtype=torch.float32, device=p.device)
        ws = torch.empty(_lib.load().mom_router_aux_workspace_size(N, nb), dtype=torch.uint8, device=p.device)
        code = _lib.I64 if idx.dtype == torch.int64 else _lib.I32
        _lib.call("mom_router_aux", p.data_ptr(), idx.data_ptr(), code, N, nb, idx.shape[-1], ws.data_ptr(),
                  ws.numel(), out.data_ptr(), _stream(p.device))
        ctx.save_for_backward(out)
        ctx.meta = (N, nb, probs.shape, probs.dtype)
        return out

    @staticmethod
    def backward(ctx, grad):
        (out,) = ctx.saved_tensors
        N, nb, shape, dtype = ctx.meta
        row = grad[0] * (nb / N) * out[3:]
        return row.repeat(N, 1).reshape(shape).to(dtype), None, None


def router_aux(probs, top_idx, num_blocks: int):
    """(3 + nb,) fp32 [aux, entropy, dead_frac, frac_e ...] of one MoM layer from
    its stashed router_probs (N, nb) and top_idx (N, top) on a CUDA device:
    aux = nb * sum_e frac_e * mean_t probs[t, e] (differentiable w.r.t. probs),
    entropy = -mean_t sum_e p log(max(p, 1e-9)), dead_frac = share of blocks no
    token selected (reference: model.py:476-517)."""
    if not probs.is_cuda or top_idx.dtype not in (torch.int32, torch.int64):
        raise RuntimeError("router_aux: CUDA probs and int32/int64 top_idx")
    return _RouterAuxFunction.apply(probs, top_idx, int(num_blocks))


def gumbel_noise(shape, device, noise_scale: float):
    """Scaled Gumbel noise drawn exactly as the reference draws it
    (model.py:209-213: torch.rand_like on the fp32 logits, then
    noise_scale * -log(-log(u + 1e-9) + 1e-9)); on CUDA the transform is one
    kernel (csrc/scale.cu, gumbel) with the same fp32 results, in place.
    CUDA devices only."""
    if _device_type(device) != "cuda":
        raise RuntimeError("sm100 gumbel_noise: device must be CUDA")
    u = torch.rand(shape, device=device, dtype=torch.float32)
    _lib.call("mom_gumbel", u.data_ptr(), u.numel(), float(noise_scale), u.data_ptr(), _stream(u.device))
    return u


__all__ = ["MODE", "preflight", "resolve_mode", "announce", "mom_read", "mom_route", "mom_scale", "router_aux",
           "gumbel_noise"]
