"""CPU tests of the C ABI boundary and the Python door (no GPU needed):
the library loads, exports every function include/naylis_mom.h declares, and
rejects bad arguments with the documented status codes before any device work.
"""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "naylis_mom.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:MOM_API\s+)?(?:const\s+)?\w+\s*\*?\s*(mom_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from naylis_b200 import _lib, build
    build.build()
    return _lib.load()


def test_header_declares_the_survey_minimum():
    names = _declared_functions()
    for required in ("mom_route_fwd", "mom_route_bwd", "mom_bucket", "mom_read_fwd", "mom_read_bwd",
                     "mom_last_error_string", "mom_plan_size", "mom_route_workspace_size",
                     "mom_read_bwd_workspace_size", "mom_prefix_mean"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    from naylis_b200 import _lib
    names = _declared_functions()
    assert names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in naylis_mom.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_only_declared_symbols_are_exported(lib):
    import subprocess
    from naylis_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    exported = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}
    ours = {s for s in exported if s.startswith("mom_")}
    assert ours == set(_declared_functions())


def test_version_and_error_string(lib):
    assert lib.mom_version() >= 100
    assert isinstance(lib.mom_last_error_string(), bytes)


def test_invalid_arguments_fail_before_device_work(lib):
    from naylis_b200 import _lib
    # router: d not a multiple of 8
    rc = lib.mom_route_fwd(None, _lib.BF16, 1, 4, 12, None, None, _lib.BF16, 32, 8, 2, None, 0,
                           None, None, _lib.I64, None, None, None, None, 0, None)
    assert rc == 1 and b"multiple of 8" in lib.mom_last_error_string()
    # router: top > nb
    rc = lib.mom_route_fwd(None, _lib.BF16, 1, 4, 64, None, None, _lib.BF16, 32, 2, 3, None, 0,
                           None, None, _lib.I64, None, None, None, None, 0, None)
    assert rc == 1
    # read: head_dim 96 is unsupported (status 2), fp32 is invalid (status 1)
    rc = lib.mom_read_fwd(None, None, None, _lib.BF16, 1, 1, 2, 96, 4, 64, 2, None, None, None, None, None)
    assert rc == 2
    rc = lib.mom_read_fwd(None, None, None, _lib.F32, 1, 1, 2, 64, 4, 64, 2, None, None, None, None, None)
    assert rc == 1
    # read: a missing q_rows buffer is an invalid argument
    rc = lib.mom_read_fwd(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), _lib.BF16, 1, 4, 2,
                          64, 4, 64, 2, ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), None,
                          None)
    assert rc == 1 and "null" in _lib.last_error()
    # bucketing: too many routing sets (top-4 of 32 blocks) is reported as unsupported
    rc = lib.mom_bucket(None, _lib.I64, None, 16, 32, 4, None, 0, None)
    assert rc == 2
    assert lib.mom_plan_size(16, 32, 4) == 0
    # plan too small
    rc = lib.mom_bucket(None, _lib.I64, None, 1024, 8, 2, ctypes.c_void_p(16), 8, None)
    assert rc == 4


def test_block_split_and_shard_entries_validate_first(lib):
    from naylis_b200 import _lib
    # the block-split plan takes what set bucketing cannot (top-4 of 32 blocks) ...
    N, nb, top = 16384, 32, 4
    assert lib.mom_plan_size(N, nb, top) == 0
    split = lib.mom_plan_split_size(N, nb, top)
    # ... a top-1 plan over N*top rows plus the rows' log-gates and inverse permutation
    assert split >= lib.mom_plan_size(N * top, nb, 1) + 2 * 4 * N * top
    assert lib.mom_plan_split_size(N, nb, 9) == 0 and lib.mom_plan_split_size(N, 4, 5) == 0
    # workspaces: the rows' outputs (fwd); delta + weighted dO + dQ rows + dO rows (bwd)
    rows = N * top * 16 * 128 * 2
    assert lib.mom_read_split_fwd_workspace_size(4, 4096, 16, 128, top) >= rows
    assert lib.mom_read_split_bwd_workspace_size(4, 4096, 16, 128, top) >= 3 * rows + N * top * 16 * 4
    # argument errors come before any device work
    rc = lib.mom_bucket_split(None, _lib.I64, None, 16, 32, 9, None, 0, None)
    assert rc == 1
    rc = lib.mom_bucket_split(None, _lib.I64, None, 1024, 32, 4, ctypes.c_void_p(256), 16, None)
    assert rc == 4
    rc = lib.mom_read_split_fwd(None, None, None, _lib.BF16, 1, 4, 2, 96, 32, 128, 4, None, _lib.I64, None,
                                None, None, None, None, None, 0, None)
    assert rc == 2      # head_dim 96
    rc = lib.mom_read_split_fwd(ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256), _lib.BF16, 1, 4,
                                2, 64, 32, 128, 4, ctypes.c_void_p(256), _lib.I64, ctypes.c_void_p(256),
                                ctypes.c_void_p(256), ctypes.c_void_p(256), ctypes.c_void_p(256),
                                ctypes.c_void_p(256), None, 0, None)
    assert rc == 4      # no workspace
    # sequence shards: bad (world, rank), bad d, and a later shard without a carry
    rc = lib.mom_route_shard_carry(ctypes.c_void_p(256), 4, 4, 1, 64, ctypes.c_void_p(256), ctypes.c_void_p(256),
                                   None)
    assert rc == 1
    rc = lib.mom_route_shard_stats(ctypes.c_void_p(256), _lib.BF16, 1, 8, 12, ctypes.c_void_p(256), None)
    assert rc == 1
    rc = lib.mom_route_fwd_shard(None, _lib.BF16, 1, 4, 64, None, None, _lib.BF16, 32, 8, 2, None, 0, 128,
                                 None, None, None, None, _lib.I64, None, None, None, None, 0, None)
    assert rc == 1 and "carry_in" in _lib.last_error()
    rc = lib.mom_route_fwd_shard(None, _lib.BF16, 1, 4, 64, None, None, _lib.BF16, 32, 8, 2, None, 0,
                                 (1 << 24) - 2, ctypes.c_void_p(256), None, None, None, _lib.I64, None, None, None,
                                 None, 0, None)
    assert rc == 1 and "2^24" in _lib.last_error()


def test_plan_size_grows_with_tokens(lib):
    a, b = lib.mom_plan_size(1024, 8, 2), lib.mom_plan_size(16384, 8, 2)
    assert 0 < a < b
    # delta (fp32 per token and head) + dO in plan order (bf16)
    assert lib.mom_read_bwd_workspace_size(8, 2048, 16, 64) >= 8 * 2048 * 16 * (4 + 64 * 2)
    assert lib.mom_route_workspace_size(8, 2048, 1024, 32, 8, 1) >= 8 * 2048 * 1024 * 2


def test_door_fails_loud_off_gpu():
    from naylis_b200 import mom_kernels as mk
    with pytest.raises(RuntimeError):
        mk.preflight("cpu")
    with pytest.raises(RuntimeError):
        mk.resolve_mode(torch.device("cpu"), torch.bfloat16, head_dim=64)
    with pytest.raises(RuntimeError):
        mk.resolve_mode("cuda", torch.float32, head_dim=64)
    with pytest.raises(RuntimeError):
        mk.resolve_mode("cuda", torch.bfloat16, head_dim=96)
    q = torch.zeros(1, 4, 2, 64, dtype=torch.bfloat16)
    k = torch.zeros(256, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        mk.mom_read(q, k, k, torch.zeros(1, 4, 2, dtype=torch.int64), torch.ones(1, 4, 2),
                    num_blocks=4, block_size=64)
    with pytest.raises(RuntimeError):
        mk.mom_route(torch.zeros(1, 4, 64), torch.zeros(8, 64), torch.zeros(4, 8), 2)
    # the log-gate variants fail the same way off the GPU
    with pytest.raises(RuntimeError):
        mk.mom_read_log_gates(q, k, k, torch.zeros(1, 4, 2, dtype=torch.int64), torch.zeros(1, 4, 2),
                              num_blocks=4, block_size=64)
    with pytest.raises(RuntimeError):
        mk.mom_route_log_gates(torch.zeros(1, 4, 64), torch.zeros(8, 64), torch.zeros(4, 8), 2)
    with pytest.raises(RuntimeError):
        mk.mom_route_log_gates(torch.zeros(1, 4, 64), torch.zeros(8, 64), torch.zeros(4, 8), 2, scan_mode="fp16")


def test_layer_is_a_drop_in_for_the_reference_module():
    """naylis_b200.model.MoMLayer takes the reference's constructor arguments,
    raises its ValueErrors and has its parameter names and shapes, so a
    reference checkpoint loads into it (checked against the reference's own
    model.MoMLayer where the reference checkout is importable)."""
    from naylis_b200.model import MoMLayer
    args = dict(d_model=256, n_heads=4, mem_size=1024, block_size=128, top_blocks=2, router_rank=32)
    ours = MoMLayer(**args)
    assert ours.head_dim == 64 and ours.num_blocks == 8 and ours.scan_mode == "fp32"
    for bad in (dict(args, n_heads=3), dict(args, mem_size=1000), dict(args, top_blocks=9)):
        with pytest.raises(ValueError):
            MoMLayer(**bad)
    with pytest.raises(ValueError, match="eager"):
        MoMLayer(**args, use_kernel=False)
    ref_root = os.environ.get("NAYLIS_REFERENCE", "/root/reference")
    if not os.path.exists(os.path.join(ref_root, "model.py")):
        pytest.skip("reference checkout not importable here")
    import importlib
    import sys as _sys
    _sys.path.insert(0, ref_root)
    try:
        ref_model = importlib.import_module("model")
    finally:
        _sys.path.remove(ref_root)
    ref = ref_model.MoMLayer(**args)
    assert {k: tuple(v.shape) for k, v in ref.state_dict().items()} == \
        {k: tuple(v.shape) for k, v in ours.state_dict().items()}
    ours.load_state_dict(ref.state_dict())
    for name in ("num_blocks", "block_size", "top_blocks", "mem_slots", "n_heads", "head_dim", "noise_scale"):
        assert getattr(ours, name) == getattr(ref, name), name


def test_ctypes_signatures_match_the_header():
    """Every binding in naylis_b200/_lib.py has the argument count and return
    type class of its declaration in include/naylis_mom.h (a mismatch would pass
    arguments in the wrong registers without any error)."""
    import ctypes
    from naylis_b200 import _lib
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    decls = {}
    for ret, name, args in re.findall(r"MOM_API\s+((?:const\s+)?\w+\s*\*?)\s*(mom_\w+)\s*\(([^;]*?)\)\s*;", src,
                                      flags=re.S):
        args = " ".join(args.split())
        kinds = []
        for a in ([] if args in ("", "void") else args.split(",")):
            a = a.strip()
            kinds.append("ptr" if "*" in a else a.split()[-2] if len(a.split()) > 1 else a)
        decls[name] = (ret.replace(" ", ""), kinds)
    assert set(decls) == set(_lib.SIGNATURES)
    arg_type = {"ptr": ctypes.c_void_p, "int": ctypes.c_int, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t,
                "double": ctypes.c_double, "float": ctypes.c_float}
    for name, (res, argtypes) in _lib.SIGNATURES.items():
        ret, kinds = decls[name]
        assert len(argtypes) == len(kinds), f"{name}: {len(argtypes)} ctypes args, header has {len(kinds)}"
        for i, (got, kind) in enumerate(zip(argtypes, kinds)):
            assert got is arg_type[kind], f"{name} argument {i}: ctypes {got}, header {kind}"
        want = {"int": ctypes.c_int, "size_t": ctypes.c_size_t, "uint64_t": ctypes.c_uint64,
                "constchar*": ctypes.c_char_p}[ret]
        assert res is want, f"{name}: restype {res}, header returns {ret}"
