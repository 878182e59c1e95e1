"""qlin_sharded_fwd: the column-partitioned layer through the C ABI with an
NCCL communicator (the communicator made by the library's own bootstrap
helpers, as a host without an NCCL binding would).

* one rank (a world of one on one GPU): the all-gather is a copy, and the
  output must equal qlin_forward_ex on the same slice, for one token (the
  all-gather in place in y) and for several (the gather buffer and the
  column placement), with bias and LoRA;
* two ranks on two GPUs (skipped with fewer): each rank passes its half of
  the output quaternions and both receive the full layer's output, checked
  against the float64 oracle and, for each rank's own columns, against that
  rank's single-GPU forward bit for bit."""

import ctypes
import os

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, to_device

pytestmark = pytest.mark.gpu

FLAG_ZEROED = 2


def _ptr(t):
    return None if t is None else t.data_ptr()


def _forward_slice(qb, lib, d, y, ld_y, M, K_g, N_g, rank, scale, flags):
    dt = d["x"].dtype
    n = qb._lib.workspace_size(dt, M, K_g, N_g, rank)
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=d["x"].device)
    st = lib.qlin_forward_ex(qb._lib.dtype_code(dt), _ptr(d["x"]), 4 * K_g, *(_ptr(w) for w in d["w"]), K_g,
                             _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, scale, _ptr(y), ld_y, M,
                             K_g, N_g, _ptr(ws), n, 0, flags, qb._lib.stream_handle(d["x"].device))
    assert st == 0


def _sharded(qb, lib, comm, world, r, d, y, M, K_g, N_g, rank, scale, flags):
    dt = d["x"].dtype
    n = ctypes.c_size_t(0)
    assert lib.qlin_sharded_workspace_size(qb._lib.dtype_code(dt), M, K_g, N_g, rank, world, ctypes.byref(n)) == 0
    ws = torch.zeros(max(n.value, 256), dtype=torch.uint8, device=d["x"].device)
    return lib.qlin_sharded_fwd(qb._lib.dtype_code(dt), _ptr(d["x"]), 4 * K_g, *(_ptr(w) for w in d["w"]), K_g,
                                _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, scale, _ptr(y),
                                y.shape[1], M, K_g, N_g, _ptr(ws), n.value, flags, comm, world, r,
                                qb._lib.stream_handle(d["x"].device))


def _slice(lay, d, lo, hi):
    """Output quaternions [lo, hi) of a layer on the device: weight rows, bias and LoRA B rows."""
    out = dict(d)
    out["w"] = [w[lo:hi].contiguous() for w in d["w"]]
    out["bias"] = None if d["bias"] is None else d["bias"][4 * lo:4 * hi].contiguous()
    out["lora_b"] = None if d["lora_b"] is None else d["lora_b"][4 * lo:4 * hi].contiguous()
    return out


@pytest.mark.parametrize("M,rank", [(1, 0), (1, 32), (5, 16), (300, 0)])
def test_world_of_one_matches_the_single_gpu_forward(qb, oracle, workloads, cuda, M, rank):
    lib = qb._lib.load()
    lay = workloads.make_layer("bf16", M, 1024, 2048, 60 + M + rank, bias="normal", lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = 256, 512
    uid = ctypes.create_string_buffer(128)
    assert lib.qlin_nccl_unique_id(uid) == 0
    comm = ctypes.c_void_p()
    assert lib.qlin_nccl_comm_init(ctypes.byref(comm), 1, uid, 0) == 0
    try:
        y = torch.full((M, 4 * N_g + 8), 7.0, dtype=torch.bfloat16, device=cuda)  # ld_y past the columns
        assert _sharded(qb, lib, comm, 1, 0, d, y, M, K_g, N_g, rank, float(d["scale"]), FLAG_ZEROED) == 0
        want = torch.empty(M, 4 * N_g, dtype=torch.bfloat16, device=cuda)
        _forward_slice(qb, lib, d, want, 4 * N_g, M, K_g, N_g, rank, float(d["scale"]), FLAG_ZEROED)
        torch.cuda.synchronize()
        assert torch.equal(y[:, :4 * N_g], want)
        assert bool((y[:, 4 * N_g:] == 7.0).all())  # columns past the layer untouched
        rows = np.arange(min(M, 8))
        assert rel_err(oracle, y[:len(rows), :4 * N_g].float().cpu().numpy(), oracle_rows(oracle, lay, rows)) <= 1e-2
    finally:
        assert lib.qlin_nccl_comm_destroy(comm) == 0
    assert qb.device_error(cuda) == 0


def _two_rank_worker(r, uid, M, rank, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    try:
        import conftest
        import gpu_helpers
        torch.cuda.set_device(r)
        dev = torch.device("cuda", r)
        qb = conftest.load_pkg()
        lib = qb._lib.load()
        wl = conftest.load_submodule("workloads")
        lay = wl.make_layer("bf16", M, 1024, 2048, 90 + M, bias="normal", lora_rank=rank, lora_std=0.02)
        d = gpu_helpers.to_device(lay, dev)
        K_g, N_g = 256, 512
        half = N_g // 2
        mine = _slice(lay, d, r * half, (r + 1) * half)
        comm = ctypes.c_void_p()
        assert lib.qlin_nccl_comm_init(ctypes.byref(comm), 2, uid, r) == 0
        y = torch.empty(M, 4 * N_g, dtype=torch.bfloat16, device=dev)
        st = _sharded(qb, lib, comm, 2, r, mine, y, M, K_g, half, rank, float(d["scale"]), FLAG_ZEROED)
        own = torch.empty(M, 4 * half, dtype=torch.bfloat16, device=dev)
        _forward_slice(qb, lib, mine, own, 4 * half, M, K_g, half, rank, float(d["scale"]), FLAG_ZEROED)
        torch.cuda.synchronize(dev)
        assert lib.qlin_nccl_comm_destroy(comm) == 0
        # numpy (bf16 widened to fp32 exactly): plain pickles, no shared-memory handles
        q.put((r, st, y.float().cpu().numpy(), own.float().cpu().numpy()))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((r, repr(e), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("M,rank", [(1, 32), (16, 0)])
def test_two_ranks_gather_the_full_layer(qb, oracle, workloads, M, rank):
    import multiprocessing as mp
    lib = qb._lib.load()
    uid = ctypes.create_string_buffer(128)
    assert lib.qlin_nccl_unique_id(uid) == 0
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, uid.raw, M, rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, st, y, own = q.get(timeout=300)
        got[r] = (st, y, own)
    for p in procs:
        p.join(timeout=60)
    lay = workloads.make_layer("bf16", M, 1024, 2048, 90 + M, bias="normal", lora_rank=rank, lora_std=0.02)
    want = oracle_rows(oracle, lay)
    half_cols = 4 * 256
    for r in range(2):
        st, y, own = got[r]
        assert st == 0, st
        assert rel_err(oracle, y, want) <= 1e-2
        assert np.array_equal(y[:, r * half_cols:(r + 1) * half_cols], own)
    assert np.array_equal(got[0][1], got[1][1])
