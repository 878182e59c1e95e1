"""A device-side wait that runs out reports QLIN_ERR_TIMEOUT and leaves the
CUDA context usable.

qlin_forward_allgather is called with a world of two on one GPU.  The
"peer" output and the peer's flag array are local buffers that no other rank
ever writes, so this rank's entry and exit barrier waits both run out after
their 2 s limit.  The kernels must return by themselves, the device error
word must read QLIN_ERR_TIMEOUT, and after clearing it an ordinary call on
the same GPU must be correct and leave the word at zero.  Every access stays
inside the buffers below: the barrier writes slot `slot0 + rank` of the
peer's flag array [2 * world] and polls slots of its own."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import rel_err, to_device

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = 7


def _ptr(t):
    return None if t is None else t.data_ptr()


def test_barrier_wait_runs_out_and_context_stays_usable(qb, oracle, workloads, cuda):
    lib = qb._lib.load()
    code = qb._lib.dtype_code(torch.bfloat16)
    stream = qb._lib.stream_handle(cuda)
    M, fin, fout = 16, 512, 512
    K_g, N_g = fin // 4, fout // 4
    lay = workloads.make_layer("bf16", M, fin, fout, 77, bias="normal")
    d = to_device(lay, cuda)
    assert qb.device_error(cuda) == 0

    world, cols = 2, 2 * fout
    own = torch.zeros(M, cols, dtype=torch.bfloat16, device=cuda)
    peer = torch.zeros(M, cols, dtype=torch.bfloat16, device=cuda)
    own_flags = torch.zeros(2 * world, dtype=torch.int32, device=cuda)
    peer_flags = torch.zeros(2 * world, dtype=torch.int32, device=cuda)  # nobody answers
    epoch = torch.zeros(2, dtype=torch.int32, device=cuda)
    P = ctypes.c_void_p
    outs = (P * world)(own.data_ptr(), peer.data_ptr())
    flags = (P * world)(own_flags.data_ptr(), peer_flags.data_ptr())
    n = qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, 0)
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=cuda)
    st = lib.qlin_forward_allgather(code, _ptr(d["x"]), fin, *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]),
                                    None, None, 0, 0.0, M, K_g, N_g, _ptr(ws), n, 0, world, 0, outs, cols, 0,
                                    flags, _ptr(epoch), stream)
    assert st == 0  # launched; the waits run out on the device
    assert qb.device_error(cuda, clear=True) == ERR_TIMEOUT
    # both barriers signalled the (absent) peer and advanced their counters
    assert own_flags.tolist() == [0, 0, 0, 0]
    assert peer_flags.tolist() == [1, 0, 1, 0]
    assert epoch.tolist() == [1, 1]
    want = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias)
    # the shard kernel still ran between the barriers: own and "peer" outputs hold its columns
    for out in (own, peer):
        assert rel_err(oracle, out[:, :fout].float().cpu().numpy(), want) <= 1e-2
        assert int(out[:, fout:].count_nonzero()) == 0

    # the context is usable: an ordinary call is correct and reports no error
    y = qb.fused_quaternion_linear(d["x"], *d["w"], d["bias"])
    torch.cuda.synchronize()
    assert rel_err(oracle, y.float().cpu().numpy(), want) <= 1e-2
    assert qb.device_error(cuda) == 0
    np.testing.assert_array_equal(own_flags.cpu().numpy(), np.zeros(4, dtype=np.int32))
