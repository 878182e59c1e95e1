"""Column-partitioned layer, host logic on CPU with world_size-2 gloo ranks.

The per-rank quaternion product runs on the device in production; here each
rank's local product is computed by the oracle (test-only stand-in, patched
into the module) so that the partitioning, padding, the all-gather order and
the column reassembly are checked end to end without a GPU."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ORACLE_DIR, REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_groups, M, result_path):
    import importlib
    import sys

    sys.path.insert(0, REPO)
    sys.path.insert(0, ORACLE_DIR)
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    qb = importlib.import_module("quaternion-based-math-1_b200")
    sh = importlib.import_module("quaternion-based-math-1_b200.sharded")
    g = torch.Generator().manual_seed(123)
    in_f, out_f = 48, 4 * out_groups
    full = qb.QuaternionLinear(in_f, out_f, bias=True)
    with torch.no_grad():
        for p in (full.wr, full.wi, full.wj, full.wk, full.bias):
            p.copy_(torch.randn(p.shape, generator=g))
    x = torch.randn(M, in_f, generator=g)
    layer = sh.ColumnParallelQuaternionLinear.from_full(full, world_size=world, rank=rank)

    def local_forward(xx):  # oracle stand-in for the device kernel
        y = O.forward_rows(xx.numpy(), *(t.detach().numpy() for t in (layer.wr, layer.wi, layer.wj,
                                                                        layer.wk)),
                           bias=layer.bias.detach().numpy())
        return torch.from_numpy(y).float()

    def gather_cpu(buf, m, n):
        return buf.permute(1, 0, 2).reshape(m, -1)

    layer.local_forward = local_forward
    sh.gather_columns = gather_cpu
    y = layer(x)
    want = O.forward_rows(x.numpy(), *(t.detach().numpy() for t in (full.wr, full.wi, full.wj, full.wk)),
                          bias=full.bias.detach().numpy())
    err = float(np.abs(y.numpy() - want).max())
    dist.barrier()
    dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as f:
        f.write(f"{tuple(y.shape)} {err}")


@pytest.mark.parametrize("out_groups,M", [(12, 5), (7, 1), (9, 3)])
def test_two_rank_column_partition(tmp_path, out_groups, M):
    world = 2
    port = _free_port()
    path = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, out_groups, M, path))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        shape, err = open(f"{path}.{r}").read().rsplit(" ", 1)
        assert shape == str((M, 4 * out_groups))
        assert float(err) < 1e-4
