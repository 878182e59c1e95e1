"""Column-partitioned layer on two GPUs (skipped with fewer).

Each rank holds half of the output quaternion rows.  The NCCL path (shard
kernel, all-gather, column gather) and the fused paths (the shard kernel's
epilogue stores into every rank's output over NVLink, then a bounded flag
barrier: peer stores, qlin_forward_allgather, and -- where NVLink multicast
is available -- one multicast store per piece, qlin_forward_allgather_mc)
must give the same [M, out] output on every rank, agreeing with each other (to fp32 summation order: the two paths may
run different device kernels) and within the bf16 tolerance of the
unpartitioned layer.  Output widths that do not divide by the world size exercise the
padded last shard; repeated calls exercise the barriers' call counters, and
back-to-back calls on different inputs the entry barrier (no rank overwrites
a peer's output before that peer has copied out the previous result).
Ranks are child processes (spawn) with a short process-group timeout; the
parent bounds their lifetime."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_q):
    import datetime
    import importlib
    import sys

    import torch.distributed as dist

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if repo not in sys.path:
        sys.path.insert(0, repo)
    qb = importlib.import_module("quaternion-based-math-1_b200")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = False
    try:
        results = []
        # the last case runs the fused path on the CTA-pair kernel (no LoRA, > 64 tokens)
        for (M, fin, fout, rank_l) in [(1, 1024, 1024, 16), (16, 512, 520, 0), (300, 768, 1040, 8),
                                       (600, 512, 2080, 0)]:
            g = torch.Generator().manual_seed(fin + fout)
            full = qb.QuaternionLinear(fin, fout, bias=True, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                for n in ("wr", "wi", "wj", "wk"):
                    getattr(full, n).copy_(torch.randn(fout // 4, fin // 4, generator=g) / (fin ** 0.5))
                full.bias.copy_(torch.randn(fout, generator=g) * 0.02)
            la = lb = None
            scale = 0.0
            if rank_l:
                la = (torch.randn(rank_l, fin, generator=g) * 0.05).to(dev, torch.bfloat16)
                lb = (torch.randn(fout, rank_l, generator=g) * 0.05).to(dev, torch.bfloat16)
                scale = 2.0
            x = torch.randn(M, fin, generator=g).to(dev, torch.bfloat16)
            want = qb.fused_quaternion_linear(x, full.wr, full.wi, full.wj, full.wk, full.bias, la, lb, scale)
            plain = qb.ColumnParallelQuaternionLinear.from_full(full, lora_A=la, lora_B=lb, lora_scale=scale)
            plain.fused_allgather = False
            fused = qb.ColumnParallelQuaternionLinear.from_full(full, lora_A=la, lora_B=lb, lora_scale=scale)
            fused.fused_allgather = True  # multicast stores where available
            peer = qb.ColumnParallelQuaternionLinear.from_full(full, lora_A=la, lora_B=lb, lora_scale=scale)
            peer.fused_allgather = True
            peer._multicast = False  # peer stores
            for _ in range(3):
                y_plain = plain(x)
                y_fused = fused(x)
                y_peer = peer(x)
            torch.cuda.synchronize()
            # the same kernels on the same inputs: the two fused paths agree bit for bit
            same_fused = bool(torch.equal(y_fused, y_peer))
            err = ((y_fused.float() - want.float()).norm() / want.float().norm()).item()
            # the NCCL path's per-shard calls may run the decode GEMV (1-2
            # tokens), the fused path the tensor-core kernel: fp32 summation
            # order differs, so agreement, not bit equality
            diff = ((y_plain.float() - y_fused.float()).norm() / y_fused.float().norm()).item()
            # back-to-back fused calls on different inputs, no host sync in
            # between: each call's stores into a peer's output must wait
            # until that peer has copied out the previous call's result
            xs = [torch.randn(M, fin, generator=g).to(dev, torch.bfloat16) for _ in range(4)]
            wants = [qb.fused_quaternion_linear(xi, full.wr, full.wi, full.wj, full.wk, full.bias, la, lb, scale)
                     for xi in xs]
            gots = [fused(xi) for xi in xs]
            torch.cuda.synchronize()
            for gi, wi in zip(gots, wants):
                e = ((gi.float() - wi.float()).norm() / wi.float().norm()).item()
                err = max(err, e)
            results.append((M, fout, diff <= 4e-3 and same_fused, err, bool(fused._multicast)))
        results.append(("device_error", qb.device_error(dev)))
        out_q.put((rank, results))
        ok = True
    except BaseException as e:  # report at once: the parent must not wait for a timeout
        out_q.put((rank, f"error: {e!r}"))
        raise
    finally:
        if ok:
            dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs two GPUs")
def test_column_partition_fused_allgather_matches_nccl_path():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(WORLD):
            r, res = q.get(timeout=180)
            got[r] = res
            if isinstance(res, str):
                break
    finally:
        for p in procs:
            p.join(timeout=90 if all(not isinstance(v, str) for v in got.values()) else 5)
            if p.is_alive():
                p.kill()
    errors = {r: v for r, v in got.items() if isinstance(v, str)}
    assert not errors, errors
    assert sorted(got) == list(range(WORLD))
    for r, res in got.items():
        *cases, (_, dev_err) = res
        assert dev_err == 0, (r, dev_err)
        for M, fout, same, err, _multicast in cases:
            assert same, (r, M, fout)
            assert err <= 1e-2, (r, M, fout, err)
