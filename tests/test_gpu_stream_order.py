"""Stream-order guarantees of the programmatic dependent launches.

Every kernel of the tensor-core path is launched as a programmatic dependent
of the previous kernel of the stream and waits for it before touching memory;
with static weights it may stream the weights before that.  These tests run
dependent chains (each layer's input is the previous layer's output) eagerly
and inside one CUDA graph, and a weight update immediately followed by a call,
and compare with results computed one synchronised call at a time."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(qb, cuda, n, width, M, lora):
    g = torch.Generator().manual_seed(7)
    out = []
    for _ in range(n):
        w = [(torch.randn(width // 4, width // 4, generator=g) / (width ** 0.5)).to(cuda, torch.bfloat16)
             for _ in range(4)]
        b = (torch.randn(width, generator=g) * 0.05).to(cuda, torch.bfloat16)
        la = lb = None
        if lora:
            la = (torch.randn(16, width, generator=g) * 0.05).to(cuda, torch.bfloat16)
            lb = (torch.randn(width, 16, generator=g) * 0.05).to(cuda, torch.bfloat16)
        out.append((w, b, la, lb))
    x = torch.randn(M, width, generator=g).to(cuda, torch.bfloat16)
    return out, x


def _chain(qb, layers, x, static):
    for w, b, la, lb in layers:
        x = qb.fused_quaternion_linear(x, *w, b, la, lb, 2.0 if la is not None else 0.0,
                                       static_weights=static)
    return x


def _reference(qb, layers, x):
    for w, b, la, lb in layers:
        x = qb.fused_quaternion_linear(x, *w, b, la, lb, 2.0 if la is not None else 0.0)
        torch.cuda.synchronize()
    return x


@pytest.mark.parametrize("M,lora", [(1, False), (16, True), (100, False), (200, True)])
@pytest.mark.parametrize("static", [False, True])
def test_dependent_chain_eager_and_graph(qb, cuda, M, lora, static):
    layers, x = _layers(qb, cuda, 12, 512, M, lora)
    want = _reference(qb, layers, x)
    got = _chain(qb, layers, x, static)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # the same chain captured in one graph and replayed
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _chain(qb, layers, x, static)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = _chain(qb, layers, x, static)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert qb.device_error(cuda) == 0


@pytest.mark.parametrize("M", [1, 16, 130])
def test_weight_update_right_before_call_is_seen(qb, cuda, M):
    g = torch.Generator().manual_seed(3)
    w = [(torch.randn(128, 128, generator=g) / 16).to(cuda, torch.bfloat16) for _ in range(4)]
    x = torch.randn(M, 512, generator=g).to(cuda, torch.bfloat16)
    w2 = [a * -0.5 + 0.01 for a in w]
    want = qb.quaternion_linear(x, *w2)
    torch.cuda.synchronize()
    y1 = qb.quaternion_linear(x, *w)  # a first call, then an in-place update on the stream
    for a, b in zip(w, w2):
        a.copy_(b)
    y2 = qb.quaternion_linear(x, *w)  # must see the updated weights
    torch.cuda.synchronize()
    assert torch.equal(y2, want)
    assert not torch.equal(y1, y2)


def test_plan_reports_the_decode_split(qb, cuda):
    # one kernel: the LoRA rank <= 32 down projection runs inside it and its
    # 8-way K split is summed inside a thread-block cluster, whatever the
    # workspace; without LoRA the same.  A rank-64 LoRA adds the prologue.
    plan = qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 32, flags=0)
    assert plan["algo"] == "tcgen05" and plan["tile_tokens"] == 16
    assert plan["split_k"] == 8 and plan["launches"] == 1
    assert qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 64, flags=0)["launches"] == 2
    assert qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 0, flags=0)["launches"] == 1
