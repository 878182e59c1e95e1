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


@pytest.mark.parametrize("M,lora", [(1, False), (1, True), (2, True), (3, True), (4, True), (16, True),
                                    (100, False), (200, True), (300, False)])
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
    # checked after the first replay: later replays would find each layer's
    # input already holding the right values and could hide a layer that
    # reads its input before the previous layer has written it
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


@pytest.mark.parametrize("M2,lora", [(1, False), (1, True), (2, False), (16, False), (130, False)])
def test_weights_written_by_the_previous_call_are_seen(qb, cuda, M2, lora):
    # call 1 (a decode call of this library) writes its output into the buffer
    # that call 2 reads as its weight wr; call 2 is launched right behind it
    # and must not read wr before call 1 has finished (no static weights)
    g = torch.Generator().manual_seed(9)
    w1 = [(torch.randn(1024, 256, generator=g) / 32).to(cuda, torch.bfloat16) for _ in range(4)]
    x1 = torch.randn(1, 1024, generator=g).to(cuda, torch.bfloat16)
    wr2 = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda)  # call 1's output = call 2's wr [64, 64]
    w2 = [(torch.randn(64, 64, generator=g) / 16).to(cuda, torch.bfloat16) for _ in range(3)]
    x2 = torch.randn(M2, 256, generator=g).to(cuda, torch.bfloat16)
    la = lb = None
    if lora:
        la = (torch.randn(16, 256, generator=g) * 0.05).to(cuda, torch.bfloat16)
        lb = (torch.randn(256, 16, generator=g) * 0.05).to(cuda, torch.bfloat16)
    scale = 2.0 if lora else 0.0

    def two_calls():
        wr2.zero_()
        y1 = qb.fused_quaternion_linear(x1, *w1)
        wr2.copy_(y1)  # (a copy kernel in between, as a framework would issue)
        return qb.fused_quaternion_linear(x2, wr2.view(64, 64), *w2, None, la, lb, scale)

    def two_calls_direct():
        wr2.zero_()
        # call 1 stores straight into wr2: call 2 directly follows the kernel
        # that writes its weights (a programmatic dependent launch)
        ws, ld = qb.linear._weights(tuple(w1))
        qb._lib.forward_raw(x1, 1024, ws, ld, None, None, None, 0, 0.0, wr2, 4096, 1, 256, 1024)
        return qb.fused_quaternion_linear(x2, wr2.view(64, 64), *w2, None, la, lb, scale)

    y1 = qb.fused_quaternion_linear(x1, *w1)
    torch.cuda.synchronize()
    want = qb.fused_quaternion_linear(x2, y1.view(64, 64).clone(), *w2, None, la, lb, scale)
    torch.cuda.synchronize()
    for fn in (two_calls, two_calls_direct):
        for _ in range(3):
            got = fn()
            torch.cuda.synchronize()
            assert torch.equal(got, want), fn.__name__
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want), fn.__name__
        del graph
    assert qb.device_error(cuda) == 0


@pytest.mark.parametrize("M,lora", [(1, False), (1, True), (2, False), (16, True), (130, False)])
def test_inputs_rewritten_every_replay_are_seen(qb, cuda, M, lora):
    # a graph whose first node rewrites x0 in place every replay, then two
    # calls where call 2 reads call 1's output as its input: every replay's
    # outputs must follow the new x0 (no stale cached lines of an earlier
    # replay's values)
    layers, x0 = _layers(qb, cuda, 2, 512, M, lora)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _chain(qb, layers, x0, False)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        x0.mul_(-1.5)
        out = _chain(qb, layers, x0, False)
    for _ in range(4):
        graph.replay()
        torch.cuda.synchronize()
        want = _reference(qb, layers, x0.clone())
        assert torch.equal(out, want)
    del graph
    assert qb.device_error(cuda) == 0


def test_plan_reports_the_decode_split(qb, cuda):
    # decode calls: the CUDA-core decode kernel, after the LoRA down-projection
    # prologue when there is a rank <= 32 LoRA; a rank-64 LoRA goes to the
    # tensor-core kernel and its prologue
    plan = qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 32, flags=0)
    assert plan["algo"] == "gemv" and plan["tile_tokens"] == 1
    assert plan["split_k"] == 1 and plan["launches"] == 2
    assert qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 64, flags=0)["launches"] == 2
    assert qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 0, flags=0)["launches"] == 1


def test_graph_replay_after_zeroed_workspace_grows(qb, cuda):
    """Decode-sized calls use a zero-filled workspace kept per stream.  A
    graph captured while the stream's buffer was small must still replay
    correctly after a larger layer made that buffer grow: the superseded
    buffer stays alive (its memory is not handed to other tensors)."""
    small, x = _layers(qb, cuda, 2, 512, 3, True)
    big, xb = _layers(qb, cuda, 1, 4096, 4, True)
    want = _reference(qb, small, x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.no_grad():
        with torch.cuda.stream(s):
            _chain(qb, small, x, False)  # creates the stream's zero-filled buffer
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out = _chain(qb, small, x, False)
        with torch.cuda.stream(s):
            _chain(qb, big, xb, False)  # needs a larger buffer: the small one is replaced
        s.synchronize()
        # fill whatever memory the allocator hands out now with non-zero bytes
        junk = [torch.full((1 << 16,), 255, dtype=torch.uint8, device=cuda) for _ in range(64)]
        torch.cuda.synchronize()
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
    del junk, graph
    assert qb.device_error(cuda) == 0
