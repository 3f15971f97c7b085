"""Gradient sinks of the B200 backend (host-side logic, CPU): where each weight gradient goes in the
flat-buffer, routed and plain modes, and which launch a routed sink asks for."""

from __future__ import annotations

import torch

from cs244c_llama_zero_b200.ops import functional as F


class _Route:
    chunk = 4096
    bases = [1, 2]

    def __init__(self):
        self.pushes = []

    def push(self, src, flat0):
        self.pushes.append((flat0, src.clone()))


def _params(*shapes):
    return [torch.nn.Parameter(torch.zeros(s)) for s in shapes]


def test_flat_buffer_mode_writes_in_place():
    q, k = _params((4, 8), (2, 8))
    main = torch.zeros(48)
    q.main_grad, k.main_grad = main[:32].view(4, 8), main[32:].view(2, 8)
    sink = F._GradSink([q, k])
    assert sink.direct and sink.buffer.shape == (6, 8) and sink.route_of_fused() is None
    sink.buffer.fill_(1.0)
    assert sink.finish() == [None, None] and torch.all(main == 1.0)


def test_routed_mode_pushes_each_weight_at_its_flat_offset():
    q, k, v = _params((4, 8), (2, 8), (2, 8))
    route = _Route()
    for p, off in zip((q, k, v), (64, 96, 112)):
        p.grad_route = (route, off)
    sink = F._GradSink([q, k, v])
    assert not sink.direct
    assert sink.route_of_fused() == (route, 64, 8)  # back to back: one matrix in the flat space
    buf = sink.buffer
    buf.copy_(torch.arange(64, dtype=torch.float32).view(8, 8))
    assert sink.finish() == [None, None, None]
    assert [off for off, _ in route.pushes] == [64, 96, 112]
    assert torch.equal(route.pushes[1][1], torch.arange(32, 48, dtype=torch.float32))


def test_routed_mode_with_a_gap_falls_back_to_the_push():
    q, k = _params((4, 8), (2, 8))
    route = _Route()
    q.grad_route, k.grad_route = (route, 0), (route, 64)  # a gap after q: not one matrix
    sink = F._GradSink([q, k])
    assert sink.route_of_fused() is None
    sink.buffer.fill_(2.0)
    sink.finish()
    assert [off for off, _ in route.pushes] == [0, 64]


def test_routed_sink_asks_for_the_routed_grouped_launch(monkeypatch):
    calls = []

    class Ext:
        def linear_dgrad_wgrad_routed(self, *args):
            calls.append(("routed", args[4:7]))

        def linear_dgrad_wgrad(self, *args):
            calls.append(("plain",))

    monkeypatch.setattr(F, "_ext", lambda: Ext())
    w = torch.nn.Parameter(torch.zeros(16, 8))
    route = _Route()
    w.grad_route = (route, 128)
    sink = F._GradSink([w])
    launcher = F._WgradLauncher(torch.device("cpu"))
    F._dgrad_and_wgrad_sink(None, None, None, None, sink, launcher)
    assert calls == [("routed", (128, 8, 4096))]
    assert sink.finish() == [None] and route.pushes == []  # the epilogue delivered it: nothing to push


def test_plain_mode_hands_gradients_back_to_autograd():
    (w,) = _params((3, 4))
    sink = F._GradSink([w])
    sink.buffer.fill_(0.5)
    (g,) = sink.finish()
    assert g.shape == (3, 4) and torch.all(g == 0.5)
