"""bench.e2e_pipelined on CPU with fake streams and events: every step copies
each layer's input in, runs the layer and copies its output out; a device
input buffer is refilled only after the forward that read it; every output is
kept alive on the copy-out stream; the compute stream waits for the last copy
out before the end event."""

import contextlib
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


class FakeEvent:
    def __init__(self, timing):
        self.timing = timing
        self.stream = None

    def record(self, stream):
        self.stream = stream
        stream.log.append(("record", self))

    def elapsed_time(self, other):
        assert self.timing and other.timing
        return 7.5


class FakeStream:
    def __init__(self, name):
        self.name = name
        self.log = []

    def wait_event(self, ev):
        assert ev.stream is not None, "waiting on an event that was never recorded"
        self.log.append(("wait", ev))


class FakeCuda:
    def __init__(self):
        self.comp = FakeStream("compute")
        self.made = []
        self.kept = []
        self.active = [self.comp]

    def stream(self):
        s = FakeStream(f"side{len(self.made)}")
        self.made.append(s)
        return s

    def current(self):
        return self.comp

    def event(self, timing=False):
        return FakeEvent(timing)

    @contextlib.contextmanager
    def use(self, stream):
        self.active.append(stream)
        try:
            yield
        finally:
            self.active.pop()

    def keep_alive(self, tensor, stream):
        self.kept.append((tensor, stream))

    def synchronize(self):
        pass


def test_pipelined_e2e_outputs_and_ordering():
    torch.manual_seed(0)
    hx = [torch.randn(2, 3), torch.randn(4), torch.randn(1, 5)]
    dx = [torch.zeros_like(t) for t in hx]
    hy = [torch.zeros_like(t) for t in hx]
    calls = []

    def make(k):
        def fwd(t):
            calls.append(k)
            return t * (k + 2) + 1
        return fwd

    fwds = [make(k) for k in range(3)]
    cu = FakeCuda()
    steps = 4
    ms = bench.e2e_pipelined(hx, dx, hy, fwds, steps, cu)
    assert ms == 7.5
    for k in range(3):
        assert torch.equal(hy[k], hx[k] * (k + 2) + 1)
    assert calls == [0, 1, 2] * steps
    s_in, s_out = cu.made
    # Every output stays alive on the copy-out stream.
    assert len(cu.kept) == 3 * steps and all(s is s_out for _, s in cu.kept)
    # The copy-in stream starts after the start event, then waits, for every
    # refill after the first step, on the forward that read the buffer.
    waits_in = [e for op, e in s_in.log if op == "wait"]
    assert len(waits_in) == 1 + 3 * (steps - 1)
    assert all(e.stream is cu.comp for e in waits_in)
    # Each copy out waits for its forward; compute waits for each landed input
    # and, at the end, for the last copy out.
    waits_out = [e for op, e in s_out.log if op == "wait"]
    assert len(waits_out) == 3 * steps and all(e.stream is cu.comp for e in waits_out)
    waits_comp = [e for op, e in cu.comp.log if op == "wait"]
    assert len(waits_comp) == 3 * steps + 1
    assert waits_comp[-1].stream is s_out
    assert all(e.stream is s_in for e in waits_comp[:-1])
