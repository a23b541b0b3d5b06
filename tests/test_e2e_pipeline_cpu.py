"""bench.e2e_pipelined on CPU with fake streams and events: every step copies
each layer's input in, runs the layer and copies its output out; a device
input buffer is refilled only after the forward that read it; each layer's next
forward waits for the previous output's copy out; the compute stream waits for
the last copy out before the end event."""

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
    # The copy-in stream starts after the start event, then waits, for every
    # refill after the first step, on the forward that read the buffer.
    waits_in = [e for op, e in s_in.log if op == "wait"]
    assert len(waits_in) == 1 + 3 * (steps - 1)
    assert all(e.stream is cu.comp for e in waits_in)
    # Each copy out waits for its forward; compute waits for each landed input,
    # for the previous copy out of the same layer before every later forward,
    # and, at the end, for the last copy out.
    waits_out = [e for op, e in s_out.log if op == "wait"]
    assert len(waits_out) == 3 * steps and all(e.stream is cu.comp for e in waits_out)
    waits_comp = [e for op, e in cu.comp.log if op == "wait"]
    assert len(waits_comp) == 3 * steps + 3 * (steps - 1) + 1
    assert waits_comp[-1].stream is s_out
    assert sum(e.stream is s_in for e in waits_comp) == 3 * steps
    assert sum(e.stream is s_out for e in waits_comp) == 3 * (steps - 1) + 1


def test_e2e_report_never_slower_than_serial():
    """The reported end-to-end figure is the faster verified mode, and the mode
    names the figure reported."""
    cases = [(3.88, 6.92, True), (3.88, 2.10, True), (3.88, 2.10, False), (2.0, 2.0, True)]
    for serial, pipe, ok in cases:
        ms, mode, note = bench.choose_e2e(serial, pipe, ok)
        assert ms <= serial
        if ok and pipe <= serial:
            assert ms == pipe and mode.startswith("copies overlapped") and note is None
        else:
            assert ms == serial and mode.startswith("serial") and note
    # A failure note from the caller is kept.
    assert bench.choose_e2e(1.0, 0.5, False, "boom")[2] == "boom"


def test_parity_sample_indices():
    assert bench.sample_indices(128) == [0, 1, 126, 127]
    assert bench.sample_indices(1) == [0]
    assert bench.sample_indices(2) == [0, 1]
    assert bench.sample_indices(3) == [0, 1, 2]


def test_sample_parity_flags_a_wrong_output():
    import numpy as np
    import nova_oracle as o
    x, w = o.synthetic_case(4, 8, 8, 12, 12, seed=3)
    y = o.nova_forward(x, w, 1, "ref")
    xt, wt = torch.from_numpy(x), torch.from_numpy(w)
    good = bench.sample_parity("t", xt, wt, torch.from_numpy(y))
    assert good["ok"] and good["rel_l2_vs_oracle"] == 0.0 and good["images"] == [0, 1, 2, 3]
    bad = y.copy()
    bad[3, :, 5, 5] += np.float16(1.0)
    assert not bench.sample_parity("t", xt, wt, torch.from_numpy(bad))["ok"]
