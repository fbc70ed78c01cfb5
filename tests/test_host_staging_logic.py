"""HostStaging's slot rotation and stream ordering, on the CPU.

torch.cuda's Stream / Event / stream context are replaced by fakes that log
every record and wait, and the tensors are CPU tensors, so the test checks the
host logic without a GPU: which slot each layer-step uses, that a slot is
refilled only after the layer-step that read it released it, that the
current stream waits for a slot's copy before using it, that the copy-out
waits for the layer-step's work, and that calls out of order are refused.
"""
from __future__ import annotations

import contextlib

import pytest
import torch

LOG: list = []


class FakeEvent:
    n = 0

    def __init__(self, *a, **k):
        FakeEvent.n += 1
        self.name = f"e{FakeEvent.n}"
        self.records = 0

    def record(self, stream=None):
        self.records += 1
        LOG.append(("record", self.name, getattr(stream, "name", None)))

    def synchronize(self):
        pass


class FakeStream:
    def __init__(self, name):
        self.name = name

    def wait_event(self, ev):
        LOG.append(("wait", self.name, ev.name, ev.records))

    def synchronize(self):
        pass


MAIN = FakeStream("main")


@pytest.fixture
def staging(monkeypatch):
    from pyramidkv import host_staging
    names = iter(["copy_in", "copy_out"])
    monkeypatch.setattr(torch.cuda, "Stream", lambda *a, **k: FakeStream(next(names)))
    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: MAIN)
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.Tensor, "record_stream", lambda self, s: None)
    LOG.clear()
    return host_staging.HostStaging


def test_slots_rotate_and_carry_the_data(staging):
    like = [torch.zeros(3, 4), torch.zeros(3, 4)]
    st = staging(like, "cpu", depth=2)
    steps = [[torch.full((3, 4), float(10 * i + k)) for k in range(2)] for i in range(5)]
    outs = [torch.empty(3, 4) for _ in steps]
    st.put(steps[0])
    used = []
    for i in range(len(steps)):
        if i + 1 < len(steps):
            st.put(steps[i + 1])
        a, b = st.get()
        used.append(id(a))
        assert torch.equal(a, steps[i][0]) and torch.equal(b, steps[i][1])
        st.done(a + b, outs[i])
    for i, o in enumerate(outs):
        assert torch.equal(o, steps[i][0] + steps[i][1])
    # two device slots, used alternately
    assert used[0] == used[2] == used[4] and used[1] == used[3] and used[0] != used[1]


def test_stream_ordering(staging):
    x = torch.zeros(2)
    st = staging([x], "cpu", depth=2)
    ready = [e.name for e in st.ready]
    free = [e.name for e in st.free]
    st.put([x])
    st.put([x])
    st.get()
    st.done(x.clone(), torch.empty(2))
    LOG.clear()
    st.put([x])  # slot 0 again: must wait for the release recorded by done()
    assert LOG[0] == ("wait", "copy_in", free[0], 1)
    assert LOG[-1] == ("record", ready[0], "copy_in")
    LOG.clear()
    st.get()  # step 1 uses slot 1: the current stream waits for its copy
    assert LOG == [("wait", "main", ready[1], 1)]
    LOG.clear()
    st.done(x.clone(), torch.empty(2))
    # release recorded on the current stream, copy-out waits for it
    assert LOG[0] == ("record", free[1], "main")
    assert LOG[1] == ("wait", "copy_out", free[1], 1)
    assert LOG[-1][0] == "record" and LOG[-1][2] == "copy_out"


def test_refuses_calls_out_of_order(staging):
    x = torch.zeros(2)
    st = staging([x], "cpu", depth=2)
    with pytest.raises(RuntimeError):
        st.get()
    with pytest.raises(RuntimeError):
        st.done(x, torch.empty(2))
    st.put([x])
    st.put([x])
    with pytest.raises(RuntimeError):
        st.put([x])
    st.get()
    with pytest.raises(RuntimeError):
        st.get()
    with pytest.raises(ValueError):
        staging([x], "cpu", depth=0)
