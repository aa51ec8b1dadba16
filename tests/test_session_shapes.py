"""Host logic of the decode session's per-shape step graphs (no GPU).

The tree attention has two launch shapes.  The cluster-merge shape runs while
prefix + tree fit ``short_attention_keys``; the split shape runs beyond.  A
CUDA graph bakes in the shape that was current at capture, so
``DecodeSession`` keeps one graph per shape and picks it from the prefix length
the host last read (``host_start``).  Here the engine and the graph capture are
fakes that record what the session asks of them.
"""
from __future__ import annotations

from dtree_mlx_b200.engine import DecodeSession, Qwen3Engine, StepConfig


class _FakeEngine:
    short_attention_keys = Qwen3Engine.short_attention_keys

    def __init__(self):
        self.keys = []

    def set_attention_keys(self, n):
        self.keys.append(n)


class _FakeGraph:
    def __init__(self, log, cls):
        self.log, self.cls = log, cls

    def replay(self):
        self.log.append(("replay", self.cls))


def _session(n_nodes=25):
    s = DecodeSession.__new__(DecodeSession)  # no device buffers
    s.engine = _FakeEngine()
    s.cfg = StepConfig(mode="dtree", rows=15, budget=n_nodes - 1, n_nodes=n_nodes)
    s.graph = None
    s.graphs = {}
    s.host_start = 0
    s.log = []

    def step():
        cls = s._attention_class()
        s._set_attention_shape(cls)
        s.log.append(("step", cls))

    def capture(cls):
        s._set_attention_shape(cls)
        g = _FakeGraph(s.log, cls)
        s.log.append(("capture", cls))
        s.graph = g
        s.graphs[cls] = g
        return g

    s.step = step
    s._capture = capture
    return s


def test_attention_class_follows_the_key_bound():
    s = _session()
    s.host_start = 999  # 999 + 25 = 1024 keys: still the short shape
    assert s._attention_class() == 1
    s.host_start = 1000  # 1025 keys
    assert s._attention_class() == 0


def test_engine_hint_matches_the_class():
    s = _session()
    s._set_attention_shape(1)
    s._set_attention_shape(0)
    assert s.engine.keys == [1024, 0]


def test_replay_captures_once_per_shape_and_picks_by_start():
    s = _session()
    s.host_start = 256
    s.replay()  # no graph yet: an eager step
    assert s.log == [("step", 1)]
    s.capture_step()
    assert s.log[-1] == ("capture", 1)
    for start in (300, 700, 999):
        s.host_start = start
        s.replay()
    assert s.log[-3:] == [("replay", 1)] * 3
    s.host_start = 1500  # past the bound: the split shape is captured once, then reused
    s.replay()
    s.replay()
    assert s.log[-3:] == [("capture", 0), ("replay", 0), ("replay", 0)]
    assert s.engine.keys[-1] == 0
    s.host_start = 500  # back below: the first graph again, no new capture
    s.replay()
    assert s.log[-1] == ("replay", 1)
    assert sorted(s.graphs) == [0, 1]


def test_dropped_graph_forgets_every_shape():
    s = _session()
    s.host_start = 100
    s.capture_step()
    s.host_start = 2000
    s.replay()
    assert sorted(s.graphs) == [0, 1]
    s.graph = None  # what the runtime does when the drafter changes
    s.replay()  # eager step, the old graphs dropped
    assert s.graphs == {} and s.log[-1] == ("step", 0)
    s.capture_step()
    assert sorted(s.graphs) == [0]


def test_engines_without_shapes_use_one_graph():
    s = _session()
    s.engine = type("E", (), {})()  # a Qwen3.5 engine: no attention shapes, no hint call
    s.host_start = 100
    assert s._attention_class() == 0
    s._set_attention_shape(0)
