"""Generate golden vectors by running the REFERENCE's own Python functions.

MLX is not installable in this container, so this script installs a small
NumPy-backed stand-in for the handful of ``mlx.core`` calls the tree code
uses (``array``, ``argpartition``, ``take_along_axis``, ``argsort``,
``logsumexp``, ``take`` ...) plus inert placeholder modules for the imports
the reference pulls in at module load (mlx.nn, mlx_lm, huggingface_hub).
It then imports ``dtree_mlx`` from the reference checkout and calls, unchanged:

* ``dtree_runtime.build_dtree_tree``       (dtree_runtime.py:82-163)
* ``dtree_runtime.follow_verified_tree``   (dtree_runtime.py:195-208)
* ``qwen35_tree.build_node_lineages``      (qwen35_tree.py:41-55)
* ``qwen35_tree._tree_depth_groups``       (qwen35_tree.py:104-123)
* ``adapters.Qwen3TargetAdapter.compact_kv_caches`` (adapters.py:635-668)
* ``runtime.longest_prefix_match``         (runtime.py:33-39)

The outputs are written to ``tests/golden/tree_golden.json``,
``tests/golden/tree_logits.npz`` (the draft logits of each tree case) and
``tests/golden/compact_golden.npz``.  The product never reads these files; the
tests compare the oracle (and, on a GPU, the CUDA kernels) against them.

Usage (needs the reference checkout; run from the repo root):
    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


# --------------------------------------------------------------------------
# NumPy-backed stand-in for the subset of mlx.core used on the tree path
# --------------------------------------------------------------------------
class _Arr:
    __slots__ = ("a",)

    def __init__(self, a):
        self.a = np.asarray(a)

    # numpy interop / introspection
    def __array__(self, dtype=None, copy=None):
        return self.a if dtype is None else self.a.astype(dtype)

    @property
    def shape(self):
        return tuple(self.a.shape)

    @property
    def ndim(self):
        return self.a.ndim

    @property
    def dtype(self):
        return self.a.dtype

    def astype(self, dtype):
        return _Arr(self.a.astype(dtype))

    def tolist(self):
        return self.a.tolist()

    def item(self):
        return self.a.item()

    def __getitem__(self, idx):
        if isinstance(idx, tuple):
            idx = tuple(i.a if isinstance(i, _Arr) else i for i in idx)
        elif isinstance(idx, _Arr):
            idx = idx.a
        return _Arr(self.a[idx])

    def __setitem__(self, idx, value):
        v = value.a if isinstance(value, _Arr) else value
        self.a[idx] = v

    def _bin(self, other, op):
        o = other.a if isinstance(other, _Arr) else other
        return _Arr(op(self.a, o))

    def __sub__(self, o):
        return self._bin(o, np.subtract)

    def __add__(self, o):
        return self._bin(o, np.add)

    def __neg__(self):
        return _Arr(-self.a)

    def __len__(self):
        return len(self.a)


def _unwrap(x):
    return x.a if isinstance(x, _Arr) else x


def _make_mx():
    mx = types.ModuleType("mlx.core")
    mx.float32 = np.float32
    mx.float16 = np.float16
    mx.bfloat16 = np.float32  # only used as a dtype tag on unexercised paths
    mx.bool_ = np.bool_
    mx.uint32 = np.uint32
    mx.int32 = np.int32
    mx.int64 = np.int64
    class array:  # a class, so module-level ``mx.array | None`` annotations work
        def __new__(cls, obj, dtype=None):
            return _Arr(np.array(_unwrap(obj), dtype=dtype))

    mx.array = array
    mx.argpartition = lambda a, kth, axis=-1: _Arr(np.argpartition(_unwrap(a), kth, axis=axis))
    mx.take_along_axis = lambda a, idx, axis: _Arr(
        np.take_along_axis(_unwrap(a), _unwrap(idx), axis=axis)
    )
    mx.argsort = lambda a, axis=-1: _Arr(np.argsort(_unwrap(a), axis=axis, kind="stable"))

    def _logsumexp(a, axis=None, keepdims=False):
        x = _unwrap(a)
        m = np.max(x, axis=axis, keepdims=True)
        s = np.log(np.sum(np.exp(x - m), axis=axis, keepdims=True)) + m
        if not keepdims:
            s = np.squeeze(s, axis=axis)
        return _Arr(s.astype(x.dtype))

    mx.logsumexp = _logsumexp
    mx.take = lambda a, idx, axis=None: _Arr(np.take(_unwrap(a), _unwrap(idx), axis=axis))
    mx.zeros = lambda shape, dtype=np.float32: _Arr(np.zeros(shape, dtype=dtype))
    mx.ones = lambda shape, dtype=np.float32: _Arr(np.ones(shape, dtype=dtype))
    mx.eval = lambda *a, **k: None
    mx.compile = lambda f: f
    mx.default_device = lambda: "cpu"
    mx.gpu = "gpu"
    mx.cpu = "cpu"
    mx.metal = types.SimpleNamespace(is_available=lambda: False)
    mx.fast = types.SimpleNamespace()
    mx.distributed = types.SimpleNamespace()
    return mx


class _KVCache:
    """NumPy stand-in for mlx_lm KVCache with the fields compact_kv_caches uses."""

    def __init__(self, keys, values, offset):
        self.keys = _Arr(keys)
        self.values = _Arr(values)
        self.offset = offset


class _Inert(types.ModuleType):
    """Module placeholder: any attribute is an inert class/callable."""

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        sub = f"{self.__name__}.{name}"
        if sub in sys.modules:
            return sys.modules[sub]
        return type(name, (), {"__init__": lambda self, *a, **k: None})


class _ShimFinder:
    """Meta-path finder: any not-yet-installed mlx / mlx_lm / huggingface_hub
    submodule resolves to an inert placeholder package."""

    prefixes = ("mlx", "mlx_lm", "huggingface_hub")

    def find_spec(self, fullname, path=None, target=None):
        import importlib.machinery

        if fullname.split(".")[0] in self.prefixes and fullname not in sys.modules:
            return importlib.machinery.ModuleSpec(fullname, self, is_package=True)
        return None

    def create_module(self, spec):
        mod = _Inert(spec.name)
        mod.__path__ = []
        return mod

    def exec_module(self, module):
        return None


def install_shims():
    mx = _make_mx()
    mlx = types.ModuleType("mlx")
    mlx.__path__ = []
    mlx.core = mx
    nn = _Inert("mlx.nn")
    nn.__path__ = []
    nn.Module = type("Module", (), {})
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = mx
    sys.modules["mlx.nn"] = nn
    sys.meta_path.insert(0, _ShimFinder())
    import importlib

    cache_mod = importlib.import_module("mlx_lm.models.cache")
    cache_mod.KVCache = _KVCache


# --------------------------------------------------------------------------
# golden cases
# --------------------------------------------------------------------------
def dirichlet_logits(rng, rows, vocab, support=32, alpha=0.1):
    """Draft log-probs sampled from Dirichlet(alpha) over a random top-`support`
    set; every other token gets a large negative logit."""
    logits = np.full((rows, vocab), -30.0, dtype=np.float32)
    for r in range(rows):
        ids = rng.choice(vocab, size=support, replace=False)
        p = rng.dirichlet(np.full(support, alpha))
        logits[r, ids] = np.log(np.maximum(p, 1e-30)).astype(np.float32)
    return logits


def planted_like_logits(rng, rows, vocab, p_correct=0.8):
    logits = rng.standard_normal((rows, vocab)).astype(np.float32)
    for r in range(rows):
        tok = rng.integers(vocab)
        logits[r, tok] += 8.0
    return logits


def main(reference: str) -> None:
    install_shims()
    sys.path.insert(0, str(Path(reference).resolve()))
    from dtree_mlx import dtree_runtime, qwen35_tree, runtime  # noqa: E402
    from dtree_mlx.adapters import Qwen3TargetAdapter  # noqa: E402

    cases = []
    logits_store: dict[str, np.ndarray] = {}

    def run_tree(name, logits, budget):
        tokens, depths, parents, child_maps, vis, _ = dtree_runtime.build_dtree_tree(
            _Arr(logits), budget
        )
        # the top-k log-probs the heap consumed, recomputed the reference's way
        lg = logits.astype(np.float32)
        k = max(min(budget, lg.shape[-1]), 1)
        part = np.argpartition(lg, lg.shape[-1] - k, axis=-1)[:, -k:]
        tl = np.take_along_axis(lg, part, axis=-1)
        order = np.argsort(-tl, axis=-1, kind="stable")
        top_ids = np.take_along_axis(part, order, axis=-1)
        tl = np.take_along_axis(tl, order, axis=-1)
        m = lg.max(axis=-1, keepdims=True)
        lse = (np.log(np.sum(np.exp(lg - m), axis=-1, keepdims=True)) + m).astype(np.float32)
        top_lp = (tl - lse).astype(np.float32)
        cases.append(
            {
                "name": name,
                "budget": int(budget),
                "logits_shape": list(logits.shape),
                "top_ids": top_ids.tolist(),
                "top_log_probs": top_lp.tolist(),
                "node_token_ids": [int(t) for t in tokens],
                "node_depths": [int(d) for d in depths],
                "parents": [int(p) for p in parents],
                "child_maps": [{str(k): int(v) for k, v in cm.items()} for cm in child_maps],
                "visibility": np.asarray(vis).astype(np.uint8).tolist(),
            }
        )
        logits_store[name] = logits.astype(np.float32)
        return parents, tokens, child_maps

    # 1. the reference's own unit-test input (tests/test_dtree_runtime.py:15-40)
    run_tree(
        "ref_unit_3x3_b4",
        np.array([[5.0, 4.0, 1.0], [6.0, 2.0, 1.0], [7.0, 3.0, 1.0]], dtype=np.float32),
        4,
    )
    rng = np.random.default_rng(20261201)
    # 2. Dirichlet(0.1) over top-32 (the isolated-verify sweep's topology source)
    for budget in (8, 24, 64):
        for s in range(3):
            run_tree(f"dirichlet_b{budget}_s{s}", dirichlet_logits(rng, 16, 1024), budget)
    # 3. planted-style logits (N(0,1) + 8 spike), 15 draft rows like spec=16
    for s in range(3):
        run_tree(f"planted_b24_s{s}", planted_like_logits(rng, 15, 2048), 24)
    # 4. shallow / edge cases
    run_tree("one_row_b5", rng.standard_normal((1, 64)).astype(np.float32), 5)
    run_tree("budget_gt_vocab", rng.standard_normal((4, 6)).astype(np.float32), 10)
    run_tree("budget_zero", rng.standard_normal((4, 16)).astype(np.float32), 0)

    # walk: random posteriors over every generated tree, plus the unit KAT
    walks = []
    walk_rng = np.random.default_rng(7)
    for case in cases:
        child_maps = [{int(k): v for k, v in cm.items()} for cm in case["child_maps"]]
        n = len(case["parents"])
        tree_tokens = [0] + case["node_token_ids"]
        for _ in range(4):
            post = []
            for i in range(n):
                kids = list(child_maps[i].keys())
                if kids and walk_rng.random() < 0.85:
                    post.append(int(kids[walk_rng.integers(len(kids))]))
                else:
                    post.append(int(walk_rng.integers(100000)))
            acc, nxt = dtree_runtime.follow_verified_tree(child_maps, post)
            walks.append(
                {
                    "case": case["name"],
                    "parents": case["parents"],
                    "tree_tokens": tree_tokens,
                    "posterior": post,
                    "accepted": [int(a) for a in acc],
                    "next_token": int(nxt),
                }
            )
    unit_walk = dtree_runtime.follow_verified_tree(
        [{11: 1, 12: 2}, {21: 3}, {}, {}], [11, 21, 99, 0]
    )

    # lineages + depth groups
    lineages = []
    lin_rng = np.random.default_rng(11)
    parent_sets = [[-1, 0, 0, 1, 3, 2]] + [c["parents"] for c in cases]
    for _ in range(5):
        n = int(lin_rng.integers(2, 40))
        parent_sets.append([-1] + [int(lin_rng.integers(i)) for i in range(1, n)])
    for ps in parent_sets:
        lineages.append(
            {
                "parents": ps,
                "lineages": qwen35_tree.build_node_lineages(ps),
                "depth_groups": qwen35_tree._tree_depth_groups(ps),
            }
        )

    prefix = []
    for d, v in [([1, 2, 3], [1, 2, 4]), ([5, 6], [5, 6]), ([], [1]), ([7], [8])]:
        prefix.append({"draft": d, "verifier": v, "matched": runtime.longest_prefix_match(d, v)})

    out = {
        "generator": "tests/golden/make_golden.py (reference functions under a NumPy mlx stand-in)",
        "trees": cases,
        "walks": walks,
        "unit_walk": {"accepted": unit_walk[0], "next_token": unit_walk[1]},
        "lineages": lineages,
        "prefix_match": prefix,
    }
    (HERE / "tree_golden.json").write_text(json.dumps(out))
    np.savez_compressed(HERE / "tree_logits.npz", **logits_store)

    # compaction through Qwen3TargetAdapter.compact_kv_caches
    adapter = Qwen3TargetAdapter()
    c_rng = np.random.default_rng(5)
    npz = {}
    cidx = 0
    for past, t, keep in [
        (7, 9, [0, 2, 3, 8]),
        (0, 5, [0, 1, 2, 3, 4]),  # keep == current length: no-op
        (4, 6, []),  # keep nothing: offset = past
        (12, 25, [0, 1, 5, 6, 7, 19, 24]),
        (3, 65, [0, 1, 2, 40, 64]),
    ]:
        cap = past + t + 3
        layers = []
        for _ in range(2):
            k = c_rng.standard_normal((1, 2, cap, 8)).astype(np.float32)
            v = c_rng.standard_normal((1, 2, cap, 8)).astype(np.float32)
            layers.append(_KVCache(k.copy(), v.copy(), past + t))
            npz[f"c{cidx}_k_in_{len(layers) - 1}"] = k
            npz[f"c{cidx}_v_in_{len(layers) - 1}"] = v
        adapter.compact_kv_caches(None, layers, past_length=past, keep_current_indices=keep)
        for li, lc in enumerate(layers):
            npz[f"c{cidx}_k_out_{li}"] = np.asarray(lc.keys.a)
            npz[f"c{cidx}_v_out_{li}"] = np.asarray(lc.values.a)
            npz[f"c{cidx}_offset_{li}"] = np.array(lc.offset)
        npz[f"c{cidx}_meta"] = np.array([past, t, len(keep)] + list(keep), dtype=np.int64)
        cidx += 1
    npz["count"] = np.array(cidx)
    np.savez_compressed(HERE / "compact_golden.npz", **npz)
    print(f"wrote {len(cases)} trees, {len(walks)} walks, {len(lineages)} lineages, {cidx} compactions")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <path to a dtree-mlx source checkout>")
    main(sys.argv[1])
