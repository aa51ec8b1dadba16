"""Golden vectors for the Qwen3.5 tree kernels, taken from the REFERENCE's own
known-answer tests.

``tests/test_qwen35_tree_kernels.py`` of the reference builds seeded inputs,
runs the Metal kernel, and compares it with a NumPy reference it computes
inline.  This script runs those two test functions unchanged (with the
NumPy-backed mlx stand-in of ``make_golden.py``), substituting a capture for
the Metal kernel call and for ``np.testing.assert_allclose``, and stores the
test's inputs and its NumPy reference outputs in
``tests/golden/qwen35_tree_kernels.npz``:

* conv_*  : tree_conv1d_kernel  (dtree_mlx/qwen35_tree_kernels.py:86-134, 180-206)
* delta_* : tree_gated_delta_kernel (dtree_mlx/qwen35_tree_kernels.py:8-82, 207-224)

Usage (needs the reference checkout; run from the repo root):
    python tests/golden/make_qwen35_golden.py /path/to/reference
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

from make_golden import install_shims  # noqa: E402


def main(ref_root: str) -> None:
    install_shims()
    sys.path.insert(0, ref_root)
    spec = importlib.util.spec_from_file_location("ref_qwen35_kernel_tests",
                                                  Path(ref_root) / "tests" / "test_qwen35_tree_kernels.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    out: dict[str, np.ndarray] = {}
    desired: list[np.ndarray] = []
    real_assert = np.testing.assert_allclose
    np.testing.assert_allclose = lambda actual, want, *a, **k: desired.append(np.array(want))

    def fake_conv(qkv, base, weight, parents):
        out.update(conv_qkv=np.array(qkv), conv_base=np.array(base), conv_weight=np.array(weight),
                   conv_parents=np.array(parents))
        b, t, c = np.array(qkv).shape
        keep = np.array(base).shape[1]
        return mod.mx.array(np.zeros((b, t, c), np.float32)), mod.mx.array(np.zeros((b, t, keep, c), np.float32))

    def fake_delta(q, k, v, g, beta, state, parents):
        out.update(delta_q=np.array(q), delta_k=np.array(k), delta_v=np.array(v), delta_g=np.array(g),
                   delta_beta=np.array(beta), delta_state=np.array(state), delta_parents=np.array(parents))
        b, t, hv, dv = np.array(v).shape
        dk = np.array(k).shape[-1]
        return (mod.mx.array(np.zeros((b, t, hv, dv), np.float32)),
                mod.mx.array(np.zeros((b, t, hv, dv, dk), np.float32)))

    try:
        mod.tree_conv1d_kernel = fake_conv
        mod.test_tree_conv1d_kernel_matches_reference()
        out["conv_out"], out["conv_states"] = desired[0], desired[1]
        desired.clear()
        mod.tree_gated_delta_kernel = fake_delta
        mod.test_tree_gated_delta_kernel_matches_reference()
        out["delta_out"], out["delta_states"] = desired[0], desired[1]
    finally:
        np.testing.assert_allclose = real_assert
    np.savez(HERE / "qwen35_tree_kernels.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <path to a dtree-mlx source checkout>")
    main(sys.argv[1])
