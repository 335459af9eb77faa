"""The AAA preprocessing's own atan2 and tan (the reference's native
bounds, aaa/native_geometry.py:174-222, call the C library's atan2f and
tanf, which glibc does not round correctly).

CPU: the double-precision evaluation's constants are the ones
dsl_splat_b200/csrc/trig_constants.py derives, in both the CUDA source and
the oracle, and the oracle's float results equal the correctly rounded ones
(float64 NumPy rounded once) on random and special arguments.  GPU: the CUDA
functions equal the oracle's bit for bit."""

from __future__ import annotations

import ast
import os
import re
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "dsl_splat_b200", "csrc"))
import trig_constants  # noqa: E402

from oracle import oracle as O  # noqa: E402


def _arguments(n: int, seed: int):
    rng = np.random.default_rng(seed)
    y = (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 4, n)).astype(np.float32)
    x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 4, n)).astype(np.float32)
    special = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, 1e-38, -1e-38, 3.4e38, 0.5,
                        0.0625, 0.9375, 1.5707964, -1.5707964, 3.1415927, 0.7853982],
                       np.float32)
    ys, xs = np.meshgrid(special, special)
    return np.concatenate([y, ys.ravel()]), np.concatenate([x, xs.ravel()])


def _tables(path: str, prefix: str) -> dict[str, list[float]]:
    text = open(path).read()
    out = {}
    for name in trig_constants.tables():
        m = re.search(prefix + r"\s+" + name + r"(?:\[\d+\])?\s*=\s*\{?([^;}]*)\}?;", text)
        assert m, f"{name} missing in {path}"
        out[name] = [float(ast.literal_eval(v.strip())) for v in m.group(1).split(",") if v.strip()]
    return out


@pytest.mark.parametrize("path,prefix", [
    (os.path.join(ROOT, "dsl_splat_b200", "csrc", "aaa.cuh"), r"(?:__constant__|constexpr) double"),
    (os.path.join(ROOT, "oracle", "aaa_oracle.cpp"), r"static const double"),
])
def test_constants_match_their_derivation(path, prefix):
    assert _tables(path, prefix) == trig_constants.tables()


def test_oracle_is_correctly_rounded():
    y, x = _arguments(100_000, 0)
    got = O.atan2f(y, x)
    want = np.arctan2(y.astype(np.float64), x.astype(np.float64)).astype(np.float32)
    np.testing.assert_array_equal(got, want)
    t = np.concatenate([np.random.default_rng(1).uniform(-3.3, 3.3, 100_000),
                        [0.0, -0.0, 0.7853982, -0.7853982, 1.5707963, 3.1415927]]).astype(np.float32)
    np.testing.assert_array_equal(O.tanf(t), np.tan(t.astype(np.float64)).astype(np.float32))


@pytest.mark.gpu
def test_cuda_matches_oracle():
    import torch

    from dsl_splat_b200._native import check, lib

    y, x = _arguments(200_000, 2)
    dev = torch.device("cuda", 0)
    ty, tx = torch.from_numpy(y).to(dev), torch.from_numpy(x).to(dev)
    a, t = torch.empty_like(ty), torch.empty_like(tx)
    check(lib.splat_test_trig(len(y), ty.data_ptr(), tx.data_ptr(), a.data_ptr(), t.data_ptr(),
                              torch.cuda.current_stream(dev).cuda_stream), "test_trig")
    torch.cuda.synchronize(dev)
    np.testing.assert_array_equal(a.cpu().numpy(), O.atan2f(y, x))
    np.testing.assert_array_equal(t.cpu().numpy(), O.tanf(x))
