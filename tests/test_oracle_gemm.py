"""The GEMM oracle (scope row f4: linear() = matmul + add_bias_inplace, and
the MLP's gate/up linears + silu_mul) pinned before it checks a kernel: the
reference's own known-answer tests (tests/test_matmul.cpp:7-13,
tests/test_ops.cpp:59-68), the golden fixtures made by the compiled
reference, and bit-identity with the compiled kllm::op::matmul (CPU, F32)
on seeded inputs."""
from __future__ import annotations

import numpy as np
import pytest


def test_reference_kat(oracle):
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[1, 0, 1], [0, 1, 1]], np.float32)
    assert np.array_equal(oracle.matmul(a, b), [[4, 5], [10, 11]])
    assert np.array_equal(oracle.linear(a, b, np.array([1, -1], np.float32)), [[5, 4], [11, 10]])


def test_golden_linear_and_mlp(oracle, golden):
    g = golden
    assert np.array_equal(oracle.matmul(g["mm_x"], g["mm_w"]), g["mm_out"])
    assert np.array_equal(oracle.linear(g["mm_x"], g["mm_w"], g["mm_b"]), g["lin_out"])
    gate = oracle.linear(g["mlp_x"], g["mlp_wg"], g["mlp_bg"])
    up = oracle.linear(g["mlp_x"], g["mlp_wu"], g["mlp_bu"])
    assert np.array_equal(oracle.silu_mul(gate, up), g["mlp_out"])


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 13), (33, 64, 96), (16, 200, 896)])
def test_oracle_matches_reference_bitwise(oracle, reference, m, n, k):
    rng = np.random.default_rng(m * 1000 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    assert np.array_equal(oracle.matmul(a, b), reference.matmul(a, b))
