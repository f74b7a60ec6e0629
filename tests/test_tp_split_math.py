"""Tensor-parallel split arithmetic on the CPU oracle (no GPU): the library cuts each GGUF row of o and down into G
contiguous runs of whole blocks (row_bytes / G bytes each) and each rank dots its run with its slice of the input;
the G partial dots must sum to the full row's dot, and the row split (q, k, v, gate, up, the head) must give the
full matrix's rows. This is the byte slicing of load_from_gguf / open_synthetic, restated on host arrays."""
import numpy as np
import pytest


@pytest.mark.parametrize("tname,G", [("q4_K", 2), ("q4_K", 8), ("q6_K", 4), ("q8_0", 2)])
def test_column_split_partials_sum_to_the_full_dot(oracle, tname, G):
    O = oracle
    t = O.TYPE_OF[tname]
    rows, cols = 24, 2048
    w = O.matrix(O.Rng(9), t, rows, cols, 0.02)
    x = np.random.default_rng(G).standard_normal((1, cols)).astype(np.float32)
    full = O.matmul(t, w, rows, cols, x)[0].astype(np.float64)
    rb = O.row_bytes(t, cols)
    lrb, lc = rb // G, cols // G
    parts = np.zeros(rows)
    for r in range(G):
        sub = np.concatenate([w[i * rb + r * lrb:i * rb + (r + 1) * lrb] for i in range(rows)])
        parts += O.matmul(t, sub, rows, lc, x[:, r * lc:(r + 1) * lc])[0].astype(np.float64)
    assert np.max(np.abs(parts - full)) <= 1e-5 * np.max(np.abs(full)) + 1e-6


def test_row_split_is_the_rows_of_the_full_matrix(oracle):
    O = oracle
    t = O.TYPE_OF["q4_K"]
    rows, cols, G = 32, 512, 4
    w = O.matrix(O.Rng(3), t, rows, cols, 0.02)
    x = np.random.default_rng(1).standard_normal((1, cols)).astype(np.float32)
    full = O.matmul(t, w, rows, cols, x)[0]
    rb = O.row_bytes(t, cols)
    n = rows // G
    got = np.concatenate([O.matmul(t, w[r * n * rb:(r + 1) * n * rb], n, cols, x)[0] for r in range(G)])
    assert np.array_equal(got, full)
