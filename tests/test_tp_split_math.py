"""Tensor-parallel split arithmetic on the CPU oracle (no GPU): the library cuts each GGUF row of o and down into G
contiguous runs of whole blocks (row_bytes / G bytes each) and each rank dots its run with its slice of the input;
the G partial dots must sum to the full row's dot, and the row split (q, k, v, gate, up, the head) must give the
full matrix's rows. This is the byte slicing of load_from_gguf / open_synthetic, restated on host arrays. Mixture-of-
experts layers place whole experts on each GPU (rank r holds experts r*NE/G .. (r+1)*NE/G - 1): each rank adds its
own chosen experts' weighted outputs in ascending expert order (the reference's order, src/Transformer.cs:280-293)
and the all-reduce adds the ranks' sums."""
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


@pytest.mark.parametrize("G", [2, 4, 8])
def test_expert_placement_partials_sum_to_the_full_combine(oracle, G):
    """Every chosen expert lives on exactly one rank, so the ranks' partial combines add up to the one-GPU combine
    (to fp32 rounding: the association differs), and a rank with none of a token's experts contributes zero."""
    rng = np.random.default_rng(G)
    NE, K, T, E = 16, 4, 6, 64
    logits = rng.standard_normal((T, NE)).astype(np.float32)
    y = rng.standard_normal((T * K, E)).astype(np.float32)
    per = NE // G
    for t in range(T):
        sel, w, _ = oracle.route(logits[t], K, 1)
        order = np.argsort(sel, kind="stable")
        full = np.float32(0) * np.zeros(E, dtype=np.float32)
        for j in order:
            full = (full + np.float32(w[j]) * y[t * K + j]).astype(np.float32)
        total = np.zeros(E, dtype=np.float32)
        owners = set()
        for r in range(G):
            part = np.zeros(E, dtype=np.float32)
            for j in order:
                if r * per <= sel[j] < (r + 1) * per:
                    part = (part + np.float32(w[j]) * y[t * K + j]).astype(np.float32)
                    owners.add(int(sel[j]))
            total = (total + part).astype(np.float32)
        assert owners == set(int(e) for e in sel)
        assert np.max(np.abs(total - full)) <= 1e-5 * (np.max(np.abs(full)) + 1)
