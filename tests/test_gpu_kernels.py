"""GPU kernel parity against the CPU oracle, through the C ABI.

- wl_dequant is bit-exact with Quants.DecodeRow for every decodable type (src/Quants.cs:32-52, IQuants.cs:27-42).
- wl_matvec matches the reference's dot products within 1e-4 relative L2 (fp32 accumulate, different order),
  and each activation column's result is bit-identical whatever the number of columns beside it
  (the property ForwardBatch relies on, src/Transformer.cs:127-131).
- wl_synth_tensor writes the same bytes as the oracle's generator.
- Full-size (configs[1], 8192 x 8192) matvecs for the five benchmark formats against the oracle.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import dev, empty, host, ptr, rel_l2, weights, IQ_TYPES

pytestmark = pytest.mark.gpu

ALL_TYPES = ["f32", "f16", "bf16", "q4_0", "q4_1", "q5_0", "q5_1", "q8_0", "q2_K", "q3_K", "q4_K", "q5_K", "q6_K"] + \
            list(IQ_TYPES)
BENCH_TYPES = ["q4_K", "q6_K", "q8_0", "iq4_xs", "iq2_xxs"]


@pytest.mark.parametrize("tname", ALL_TYPES)
def test_dequant_bit_exact(wl, oracle, tname):
    O = oracle
    t = O.TYPE_OF[tname]
    rows, cols = 5, 512
    w = weights(O, tname, rows, cols)
    want = O.decode(t, w, rows * cols)
    dw = dev(w)
    out = empty(rows * cols)
    wl.check(wl.lib().wl_dequant(t, ptr(dw), rows * cols, ptr(out), None))
    got = host(out)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{tname}: {int((got.view(np.uint32) != want.view(np.uint32)).sum())} values differ"


def _matvec(wl, t, dw, rows, cols, x, ncols):
    dx = dev(x.reshape(-1))
    dy = empty(ncols * rows)
    wl.check(wl.lib().wl_matvec(t, ptr(dw), rows, cols, ptr(dx), ncols, ptr(dy), None))
    return host(dy).reshape(ncols, rows)


@pytest.mark.parametrize("tname", ALL_TYPES)
def test_matvec_matches_reference_and_columns_are_independent(wl, oracle, tname):
    O = oracle
    t = O.TYPE_OF[tname]
    rows, cols = 67, 1024
    w = weights(O, tname, rows, cols)
    dec = O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((11, cols)).astype(np.float32)
    dw = dev(w)
    y11 = _matvec(wl, t, dw, rows, cols, x, 11)
    want = x.astype(np.float64) @ dec.T
    for c in range(11):
        assert rel_l2(y11[c], want[c]) <= 1e-4, (tname, c, rel_l2(y11[c], want[c]))
    # each column alone gives the same bits as inside a batch of 11 (two launches of 8 and 3 columns)
    for c in (0, 5, 8, 10):
        y1 = _matvec(wl, t, dw, rows, cols, x[c:c + 1], 1)
        assert np.array_equal(y1[0].view(np.uint32), y11[c].view(np.uint32)), (tname, c)
    if O.lib().or_can_dot(t):
        ref = O.matmul(t, w, rows, cols, x[:1])[0]      # Quants.DotRow, the reference's own single-token kernel
        assert rel_l2(y11[0], ref) <= 1e-4


@pytest.mark.parametrize("tname,rows,cols", [("f32", 3, 256), ("f16", 9, 512), ("q8_0", 4, 1408), ("q4_K", 2, 256),
                                             ("q6_K", 1, 512), ("q8_0", 1, 32)])
def test_matvec_edge_shapes(wl, oracle, tname, rows, cols):
    """Ragged and minimal shapes: one block per row, a single row, a non-256 Q8_0 width (configs[0] ffn_down)."""
    O = oracle
    t = O.TYPE_OF[tname]
    w = weights(O, tname, rows, cols)
    dec = O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64)
    x = np.random.default_rng(1).standard_normal((3, cols)).astype(np.float32)
    y = _matvec(wl, t, dev(w), rows, cols, x, 3)
    assert rel_l2(y, x.astype(np.float64) @ dec.T) <= 1e-4


@pytest.mark.parametrize("tname", ["f32", "q8_0", "q4_K", "q6_K"])
def test_synth_bytes_match_oracle(wl, oracle, tname):
    O = oracle
    t = O.TYPE_OF[tname]
    rows, cols = 33, 512
    offset = 1.0 if t == O.F32 else 0.0
    want = O.synth_tensor(t, 1234, 0x305, rows, cols, 0.02, offset)
    out = empty(want.size, "uint8")
    wl.check(wl.lib().wl_synth_tensor(t, 1234, 0x305, rows, cols, C.c_float(0.02), C.c_float(offset), ptr(out), None))
    assert np.array_equal(host(out), want)


@pytest.mark.parametrize("tname", BENCH_TYPES)
def test_config1_full_size_matvec(wl, oracle, tname):
    """8192 x 8192, batch columns 1, 4, 8 (fused matvec) and 64 (matmul), against the oracle's dot
    products on a sample of rows; synthetic Q8_0/Q6_K/Q4_K bytes are also compared with the oracle's whole tensor."""
    O = oracle
    t = O.TYPE_OF[tname]
    n = 8192
    if tname in ("iq4_xs", "iq2_xxs"):
        w = weights(O, tname, n, n, seed=7)
        dw = dev(w)
    else:
        w = O.synth_tensor(t, 42, 0x7001, n, n, 0.02)
        dw = empty(w.size, "uint8")
        wl.check(wl.lib().wl_synth_tensor(t, 42, 0x7001, n, n, C.c_float(0.02), C.c_float(0.0), ptr(dw), None))
        assert np.array_equal(host(dw), w), f"{tname}: synthetic bytes differ from the oracle's"
    rng = np.random.default_rng(11)
    sample = np.sort(rng.choice(n, 96, replace=False))
    rb = O.row_bytes(t, n)
    sub = np.concatenate([w[r * rb:(r + 1) * rb] for r in sample])
    dec = O.decode(t, sub, sample.size * n).reshape(sample.size, n).astype(np.float64)
    for ncols in (1, 4, 8, 64):
        x = rng.standard_normal((ncols, n)).astype(np.float32)
        dx = dev(x.reshape(-1))
        dy = empty(ncols * n)
        if ncols <= 8:
            wl.check(wl.lib().wl_matvec(t, ptr(dw), n, n, ptr(dx), ncols, ptr(dy), None))
        else:
            wl.check(wl.lib().wl_matmul(t, ptr(dw), n, n, ptr(dx), ncols, ptr(dy), 0, None))
        y = host(dy).reshape(ncols, n)[:, sample]
        want = x.astype(np.float64) @ dec.T
        assert rel_l2(y, want) <= 1e-4, (tname, ncols, rel_l2(y, want))


TILE_BYTES = {"q4_K": 2304, "q6_K": 3360, "q8_0": 4352, "iq4_xs": 2208, "iq2_xxs": 1056}


@pytest.mark.parametrize("tname", ["q4_K", "q6_K", "q8_0", "iq4_xs", "iq2_xxs"])
def test_tile_layout_matvec_matches_reference(wl, oracle, tname):
    """wl_make_tiles + wl_matvec_tiles (the model's weight layout) against the reference dot products, and bit-equal
    to wl_matvec (which repacks per call); ragged row count (not a multiple of 16)."""
    O = oracle
    t = O.TYPE_OF[tname]
    L = wl.lib()
    rows, cols, ncols = 75, 2048, 3
    w = weights(O, tname, rows, cols, seed=11)
    dec = O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64)
    x = np.random.default_rng(9).standard_normal((ncols, cols)).astype(np.float32)
    dw, dx = dev(w), dev(x.reshape(-1))
    nb = C.c_int64()
    wl.check(L.wl_tiles_size(t, rows, cols, C.byref(nb)))
    assert nb.value == (rows + 15) // 16 * (cols // 256) * TILE_BYTES[tname]
    tiles = empty(nb.value, "uint8")
    wl.check(L.wl_make_tiles(t, ptr(dw), rows, cols, ptr(tiles), None))
    dy = empty(ncols * rows)
    wl.check(L.wl_matvec_tiles(t, ptr(tiles), rows, cols, ptr(dx), ncols, ptr(dy), None))
    got = host(dy).reshape(ncols, rows)
    want = x.astype(np.float64) @ dec.T
    for c in range(ncols):
        assert rel_l2(got[c], want[c]) <= 1e-4, (tname, c, rel_l2(got[c], want[c]))
    assert np.array_equal(got, _matvec(wl, t, dw, rows, cols, x, ncols))
    with pytest.raises(wl.NotSupportedError):
        wl.check(L.wl_tiles_size(O.TYPE_OF["q5_K"], rows, cols, C.byref(nb)))
    with pytest.raises(wl.NotSupportedError):
        wl.check(L.wl_tiles_size(t, rows, cols + 32, C.byref(nb)))


@pytest.mark.parametrize("tname,rows,cols", [("q4_K", 75, 2048), ("q4_K", 1000, 256), ("q4_K", 4099, 1024),
                                             ("q4_K", 19000, 512), ("q4_K", 8192, 8192), ("q8_0", 75, 2048),
                                             ("q8_0", 19000, 512), ("iq4_xs", 1000, 256), ("iq4_xs", 4099, 1024),
                                             ("iq2_xxs", 75, 2048), ("iq2_xxs", 19000, 512)])
def test_tile_matvec_columns_independent_of_batch(wl, oracle, tname, rows, cols):
    """For each tiled format, a column's result from wl_matvec_tiles does not depend on how many columns share the call: at every column
    count 1..8 each column equals the one-column call on that column bit for bit (the decode step's rows equal
    single-sequence steps, tests/BatchTests.cs:29-94), on ragged rows, fewer superblocks than the warps that share a
    row (1000 x 256), and row counts on both sides of the launch-shape threshold (19000 rows: 1188 row tiles);
    within 1e-4 relative L2 of the float64 products."""
    O = oracle
    t = O.TYPE_OF[tname]
    L = wl.lib()
    w = weights(O, tname, rows, cols, seed=rows + cols)
    x = np.random.default_rng(rows).standard_normal((8, cols)).astype(np.float32)
    dw, dx = dev(w), dev(x.reshape(-1))
    nb = C.c_int64()
    wl.check(L.wl_tiles_size(t, rows, cols, C.byref(nb)))
    tiles = empty(nb.value, "uint8")
    wl.check(L.wl_make_tiles(t, ptr(dw), rows, cols, ptr(tiles), None))
    one = []
    for c in range(8):
        dy = empty(rows)
        wl.check(L.wl_matvec_tiles(t, ptr(tiles), rows, cols, ptr(dev(x[c])), 1, ptr(dy), None))
        one.append(host(dy))
    one = np.stack(one)
    if rows * cols <= 4096 * 4096:
        dec = O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64)
        want = x.astype(np.float64) @ dec.T
        for c in range(8):
            assert rel_l2(one[c], want[c]) <= 1e-4, (c, rel_l2(one[c], want[c]))
    for n in range(2, 9):
        dy = empty(n * rows)
        wl.check(L.wl_matvec_tiles(t, ptr(tiles), rows, cols, ptr(dx), n, ptr(dy), None))
        got = host(dy).reshape(n, rows)
        for c in range(n):
            assert np.array_equal(got[c].view(np.uint32), one[c].view(np.uint32)), (n, c)


@pytest.mark.parametrize("tname", ["q4_K", "q6_K"])
@pytest.mark.parametrize("rows,cols,T", [(128, 256, 9), (100, 512, 64), (300, 1024, 65), (16, 256, 130),
                                          (2048, 2048, 200), (300, 1024, 600)])
def test_tcgen05_gemm_matches_reference(wl, oracle, tname, rows, cols, T):
    """Rows of Q4_K or Q6_K on the tcgen05 GEMM (bf16 hi/lo planes, fp32 accumulation in tensor memory):
    within 1e-4 relative L2 of the decoded weights' float64 products, like the matvec, on ragged row counts (not
    multiples of the 128-row tile or of 16), token counts around the 128-token tile, and against the integer
    tensor-core matvec in 8-column chunks (path 2)."""
    O = oracle
    t = O.TYPE_OF[tname]
    L = wl.lib()
    w = weights(O, tname, rows, cols, seed=rows + T)
    dec = O.decode(t, w, rows * cols).reshape(rows, cols).astype(np.float64)
    x = np.random.default_rng(T).standard_normal((T, cols)).astype(np.float32)
    dw, dx = dev(w), dev(x.reshape(-1))
    nb = C.c_int64()
    wl.check(L.wl_tiles_size(t, rows, cols, C.byref(nb)))
    tiles = empty(nb.value, "uint8")
    wl.check(L.wl_make_tiles(t, ptr(dw), rows, cols, ptr(tiles), None))
    dy, dy2, dy3 = empty(T * rows), empty(T * rows), empty(T * rows)
    wl.check(L.wl_gemm_tiles(t, ptr(tiles), rows, cols, ptr(dx), T, ptr(dy), None))
    wl.check(L.wl_matmul(t, ptr(dw), rows, cols, ptr(dx), T, ptr(dy2), 2, None))
    wl.check(L.wl_matmul(t, ptr(dw), rows, cols, ptr(dx), T, ptr(dy3), 0, None))
    y, y2, y3 = (host(d).reshape(T, rows) for d in (dy, dy2, dy3))
    want = x.astype(np.float64) @ dec.T
    assert rel_l2(y, want) <= 1e-4, rel_l2(y, want)
    assert rel_l2(y, y2) <= 1e-4
    # the library's own rule (GEMM from gemm_min_rows rows on, the 8-column matvec below) gives one of the two
    assert np.array_equal(y3, y if T >= {"q4_K": 81, "q6_K": 57}[tname] else y2)


def test_zz_no_kernel_level_wait_gave_up(wl):
    """After every kernel-level call above, no bounded device-side wait gave up (wl_kernel_status)."""
    wl.check(wl.lib().wl_kernel_status(0))


@pytest.mark.parametrize("n,k,renorm", [(128, 8, 1), (8, 2, 1), (60, 4, 0), (256, 32, 1), (3, 3, 1)])
def test_route_matches_oracle(wl, oracle, n, k, renorm):
    """Transformer.Route (src/Transformer.cs:315-340) on the device, bit for bit against the oracle's restatement, on
    random router logits, on logits with ties (equal probabilities: the lower expert id first) and on all -inf rows
    (every probability NaN: ids 0, 1, ... in order)."""
    rng = np.random.default_rng(n * 31 + k)
    T = 37
    lg = (rng.standard_normal((T, n)) * 3).astype(np.float32)
    lg[1, :] = 0.5                                     # every expert tied
    lg[2, ::2] = 1.25                                  # half of them tied at the top
    lg[3, :] = -np.inf
    lg[4, [n - 1, 0]] = 40.0
    d_lg = dev(lg.reshape(-1))
    d_sel, d_w = empty(T * k, "int32"), empty(T * k)
    wl.check(wl.lib().wl_route(ptr(d_lg), T, n, k, renorm, ptr(d_sel), ptr(d_w), None))
    sel, w = host(d_sel).reshape(T, k), host(d_w).reshape(T, k)
    for t in range(T):
        ws, ww, _ = oracle.route(lg[t], k, renorm)
        assert list(sel[t]) == list(ws), (t, list(sel[t]), list(ws))
        assert np.array_equal(w[t].view(np.uint32), ww.view(np.uint32)) or (np.isnan(w[t]).all() and np.isnan(ww).all()), t
