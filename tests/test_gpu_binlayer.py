"""The seed STE model's forward matmuls on tensor cores against the
reference's goldens and the oracle: per-row masks (BinLayer) on the tf32-part
GEMM, per-element int8 codes (LogicLayer) on the GEMM that decodes the codes
into exact fp16 on chip.  Tolerance: 1e-5 normwise (max |diff| / max |ref|)
for every fp32 output; PRUNE rows exactly 0; the per-element codes and row
scales bit-exact."""
import os

import numpy as np
import pytest
import torch

import _oracle as O
import lalmodel_b200 as lb
from test_gpu_kernels import dev, host

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-5


@pytest.mark.parametrize("ci", [0, 1])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("repack", [0, 1])
def test_binlayer_matches_reference_goldens(ctx, ci, mode, repack):
    g = np.load(os.path.join(GOLD, "binlayer_ref.npz"))
    W, b, mask, X = (g[f"bl{ci}_{k}"] for k in ("W", "b", "mask", "X"))
    bl = lb.BinLayer(ctx, dev(W), dev(b), dev(mask), alpha_repack=bool(repack), max_rows=64)
    Y = host(bl.forward(dev(X), mode=mode))
    ref = g[f"bl{ci}_m{mode}_r{repack}_Y"]
    assert O.normwise_rel_err(Y, ref) < TOL
    np.testing.assert_allclose(host(bl.alpha()), g[f"bl{ci}_m{mode}_r{repack}_alpha"], rtol=2e-6, atol=0)
    assert np.all(Y[:, mask == 2] == 0.0)
    bl.close()


def test_binlayer_rejects_unaligned_in_dim(ctx):
    g = np.load(os.path.join(GOLD, "binlayer_ref.npz"))
    W, b, mask = (g[f"bl2_{k}"] for k in ("W", "b", "mask"))   # in = 100
    with pytest.raises(lb.LalbError) as e:
        lb.BinLayer(ctx, dev(W), dev(b), dev(mask))
    assert e.value.status == -4


# the seed model's phase-0 shapes (d = 448, FFN 1792, vocab 32768), X rows 1024
SHAPES = [(448, 1344, 1024), (448, 448, 1024), (448, 1792, 1024), (1792, 448, 1024),
          (448, 32768, 96), (448, 300, 100)]


@pytest.mark.parametrize("in_dim,out_dim,M", SHAPES)
@pytest.mark.parametrize("mode", [0, 1])
def test_binlayer_phase0_shapes_match_oracle(ctx, in_dim, out_dim, M, mode):
    rng = np.random.default_rng(in_dim * 7 + out_dim + M)
    W = O.normal(out_dim * in_dim, seed=out_dim, sigma=0.02).reshape(out_dim, in_dim)
    b = O.normal(out_dim, seed=out_dim + 1, sigma=0.01)
    mask = rng.choice(np.array([0, 1, 2], np.uint8), size=out_dim, p=[0.15, 0.60, 0.25])
    X = O.normal(M * in_dim, seed=M + 3).reshape(M, in_dim)
    ref, _ = O.binlayer_forward(W, b, mask, X, mode, repack=True)
    bl = lb.BinLayer(ctx, dev(W), dev(b), dev(mask), alpha_repack=True, max_rows=M)
    Y = host(bl.forward(dev(X), mode=mode))
    assert O.normwise_rel_err(Y, ref) < TOL
    assert np.all(Y[:, mask == 2] == 0.0)
    bl.close()


@pytest.mark.parametrize("rows,K,M", [(1344, 448, 1024), (448, 1792, 1024), (32768, 448, 64),
                                      (200, 64, 130)])
def test_logic_codes_pack_and_forward_match_oracle(ctx, rows, K, M):
    W = O.normal(rows * K, seed=rows + K, sigma=0.02).reshape(rows, K)
    st = O.logic_state(rows * 31 + K, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    gcodes, gsrow = lb.LogicLayer.pack(ctx, dev(W), dev(st))
    assert np.array_equal(host(gcodes), codes)
    assert np.array_equal(host(gsrow).view(np.uint32), srow.view(np.uint32))
    bias = O.normal(rows, seed=5, sigma=0.01)
    X = O.normal(M * K, seed=M).reshape(M, K)
    ref = O.logic_forward(codes, srow, bias, X)
    L = lb.LogicLayer(ctx, gcodes, gsrow, dev(bias), max_rows=M)
    Y = host(L.forward(dev(X)))
    assert O.normwise_rel_err(Y, ref) < TOL
    L.close()


# outputs with few tiles take the split-K kernel (clusters of 2 to 4 CTAs
# summing their partial tiles through distributed shared memory), outputs with
# many tiles the persistent kernel with 256-column tiles: 4-way (448 rows),
# 3-way (640 rows: 40 tiles), one wave of 128-wide tiles (1344, 1300, 1790,
# 1792 rows: ragged last tiles), a ragged last tile with rows not a multiple of
# 4 (scalar stores), token counts that end inside a tile, and the 256-wide
# persistent kernel (32768 rows; 16384 rows over 1024 tokens)
@pytest.mark.parametrize("rows,K,M", [(448, 448, 1024), (640, 448, 1024), (450, 448, 256),
                                      (1344, 448, 1024), (1300, 448, 1024), (1790, 448, 1024),
                                      (1792, 448, 1024), (448, 1792, 100), (90, 256, 33),
                                      (32768, 448, 200), (16384, 448, 1024)])
def test_logic_layer_split_k_shapes_match_oracle(ctx, rows, K, M):
    W = O.normal(rows * K, seed=rows * 3 + K, sigma=0.02).reshape(rows, K)
    st = O.logic_state(rows * 17 + K, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    bias = O.normal(rows, seed=7, sigma=0.01)
    X = O.normal(M * K, seed=M + 11).reshape(M, K)
    ref = O.logic_forward(codes, srow, bias, X)
    L = lb.LogicLayer(ctx, dev(codes), dev(srow), dev(bias), max_rows=M)
    Y = host(L.forward(dev(X)))
    assert O.normwise_rel_err(Y, ref) < TOL
    Y2 = host(L.forward(dev(X)))
    assert np.array_equal(Y, Y2)   # fixed summation order: repeatable
    L.close()


def test_logic_layer_rejects_too_many_rows(ctx):
    codes = torch.zeros((64, 64), dtype=torch.int8, device="cuda")
    srow = torch.ones(64, dtype=torch.float32, device="cuda")
    L = lb.LogicLayer(ctx, codes, srow, None, max_rows=8)
    with pytest.raises(lb.LalbError) as e:
        L.forward(torch.zeros((9, 64), dtype=torch.float32, device="cuda"))
    assert e.value.status == -1
    L.close()


@pytest.mark.parametrize("rows,K,M", [(300, 96, 70), (129, 160, 129), (256, 32, 5)])
def test_logic_layer_k_not_a_multiple_of_64(ctx, rows, K, M):
    """K % 64 == 32: the last K-block's code and token tiles are half outside
    the matrices and read as zeros."""
    W = O.normal(rows * K, seed=rows + 5 * K, sigma=0.02).reshape(rows, K)
    st = O.logic_state(rows * 13 + K, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    bias = O.normal(rows, seed=9, sigma=0.01)
    X = O.normal(M * K, seed=M + 3).reshape(M, K)
    ref = O.logic_forward(codes, srow, bias, X)
    L = lb.LogicLayer(ctx, dev(codes), dev(srow), dev(bias), max_rows=M)
    assert O.normwise_rel_err(host(L.forward(dev(X))), ref) < TOL
    L.close()


def test_logic_layer_token_magnitudes_and_zero_rows(ctx):
    """Token rows scaled by 2^-60 .. 2^40 and all-zero rows: the per-row power
    of two keeps the fp16 parts in range, so every row's relative error is the
    same; a zero row gives exactly the bias."""
    rows, K, M = 384, 448, 9
    W = O.normal(rows * K, seed=77, sigma=0.02).reshape(rows, K)
    st = O.logic_state(78, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    bias = O.normal(rows, seed=79, sigma=0.01)
    X = O.normal(M * K, seed=80).reshape(M, K)
    for t, e in enumerate([-60, -20, 0, 13, 25, 40, 0, 0, 0]):
        X[t] *= np.float32(2.0 ** e)
    X[6] = 0.0
    X[7, :100] = 0.0
    X[8, 5] = 1e6      # one spike in an otherwise N(0,1) row
    ref = O.logic_forward(codes, srow, bias, X)
    L = lb.LogicLayer(ctx, dev(codes), dev(srow), dev(bias), max_rows=M)
    Y = host(L.forward(dev(X)))
    for t in range(M):
        if t == 6:
            assert np.array_equal(Y[t], bias.astype(np.float32))
        else:
            assert O.normwise_rel_err(Y[t] - bias, ref[t] - bias) < TOL
    L.close()


def test_logic_layer_long_rows(ctx):
    """Rows many times longer than one pass of the token preparation's CTA
    (K = 4640: 1160 float4 over 128 threads, the last pass partial), each
    row's maximum at a different place: the last element, the middle, the
    first pass; 37 rows."""
    rows, K, M = 200, 4640, 37
    W = O.normal(rows * K, seed=91, sigma=0.02).reshape(rows, K)
    st = O.logic_state(92, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    bias = O.normal(rows, seed=93, sigma=0.01)
    X = O.normal(M * K, seed=94).reshape(M, K)
    X[0, K - 1] = 300.0
    X[1, 2048] = -500.0
    X[2, 10] = 1.0e3
    X[36, 4000] = 2.0e4
    ref = O.logic_forward(codes, srow, bias, X)
    L = lb.LogicLayer(ctx, dev(codes), dev(srow), dev(bias), max_rows=M)
    Y = host(L.forward(dev(X)))
    for t in range(M):
        assert O.normwise_rel_err(Y[t] - bias, ref[t] - bias) < TOL
    L.close()


def test_logic_layer_many_units_per_cta(ctx):
    """More 128 x 128 units than SMs with a count that is not a multiple of
    them (each CTA takes every 148th unit: some take one more), and a ragged
    last row and token tile."""
    rows, K, M = 19000, 256, 300
    W = O.normal(rows * K, seed=81, sigma=0.02).reshape(rows, K)
    st = O.logic_state(82, rows * K, 0.10, 0.50).reshape(rows, K)
    codes, srow = O.logic_pack(W, st)
    X = O.normal(M * K, seed=83).reshape(M, K)
    ref = O.logic_forward(codes, srow, None, X)
    L = lb.LogicLayer(ctx, dev(codes), dev(srow), None, max_rows=M)
    Y = host(L.forward(dev(X)))
    assert O.normwise_rel_err(Y, ref) < TOL
    assert np.array_equal(Y, host(L.forward(dev(X))))
    L.close()
