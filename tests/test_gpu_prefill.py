"""GPU parity of the prefill matmul (T tokens on the tcgen05 tensor cores,
straight from the Q4_K rows).

The oracle computes the exact int32 sub-block sums isum[t][r][j] and the
fp32 result of the exact dot.  The prefill kernel decodes each row's 4-bit
quants on chip and accumulates each 256-weight super-block, min terms
included, on the tensor cores (fp16 sc * q exact, xq * sx in two fp16 parts,
the min terms in three bf16 parts each) and scales it by the super-block's d
in fp32.  Bar: every output within 1e-5 of the exact value, relative to the
sum of the magnitudes of its sub-block terms (the fp32 combine's error
scale), and the normwise relative error below 1e-5.
"""
import numpy as np
import pytest
import torch

import _oracle as O
import lalmodel_b200 as lb

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def scales_mins(W, rows, K):
    """The 6-bit scales and mins [rows][K/256][8] of every super-block."""
    s = W.reshape(rows, K // 256, 144)[:, :, 4:16].astype(np.int32)
    sc = np.empty((rows, K // 256, 8), np.int32)
    mn = np.empty_like(sc)
    sc[..., :4] = s[..., 0:4] & 63
    mn[..., :4] = s[..., 4:8] & 63
    sc[..., 4:] = (s[..., 8:12] & 15) | ((s[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (s[..., 8:12] >> 4) | ((s[..., 4:8] >> 6) << 4)
    return sc, mn


def block_fields(W, rows, K):
    """Per sub-block (d*sc, dmin*m) in fp32 and the 4-bit quants, from the raw bytes."""
    b = W.reshape(rows, K // 256, 144)
    d = b[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = b[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    sc, mn = scales_mins(W, rows, K)
    qs = b[:, :, 16:].reshape(rows, K // 256, 4, 32)
    q = np.empty((rows, K // 256, 8, 32), np.int8)
    q[:, :, 0::2] = qs & 15
    q[:, :, 1::2] = qs >> 4
    dsc = (d[..., None] * sc.astype(np.float32)).astype(np.float32)
    dmm = (dmin[..., None] * mn.astype(np.float32)).astype(np.float32)
    return q.reshape(rows, K), dsc.reshape(rows, K // 32), dmm.reshape(rows, K // 32)


def make(rows, K, T, seed):
    w = O.normal(rows * K, seed=seed, sigma=0.02).reshape(rows, K)
    W = O.q4k_quantize(w)
    X = O.normal(T * K, seed=seed + 1).reshape(T, K)
    return W, X


def check(W, X, rows, K, Y):
    T = X.shape[0]
    xq, sx, sq = O.quantize_act(X)
    yref, isum = O.q4k_matmul(W, rows, K, xq, sx, sq, want_isum=True)
    _, dsc, dmm = block_fields(W, rows, K)
    # magnitude of every fp32 sub-block term, summed: the combine's error scale
    t1 = np.abs(sx[:, None, :].astype(np.float64) * dsc[None].astype(np.float64) * isum)
    t2 = np.abs((sx * sq)[:, None, :].astype(np.float64) * dmm[None].astype(np.float64))
    scale = (t1 + t2).sum(-1)
    err = np.abs(Y.astype(np.float64) - yref.astype(np.float64))
    assert np.all(err <= TOL * scale + 1e-30), float(np.max(err / (scale + 1e-30)))
    assert O.normwise_rel_err(Y, yref) < TOL


@pytest.mark.parametrize("rows,K,T", [
    (128, 256, 64),      # one tile
    (128, 512, 64),      # several K-blocks in one stage ring pass
    (256, 3584, 64),     # 28 K-blocks: the stage ring and TMEM slots wrap
    (200, 3584, 100),    # ragged rows and tokens (partial tiles)
    (96, 1024, 1),       # a single token
    (512, 3584, 512),    # the prefill batch, q/o-shaped slice
    (130, 512, 7),       # two row tiles, the second with 2 rows
    (256, 768, 130),     # three super-blocks: the raw-tile ring's first refill
    (128, 2048, 64),     # eight super-blocks: every raw slot and TMEM slot reused
    (19200, 512, 64),    # 150 output tiles: one CTA per tile, K not split
    (3584, 3584, 100),   # 28 tiles of 14 super-blocks: K split over 5 CTAs per tile
])
def test_prefill_matmul_matches_exact(ctx, rows, K, T):
    W, X = make(rows, K, T, seed=7 * rows + K + T)
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)


def test_prefill_zero_scale_super_blocks(ctx):
    """A super-block whose d is 0 (the quantizer writes d = 0 only with every
    sc 0): its weights are -dmin m, the min terms alone."""
    rows, K, T = 256, 1024, 40
    W, X = make(rows, K, T, seed=404)
    b = W.reshape(rows, K // 256, 144)
    for r, sb in [(0, 0), (1, 3), (129, 2), (255, 1)]:
        b[r, sb, 0:2] = 0          # d = 0 (dmin in bytes 2:4 kept)
        b[r, sb, 4:8] = 0          # sc 0..3, and the high bits of sc 4..7
        b[r, sb, 12:16] &= 0xF0    # the low bits of sc 4..7 (bytes 8:12 and the high
                                   # nibbles here are the mins, kept)
    sc, mn = scales_mins(W, rows, K)
    assert not sc[0, 0].any() and mn[0, 0].any()
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)


def test_prefill_down_shape_long_k(ctx):
    rows, K, T = 384, 18944, 128
    W, X = make(rows, K, T, seed=31)
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)


@pytest.mark.parametrize("K", [18944, 23040])
def test_prefill_long_k_spike_past_the_register_cache(ctx, K):
    """Token preparation keeps a token's first 4 x 20 groups of 128 weights in
    registers with 4 warps (K <= 10240) and 8 x 20 with 8 warps (rows longer
    than that: K <= 20480), and reads the rest again for the conversion.
    Spikes at the cache edges and past them (the first and the last element,
    one in between) must set the token's scales; K = 23040 is read twice."""
    rows, T = 128, 5
    W, X = make(rows, K, T, seed=37)
    X[0, 10240] = 900.0
    X[1, K - 1] = -700.0
    X[2, 15001] = 5.0e4
    X[3, 10239] = 800.0   # the last element 4 warps keep in registers
    if K > 20480:
        X[4, 20480] = -3.0e3   # the first element 8 warps read again
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)


def test_prefill_token_magnitudes(ctx):
    """Tokens scaled by 2^-60 .. 2^40: the per-token power of two keeps B in
    fp16 range, so the relative error does not depend on the magnitude."""
    rows, K, T = 128, 1024, 6
    W, X = make(rows, K, T, seed=8)
    for t, e in enumerate([-60, -20, 0, 13, 25, 40]):
        X[t] *= np.float32(2.0 ** e)
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)
    xq, sx, sq = O.quantize_act(X)
    yref, _ = O.q4k_matmul(W, rows, K, xq, sx, sq)
    for t in range(T):
        assert O.normwise_rel_err(Y[t], yref[t]) < TOL


def test_prefill_zero_and_spike_tokens(ctx):
    rows, K, T = 128, 512, 70
    W, X = make(rows, K, T, seed=5)
    X[3] = 0.0                 # all-zero token: every block scale 0
    X[4, :32] = 0.0            # one zero block
    X[5, 7] = 1e4              # a spike: that block quantizes to one +-127
    X[6, 40] = -1e4
    Y = host(ctx.matmul_q4_k_prefill(dev(W), rows, K, dev(X)))
    check(W, X, rows, K, Y)
    assert np.all(Y[3] == 0.0)


def test_prefill_matches_per_token_gemv(ctx):
    """The batched path and the matvec path agree on every token."""
    rows, K, T = 256, 3584, 8
    W, X = make(rows, K, T, seed=77)
    Wd = dev(W)
    Y = host(ctx.matmul_q4_k_prefill(Wd, rows, K, dev(X)))
    for t in range(T):
        y = host(ctx.matmul_q4_k(Wd, dev(X[t]), rows, K))
        assert O.normwise_rel_err(Y[t], y) < TOL


def test_prefill_rejects_bad_arguments(ctx):
    rows, K = 128, 256
    W, X = make(rows, K, 4, seed=3)
    Wd = dev(W)
    with pytest.raises(lb.LalbError):
        ctx.matmul_q4_k_prefill(Wd, rows, 200, dev(X[:, :200]))        # K not a multiple of 256
    ws = torch.empty(lb.prefill_ws_bytes(rows, K, 4) + 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(lb.LalbError):
        ctx.matmul_q4_k_prefill(Wd, rows, K, dev(X), ws=ws[16:])       # workspace not 256-aligned
    Wo = torch.empty(W.size + 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(lb.LalbError):
        ctx.matmul_q4_k_prefill(Wo[8:8 + W.size], rows, K, dev(X))     # rows not 16-aligned
    torch.cuda.synchronize()
    assert ctx.device_status() == 0


def test_measured_mma_peaks(ctx):
    """Back-to-back tcgen05.mma on every SM: dense kind::f16 near its 2.25
    PFLOP/s nominal (at the clock under that load), kind::i8 above it."""
    f16 = ctx.measure_mma_peak(lb.MMA_F16)
    i8 = ctx.measure_mma_peak(lb.MMA_I8)
    assert 900.0 < f16 < 2600.0, f16
    assert i8 > 1.2 * f16, (i8, f16)
    with pytest.raises(lb.LalbError):
        ctx.measure_mma_peak(7)
    assert ctx.device_status() == 0
