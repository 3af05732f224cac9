"""CPU tests of the oracle against the golden fixtures and of the CPU baseline.

Golden fixtures (tests/golden/gen_golden.py):
  formats_gguf.npz  gguf 0.19.0 Q4_K dequantization / Q8_0 quantization, numpy fp16
  binlayer_ref.npz  the reference's own bin_forward / bin_forward_pure_float
"""
import os

import numpy as np
import pytest

import _oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def fx():
    return np.load(os.path.join(GOLD, "formats_gguf.npz"))


def test_fp16_conversion_matches_numpy(fx):
    L = O.lib()
    f, h = fx["f16_in"], fx["f16_out"]
    got = np.array([L.lalb_o_f32_to_f16(float(v)) for v in f], np.uint16)
    assert np.array_equal(got, h)
    back = np.array([L.lalb_o_f16_to_f32(int(v)) for v in h], np.float32)
    assert np.array_equal(back.view(np.uint32), h.view(np.float16).astype(np.float32).view(np.uint32))


def test_unpack_scales_matches_gguf(fx):
    raw, sc, mn = fx["q4k_raw"], fx["q4k_raw_sc"], fx["q4k_raw_min"]
    for i in range(raw.shape[0]):
        u = O.unpack_scales(raw[i, 4:16])
        assert np.array_equal(u[:8], sc[i]) and np.array_equal(u[8:], mn[i])


def test_q4k_dequant_matches_gguf_bytes(fx):
    raw, deq = fx["q4k_raw"], fx["q4k_raw_deq"]
    got = O.q4k_dequantize(raw.reshape(-1), raw.shape[0], 256)
    assert np.array_equal(got.view(np.uint32), deq.reshape(raw.shape[0], 256).view(np.uint32))


def test_q4k_quantizer_roundtrip_through_gguf():
    gguf_quants = pytest.importorskip("gguf.quants")
    w = O.normal(64 * 1024, seed=11, sigma=0.02).reshape(64, 1024)
    blk = O.q4k_quantize(w)
    mine = O.q4k_dequantize(blk, 64, 1024)
    theirs = gguf_quants.Q4_K.dequantize_blocks(blk.reshape(-1, 144).copy()).reshape(64, 1024)
    assert np.array_equal(mine.view(np.uint32), theirs.astype(np.float32).view(np.uint32))
    # min-max error bound per sub-block: |w - deq| <= step/2 + 6-bit scale error
    err = np.abs(mine - w).reshape(-1, 32)
    rng = (w.reshape(-1, 32).max(1) - np.minimum(w.reshape(-1, 32).min(1), 0))
    assert np.all(err.max(1) <= rng / 15 * 0.5 + rng / 63 * 8 + 1e-7)


def test_q4k_quantizer_edge_blocks():
    w = np.zeros((4, 256), np.float32)
    w[1] = 0.5                     # all positive, constant
    w[2] = -np.linspace(0, 1, 256, dtype=np.float32)
    w[3, ::7] = 3e-3
    blk = O.q4k_quantize(w)
    deq = O.q4k_dequantize(blk, 4, 256)
    assert np.all(deq[0] == 0)
    assert np.all(blk[0, :4] == 0)          # an all-zero block stores +0 d and dmin
    assert np.allclose(deq, w, atol=0.05)


def test_activation_quantizer_matches_gguf_q8_0(fx):
    x, q, d = fx["q8_x"], fx["q8_q"], fx["q8_d"]
    xq, sx, sq = O.quantize_act(x.reshape(-1))
    assert np.array_equal(xq.reshape(q.shape), q)
    assert np.array_equal(sx.reshape(-1).view(np.uint32), d.view(np.uint32))
    assert np.array_equal(sq.reshape(-1), q.astype(np.int32).sum(1))
    assert xq.min() >= -127


def q4k_nibbles(W, rows, K):
    qn = np.empty((rows, K // 256, 256), np.int32)
    blk = W.reshape(rows, K // 256, 144)
    for g in range(4):
        b = blk[:, :, 16 + 32 * g: 48 + 32 * g].astype(np.int32)
        qn[:, :, 64 * g:64 * g + 32] = b & 15
        qn[:, :, 64 * g + 32:64 * g + 64] = b >> 4
    return qn.reshape(rows, K)


def test_q4k_matmul_equals_dequantized_dot():
    rows, K = 96, 2048
    W = O.q4k_quantize(O.normal(rows * K, seed=3, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=4)
    xq, sx, sq = O.quantize_act(x)
    y, isum = O.q4k_matmul(W, rows, K, xq, sx, sq, want_isum=True)
    wd = O.q4k_dequantize(W, rows, K).astype(np.float64)
    xd = (xq[0].astype(np.float64).reshape(-1, 32) * sx[0][:, None]).reshape(-1)
    ref = wd @ xd
    assert O.normwise_rel_err(y[0], ref) < 1e-5
    # the int32 sub-block sums are the plain integer dots
    qn = q4k_nibbles(W, rows, K)
    ref_isum = (qn.reshape(rows, -1, 32) * xq[0].astype(np.int32).reshape(1, -1, 32)).sum(-1)
    assert np.array_equal(isum[0], ref_isum)


def test_q8_lmhead_oracle_and_argmax_first_max():
    rows, K = 300, 512
    w = O.normal(rows * K, seed=5, sigma=0.02).reshape(rows, K)
    q, s = O.q8_quantize_rows(w)
    assert q.min() >= -127
    x = O.normal(K, seed=6)
    xq, sx, _ = O.quantize_act(x)
    logits, isum, am = O.q8_lmhead(q, s, xq, sx, 0, rows, want_isum=True)
    ref_isum = (q.astype(np.int32).reshape(rows, -1, 32) * xq[0].astype(np.int32).reshape(1, -1, 32)).sum(-1)
    assert np.array_equal(isum, ref_isum)
    ref = s.astype(np.float64) * (isum * sx[0][None, :].astype(np.float64)).sum(1)
    assert O.normwise_rel_err(logits, ref) < 1e-6
    assert am == int(np.argmax(logits))
    # ties: duplicate the best row further down; the first index must win
    q2 = np.concatenate([q, q[am:am + 1]], 0)
    s2 = np.concatenate([s, s[am:am + 1]])
    _, _, am2 = O.q8_lmhead(q2, s2, xq, sx, 0, rows + 1)
    assert am2 == am
    # a row range reports absolute row numbers
    lg, _, am3 = O.q8_lmhead(q, s, xq, sx, 100, 200)
    assert np.array_equal(lg, logits[100:200]) and am3 == 100 + int(np.argmax(logits[100:200]))


def test_cpu_baseline_matches_oracle():
    rows, K = 256, 3584
    W = O.q4k_quantize(O.normal(rows * K, seed=7, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=8)
    xq, sx, sq = O.quantize_act(x)
    ref, _ = O.q4k_matmul(W, rows, K, xq, sx, sq)
    y = np.empty(rows, np.float32)
    O.lib().lalb_cpu_q4k_gemv(O._p(W), rows, K, O._p(xq), O._p(sx), O._p(sq), O._p(y))
    assert O.normwise_rel_err(y, ref[0]) < 1e-5
    q, s = O.q8_quantize_rows(O.normal(rows * K, seed=9, sigma=0.02).reshape(rows, K))
    lg_ref, _, am_ref = O.q8_lmhead(q, s, xq, sx, 0, rows)
    lg = np.empty(rows, np.float32)
    am = O.lib().lalb_cpu_q8_lmhead(O._p(q), O._p(s), rows, K, O._p(xq), O._p(sx), O._p(lg))
    assert O.normwise_rel_err(lg, lg_ref) < 1e-5 and am == am_ref


def test_swiglu_and_rms_oracle():
    g = O.normal(4096, seed=12)
    u = O.normal(4096, seed=13)
    a = O.swiglu(g, u)
    ref = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.max(np.abs(a - ref) / np.maximum(np.abs(ref), 1e-30)) < 1e-6
    x = O.normal(3584, seed=14) * 7
    xn = O.rms_normalise(x)
    assert abs(np.sqrt(np.mean(xn.astype(np.float64) ** 2)) - 1) < 1e-5


def test_rms_norm_oracle_pinned_to_reference():
    """The oracle's rms_norm against the reference's own (runtime/lal_runtime.c
    :82-87, compiled from its source tree; tests/golden/decode_ref.npz).  The
    reference sums the squares in float, the oracle in double: the scales
    differ by at most a few float roundings."""
    g = np.load(os.path.join(GOLD, "decode_ref.npz"))
    for i in range(4):
        x, w, y = g[f"rms{i}_x"], g[f"rms{i}_w"], g[f"rms{i}_y"]
        o = O.rms_normalise(x, w, 1e-5)
        assert O.normwise_rel_err(o, y) < 2e-6, i
    # unit weights are rms_norm with w = 1
    x = g["rms0_x"]
    assert np.array_equal(O.rms_normalise(x), O.rms_normalise(x, np.ones_like(x)))


def test_attention_oracle_pinned_to_reference():
    """The oracle's decode attention with n_kv = n_head (the reference's
    multi-head case) against the reference's apply_rope + attention_forward
    (tests/golden/decode_ref.npz).  The reference forms the RoPE angle and
    the softmax in float, the oracle in double: they agree to ~1e-5."""
    g = np.load(os.path.join(GOLD, "decode_ref.npz"))
    for i in range(5):
        n_embd, n_head, pos = (int(v) for v in g[f"att{i}_shape"])
        hd = n_embd // n_head
        kc = np.zeros((pos + 1, n_embd), np.float32)
        vc = np.zeros((pos + 1, n_embd), np.float32)
        kc[:pos], vc[:pos] = g[f"att{i}_k_in"][:pos], g[f"att{i}_v_in"][:pos]
        out = O.attention_decode(g[f"att{i}_qkv"], n_head, n_head, hd, pos, kc, vc)
        assert O.normwise_rel_err(out, g[f"att{i}_out"]) < 1e-4, i
        assert O.normwise_rel_err(kc[pos], g[f"att{i}_k_row"]) < 1e-5, i
        assert np.array_equal(vc[pos], g[f"att{i}_v_row"]), i
        # the rotated q/k the reference attended with
        q_ref = g[f"att{i}_qkv_rope"][:n_embd]
        assert q_ref.shape[0] == n_embd
    # grouped KV heads: every head of a group attends the same cache rows
    rng = np.random.default_rng(3)
    n_head, n_kv, hd, pos = 8, 2, 64, 9
    qkv = rng.standard_normal((n_head + 2 * n_kv) * hd).astype(np.float32)
    kc = rng.standard_normal((pos + 1, n_kv * hd)).astype(np.float32)
    vc = rng.standard_normal((pos + 1, n_kv * hd)).astype(np.float32)
    out = O.attention_decode(qkv, n_head, n_kv, hd, pos, kc.copy(), vc.copy())
    # head 5 is in group 1: the same as a one-head, one-KV-head call on its slices
    q5 = qkv[5 * hd:6 * hd]
    k1 = qkv[n_head * hd + hd:n_head * hd + 2 * hd]
    v1 = qkv[(n_head + n_kv) * hd + hd:(n_head + n_kv) * hd + 2 * hd]
    out5 = O.attention_decode(np.concatenate([q5, k1, v1]), 1, 1, hd, pos,
                              np.ascontiguousarray(kc[:, hd:]), np.ascontiguousarray(vc[:, hd:]))
    assert np.array_equal(out[5 * hd:6 * hd], out5)


def test_sampling_oracle_known_answers():
    """generate_text's sampling (models/ste_train.c:2229-2318), cases worked
    out by hand from the reference code (it cannot be called on its own: it
    lives inside the trainer's generation loop)."""
    # greedy: the first maximum (sample_argmax, :1503-1509)
    assert O.sample([1, 3, 3, 2])[0] == 1
    # the special ids are masked (:2243-2245)
    assert O.sample([9, 9, 9, 1, 2], n_masked_low_ids=3)[0] == 4
    # repetition penalty once per distinct token (:2254-2264): 2/1.5 < 1.9
    assert O.sample([2.0, 1.9, -1.0, -1.2], history=[0, 0, 3], rep_penalty=1.5)[0] == 1
    tok, _, _ = O.sample([-1.0, -1.1], history=[0], rep_penalty=1.5)   # -1 * 1.5 < -1.1
    assert tok == 1
    # no-repeat trigram (:2270-2281): (5, 6) was followed by 7 once
    lg = np.zeros(10, np.float32)
    lg[7], lg[3] = 5.0, 4.0
    assert O.sample(lg, history=[5, 6, 7, 5, 6], no_repeat_ngram=3)[0] == 3
    assert O.sample(lg, history=[5, 6, 7, 5, 6], no_repeat_ngram=0)[0] == 7
    # top-k / top-p (:2283-2318): probabilities 1, .75, .5, .25 (ids 3, 2, 1, 0)
    lg = np.log(np.array([1, 2, 3, 4], np.float32))
    tok, idx, prob = O.sample(lg, temperature=1.0, top_k=4, top_p=0.5, u=0.5)
    assert list(idx) == [3, 2, 1, 0] and np.allclose(prob, [1, .75, .5, .25], rtol=1e-6)
    assert tok == 3          # nucleus {3, 2}: running sum 1.75, r = 0.875 < 1
    assert O.sample(lg, temperature=1.0, top_k=4, top_p=0.5, u=0.9)[0] == 2   # r = 1.575
    assert O.sample(lg, temperature=1.0, top_k=4, top_p=1.0, u=0.5)[0] == 2   # r = 1.25
    assert O.sample(lg, temperature=1.0, top_k=2, top_p=1.0, u=0.99)[0] == 2
    # ties: lower id first here; the reference's selection sort reorders them
    t = np.array([5, 9, 5, 9], np.float32)
    assert list(O.sample(t, temperature=1.0, top_k=4, tie_rule=0)[1]) == [1, 3, 0, 2]
    assert list(O.sample(t, temperature=1.0, top_k=4, tie_rule=1)[1]) == [1, 3, 2, 0]
    # distinct values: both rules agree
    r = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    for k in (1, 8, 50):
        a = O.sample(r, temperature=0.7, top_k=k, u=0.3, tie_rule=0)
        b = O.sample(r, temperature=0.7, top_k=k, u=0.3, tie_rule=1)
        assert a[0] == b[0] and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


def test_decode_chain_oracle_small():
    cfg = dict(hidden=256, q_rows=256, kv_rows=64, ffn=512)
    layers = []
    for l in range(2):
        def qw(rows, K, s):
            return O.q4k_quantize(O.normal(rows * K, seed=s, sigma=0.02).reshape(rows, K))
        layers.append(dict(wqkv=qw(256 + 128, 256, 20 + 4 * l), wo=qw(256, 256, 21 + 4 * l),
                           wgu=qw(1024, 256, 22 + 4 * l), wdown=qw(256, 512, 23 + 4 * l)))
    lq, ls = O.q8_quantize_rows(O.normal(500 * 256, seed=99, sigma=0.02).reshape(500, 256))
    h, logits, am = O.decode_chain(layers, lq, ls, O.normal(256, seed=100), cfg)
    assert np.all(np.isfinite(h)) and np.all(np.isfinite(logits)) and 0 <= am < 500


def test_normal_generator_moments():
    z = O.normal(1 << 20, seed=1)
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1) < 5e-3
    a = O.normal(1000, seed=1, offset=500)
    assert np.array_equal(a[:10], z[500:510])


def test_binlayer_oracle_matches_reference_goldens():
    """The restated BinLayer forward against the reference's own compiled
    bin_forward / bin_forward_pure_float (tests/golden/binlayer_ref.npz)."""
    g = np.load(os.path.join(GOLD, "binlayer_ref.npz"))
    for ci in range(3):
        W, b, mask, X = (g[f"bl{ci}_{k}"] for k in ("W", "b", "mask", "X"))
        for mode in (0, 1):
            for repack in (0, 1):
                Y, alpha = O.binlayer_forward(W, b, mask, X, mode, repack=bool(repack))
                ref = g[f"bl{ci}_m{mode}_r{repack}_Y"]
                assert O.normwise_rel_err(Y, ref) < 1e-5, (ci, mode, repack)
                np.testing.assert_allclose(alpha, g[f"bl{ci}_m{mode}_r{repack}_alpha"], rtol=2e-6,
                                           atol=0)


def test_logic_pack_and_forward_oracle():
    rows, K, M = 40, 96, 3
    W = O.normal(rows * K, seed=11, sigma=0.02).reshape(rows, K)
    st = O.logic_state(12, rows * K, 0.10, 0.50).reshape(rows, K)
    frac = np.bincount(st.ravel(), minlength=3) / st.size
    assert abs(frac[0] - 0.10) < 0.03 and abs(frac[1] - 0.50) < 0.04
    codes, srow = O.logic_pack(W, st)
    assert np.all(codes[st == 2] == 0) and np.all(np.abs(codes) <= 127)
    # BINARY codes are +-b per row, sign of w
    for j in range(rows):
        bj = np.abs(codes[j][st[j] == 1])
        assert bj.size == 0 or (np.all(bj == bj[0]) and bj[0] >= 1)
        assert np.all(np.sign(codes[j][st[j] == 1]) == np.where(W[j][st[j] == 1] > 0, 1, -1))
    X = O.normal(M * K, seed=13).reshape(M, K)
    bias = O.normal(rows, seed=14, sigma=0.01)
    Y = O.logic_forward(codes, srow, bias, X)
    ref = (X.astype(np.float64) @ codes.T.astype(np.float64)) * srow + bias
    assert O.normwise_rel_err(Y, ref) < 1e-6
