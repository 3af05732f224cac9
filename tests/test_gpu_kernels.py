"""GPU parity tests: the sm_100a kernels through the C ABI against the oracle.

Bar: integer and byte results (quantized weights and activations, int32
sub-block / block dot products, argmax) bit-exact; fp32 outputs within a
normwise relative error of 1e-5 (max |gpu - oracle| / max |oracle|).  The
kernels round every fp32 sub-block term as the oracle does and sum the
terms in double, so in practice the fp32 outputs are bit-identical too;
the tests also require that for all but a handful of elements.
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


def assert_fp32_parity(got, ref, tol=TOL, exact_frac=0.999):
    got = np.asarray(got, np.float32).reshape(-1)
    ref = np.asarray(ref, np.float32).reshape(-1)
    assert O.normwise_rel_err(got, ref) < tol
    assert np.mean(got.view(np.uint32) == ref.view(np.uint32)) >= exact_frac


# ---------------------------------------------------------------- quantizers
def test_fill_normal_matches_oracle(ctx):
    n = 1 << 20
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.fill_normal(out, seed=5, sigma=0.02, offset=123)
    ref = O.normal(n, seed=5, sigma=0.02, offset=123)
    g = host(out)
    # single-precision Box-Muller on the GPU vs double on the CPU: a few ulps
    assert np.max(np.abs(g - ref)) <= 1e-5 * 0.02 * 8
    assert abs(float(g.std()) / 0.02 - 1) < 0.01


@pytest.mark.parametrize("rows,K", [(64, 256), (37, 3584), (8, 18944)])
def test_q4k_quantizer_bit_exact(ctx, rows, K):
    w = O.normal(rows * K, seed=rows + K, sigma=0.02).reshape(rows, K)
    w[0, :256] = 0.0
    w[-1, :32] = 0.25
    g = host(ctx.q4k_quantize(dev(w)))
    ref = O.q4k_quantize(w)
    assert np.array_equal(g, ref)


def test_q8_row_and_activation_quantizers_bit_exact(ctx):
    w = O.normal(97 * 3584, seed=9, sigma=0.02).reshape(97, 3584)
    q, s = ctx.q8_quantize_rows(dev(w))
    rq, rs = O.q8_quantize_rows(w)
    assert np.array_equal(host(q), rq) and np.array_equal(host(s).view(np.uint32), rs.view(np.uint32))
    x = O.normal(5 * 4096, seed=10).reshape(5, 4096)
    x[1, :32] = 0.0
    xq, sx, sq = ctx.quantize_act(dev(x))
    rxq, rsx, rsq = O.quantize_act(x)
    assert np.array_equal(host(xq), rxq)
    assert np.array_equal(host(sx).view(np.uint32), rsx.view(np.uint32))
    assert np.array_equal(host(sq), rsq)


# ------------------------------------------------------------ Q4_K matvec
def q4k_case(rows, K, seed):
    W = O.q4k_quantize(O.normal(rows * K, seed=seed, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=seed + 1)
    return W, x


@pytest.mark.parametrize("rows,K", [
    (18944, 3584),   # single GEMV of the q4k unit-test shape (gate/up rows)
    (3584, 18944),   # down projection shape (K split over 4 warps per row)
    (512, 3584),     # k / v projection
    (1, 256), (7, 512), (13, 768), (100, 8192), (3, 4352), (5, 32768),
])
def test_q4k_gemv_parity(ctx, rows, K):
    W, x = q4k_case(rows, K, seed=rows * 7 + K)
    xq, sx, sq = O.quantize_act(x)
    ref, ref_isum = O.q4k_matmul(W, rows, K, xq, sx, sq, want_isum=True)
    Wd = dev(W)
    # pre-quantized path with the int32 sub-block dump: bit-exact integers
    y8, isum = ctx.matmul_q4_k_q8(Wd, dev(xq[0]), dev(sx[0]), dev(sq[0]), rows, K, want_isum=True)
    assert np.array_equal(host(isum), ref_isum[0])
    assert_fp32_parity(host(y8), ref[0])
    # fused-quantizer path: same activation bytes, so the same fp32 result
    y = ctx.matmul_q4_k(Wd, dev(x), rows, K)
    assert np.array_equal(host(y).view(np.uint32), host(y8).view(np.uint32))
    # and the reference-named wrapper
    y2 = lb.lal_matmul_q4_k(Wd, dev(x), rows, K, ctx=ctx)
    assert np.array_equal(host(y2), host(y))


def test_q4k_gemv_sees_weights_written_by_the_previous_kernel(ctx):
    """The standalone matvec overlaps the preceding kernel in the stream
    (programmatic dependent launch) but must see what that kernel wrote: W
    re-quantized into the same buffer by the GPU quantizer right before each
    call, alternating between two matrices, with no host synchronisation."""
    rows, K = 4096, 3584
    wa = O.normal(rows * K, seed=91, sigma=0.02).reshape(rows, K)
    wb = O.normal(rows * K, seed=92, sigma=0.02).reshape(rows, K)
    x = O.normal(K, seed=93)
    xq, sx, sq = O.quantize_act(x)
    refs = [O.q4k_matmul(O.q4k_quantize(w), rows, K, xq, sx, sq)[0][0] for w in (wa, wb)]
    wd = [dev(wa), dev(wb)]
    xd = dev(x)
    Wd = ctx.q4k_quantize(wd[0])
    ys = []
    for i in range(6):
        ctx.q4k_quantize(wd[i % 2], out=Wd)   # the kernel right before the matvec writes W
        ys.append(ctx.matmul_q4_k(Wd, xd, rows, K))
    torch.cuda.synchronize()
    for i, y in enumerate(ys):
        assert_fp32_parity(host(y), refs[i % 2])


def test_q4k_gemv_rejects_bad_arguments(ctx):
    W = torch.zeros(4 * 144 * 2 + 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(512, dtype=torch.float32, device="cuda")
    with pytest.raises(lb.LalbError) as e:
        ctx.matmul_q4_k(W[1:], x, 4, 512)          # misaligned weights
    assert e.value.status == -1
    with pytest.raises(lb.LalbError) as e:
        ctx.matmul_q4_k(W, x, 4, 500)              # K not a multiple of 256
    assert e.value.status == -1
    with pytest.raises(lb.LalbError) as e:
        ctx.matmul_q4_k(W, x, 1, 32768 + 256)      # beyond the shared-memory plan
    assert e.value.status == -4


# ---------------------------------------------------------------- LM head
def test_lm_head_full_size_parity(ctx):
    rows, K = 152064, 3584
    w = torch.empty(rows * K, dtype=torch.float32, device="cuda")
    ctx.fill_normal(w, seed=77, sigma=0.02)
    q, s = ctx.q8_quantize_rows(w.view(rows, K))
    del w
    x = O.normal(K, seed=78)
    xq, sx, _ = O.quantize_act(x)
    logits, isum, am = ctx.lm_head_int8_q8(q, s, dev(xq[0]), dev(sx[0]), 0, rows, want_isum=True)
    qh, sh = host(q), host(s)
    ref, ref_isum, ref_am = O.q8_lmhead(qh, sh, xq, sx, 0, rows, want_isum=True)
    assert np.array_equal(host(isum), ref_isum)
    g = host(logits)
    assert_fp32_parity(g, ref)
    assert int(host(am)[0]) == int(np.argmax(g))
    assert int(host(am)[0]) == ref_am
    # fused-quantizer entry point agrees bit for bit
    lg2, am2 = ctx.lm_head_int8_range(q, s, dev(x), 0, rows)
    assert np.array_equal(host(lg2).view(np.uint32), g.view(np.uint32))
    assert int(host(am2)[0]) == ref_am


@pytest.mark.parametrize("r0,r1", [(0, 1), (5, 6), (3, 1000), (999, 1000), (17, 263)])
def test_lm_head_row_ranges(ctx, r0, r1):
    rows, K = 1000, 1024
    q, s = O.q8_quantize_rows(O.normal(rows * K, seed=31, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=32)
    xq, sx, _ = O.quantize_act(x)
    ref, _, ref_am = O.q8_lmhead(q, s, xq, sx, r0, r1)
    lg, am = lb.lal_lm_head_int8_range(dev(q), dev(s), dev(x), r0, r1, ctx=ctx)
    assert_fp32_parity(host(lg), ref)
    assert int(host(am)[0]) == ref_am


def test_lm_head_ties_first_index_wins_and_repeatable(ctx):
    rows, K = 4096, 512
    q, s = O.q8_quantize_rows(O.normal(rows * K, seed=41, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=42)
    xq, sx, _ = O.quantize_act(x)
    _, _, best = O.q8_lmhead(q, s, xq, sx, 0, rows)
    # copies of the best row at several later positions, in other CTAs' ranges
    for r in (best + 1, rows // 2, rows - 1):
        if r > best:
            q[r], s[r] = q[best], s[best]
    qd, sd, xd = dev(q), dev(s), dev(x)
    for _ in range(3):  # the argmax scratch resets itself between calls
        _, am = ctx.lm_head_int8_range(qd, sd, xd, 0, rows)
        assert int(host(am)[0]) == best


def test_lm_head_empty_range_and_bad_k(ctx):
    q = torch.zeros((10, 64), dtype=torch.int8, device="cuda")
    s = torch.ones(10, dtype=torch.float32, device="cuda")
    x = torch.ones(64, dtype=torch.float32, device="cuda")
    _, am = ctx.lm_head_int8_range(q, s, x, 4, 4)
    assert int(host(am)[0]) == -1
    with pytest.raises(lb.LalbError) as e:   # K = 48 is not a multiple of 32
        lb._abi.call(ctx.h, "lalb_lm_head_int8_range", ctx.h, lb._p(q), lb._p(s), 48, 0, 10,
                     lb._p(x), None, None, lb._stream())
    assert e.value.status == -1


# ---------------------------------------------------------------- decoder
def make_decoder_weights(cfg, seed, n_vocab, norms=False):
    """Seeded Q4_K layers and an int8 LM head; with norms, every layer also
    gets RMSNorm weights attn_norm / ffn_norm = 1 + 0.1 N(0, 1)."""
    layers, dev_layers = [], []
    hid, qr, kv, ffn = cfg["hidden"], cfg["q_rows"], cfg["kv_rows"], cfg["ffn"]

    def qw(rows, K, s):
        return O.q4k_quantize(O.normal(rows * K, seed=s, sigma=0.02).reshape(rows, K))

    for l in range(cfg["n_layer"]):
        lw = dict(wqkv=qw(qr + 2 * kv, hid, seed + 10 * l), wo=qw(hid, qr, seed + 10 * l + 1),
                  wgu=qw(2 * ffn, hid, seed + 10 * l + 2), wdown=qw(hid, ffn, seed + 10 * l + 3))
        if norms:
            lw["attn_norm"] = (1 + O.normal(hid, seed=seed + 10 * l + 4, sigma=0.1)).astype(np.float32)
            lw["ffn_norm"] = (1 + O.normal(hid, seed=seed + 10 * l + 5, sigma=0.1)).astype(np.float32)
        layers.append(lw)
        dev_layers.append({k: dev(v) for k, v in lw.items()})
    lq, ls = O.q8_quantize_rows(O.normal(n_vocab * hid, seed=seed + 999, sigma=0.02).reshape(n_vocab, hid))
    return layers, dev_layers, lq, ls


def set_layers(dec, dl):
    for l, w in enumerate(dl):
        dec.set_layer(l, w["wqkv"], w["wo"], w["wgu"], w["wdown"], w.get("attn_norm"),
                      w.get("ffn_norm"))


@pytest.mark.parametrize("path", [lb.Decoder.KERNELS, lb.Decoder.PERSISTENT],
                         ids=["kernels", "persistent"])
@pytest.mark.parametrize("cfg", [
    dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000),
    dict(n_layer=1, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=20000),
    dict(n_layer=3, hidden=1024, q_rows=1024, kv_rows=256, ffn=4096, vocab=5000),
    dict(n_layer=0, hidden=768, q_rows=256, kv_rows=0, ffn=256, vocab=777),
    # down rows of 9216 bytes (one per chunk) and 3-4 of them per CTA: every
    # row goes through the persistent kernel's K-split of a CTA's last rows
    dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=16384, vocab=3000),
])
def test_decoder_step_matches_oracle_chain(ctx, cfg, path):
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=1000 + cfg["hidden"], n_vocab=cfg["vocab"])
    dec = lb.Decoder(ctx, **cfg)
    dec.set_path(path)
    assert dec.path() == path
    for l, w in enumerate(dl):
        dec.set_layer(l, w["wqkv"], w["wo"], w["wgu"], w["wdown"])
    lqd, lsd = dev(lq), dev(ls)
    dec.set_lm_head(lqd, lsd)
    h_in = O.normal(cfg["hidden"], seed=5)
    ref_h, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h_in, cfg)
    hd = dev(h_in)
    h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for rep in range(3):   # first call launches directly, later calls replay a graph
            h_out.zero_()
            logits.zero_()
            dec.step(hd, h_out, logits, am)
            s.synchronize()
            # every re-quantized activation is reproduced bit for bit, so the
            # chain stays on the oracle to fp32 rounding
            assert_fp32_parity(host(h_out), ref_h, exact_frac=0.99)
            assert_fp32_parity(host(logits), ref_logits, exact_frac=0.99)
            assert int(host(am)[0]) == ref_am
            if rep == 0:
                first = host(logits).copy()
            else:
                assert np.array_equal(host(logits), first)
    # default stream: direct launches, no graph
    dec.step(hd, h_out, logits, am)
    assert np.array_equal(host(logits), first)
    # host-buffer entry point: H2D input, D2H argmax, same answer
    pinned = torch.from_numpy(h_in).pin_memory()
    with torch.cuda.stream(s):
        assert dec.step_host(pinned) == ref_am
        us = dec.profile_step(hd)
    assert len(us) == 4 * cfg["n_layer"] + 1
    assert dec.launches_per_step() == (1 if path == lb.Decoder.PERSISTENT else len(us))
    assert all(u > 0 for u in us)
    dec.close()


@pytest.mark.parametrize("path", [lb.Decoder.KERNELS, lb.Decoder.PERSISTENT],
                         ids=["kernels", "persistent"])
@pytest.mark.parametrize("cfg", [
    dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000, rms_eps=1e-6),
    dict(n_layer=1, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=20000, rms_eps=0.0),
    dict(n_layer=0, hidden=768, q_rows=256, kv_rows=0, ffn=256, vocab=777, rms_eps=1e-3),
])
def test_decoder_weighted_rmsnorm_matches_oracle(ctx, cfg, path):
    """rms_norm with weights (runtime/lal_runtime.c:82-87) before qkv, gate/up
    and the LM head, at the reference's epsilon (0 selects 1e-5) and others."""
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=1500 + cfg["hidden"], n_vocab=cfg["vocab"],
                                              norms=True)
    out_norm = (1 + O.normal(cfg["hidden"], seed=1501, sigma=0.1)).astype(np.float32)
    dec = lb.Decoder(ctx, **cfg)
    dec.set_path(path)
    set_layers(dec, dl)
    lqd, lsd = dev(lq), dev(ls)
    dec.set_lm_head(lqd, lsd)
    dec.set_output_norm(dev(out_norm))
    h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for tok in range(2):
            h_in = O.normal(cfg["hidden"], seed=1502 + tok)
            ref_h, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h_in, cfg, out_norm)
            dec.step(dev(h_in), h_out, logits, am)
            s.synchronize()
            assert_fp32_parity(host(h_out), ref_h, exact_frac=0.99)
            assert_fp32_parity(host(logits), ref_logits, exact_frac=0.99)
            assert int(host(am)[0]) == ref_am
    # unit weights are not the same as these: the norms are really applied
    _, unit_logits, _ = O.decode_chain([{k: v for k, v in lw.items() if "norm" not in k}
                                        for lw in layers], lq, ls, h_in, cfg)
    assert O.normwise_rel_err(unit_logits, ref_logits) > 1e-3
    dec.close()


def test_decoder_persistent_two_tokens_and_path_switch(ctx):
    """Counters left by one token do not leak into the next: alternate
    inputs and paths on one decoder and compare each token with the oracle."""
    cfg = dict(n_layer=2, hidden=1024, q_rows=512, kv_rows=256, ffn=2048, vocab=4099)
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=77, n_vocab=cfg["vocab"])
    dec = lb.Decoder(ctx, **cfg)
    assert dec.path() == lb.Decoder.PERSISTENT   # AUTO picks it when the shapes fit
    for l, w in enumerate(dl):
        dec.set_layer(l, w["wqkv"], w["wo"], w["wgu"], w["wdown"])
    lqd, lsd = dev(lq), dev(ls)   # the decoder keeps the pointers: keep the tensors
    dec.set_lm_head(lqd, lsd)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i, path in enumerate([lb.Decoder.PERSISTENT, lb.Decoder.PERSISTENT,
                                  lb.Decoder.KERNELS, lb.Decoder.PERSISTENT]):
            dec.set_path(path)
            h_in = O.normal(cfg["hidden"], seed=300 + i)
            _, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h_in, cfg)
            hd = dev(h_in)
            dec.step(hd, None, logits, am)
            s.synchronize()
            assert_fp32_parity(host(logits), ref_logits, exact_frac=0.99)
            assert int(host(am)[0]) == ref_am
    dec.close()


def test_decoder_persistent_rejects_unfit_shapes(ctx):
    cfg = dict(n_layer=1, hidden=512, q_rows=512, kv_rows=0, ffn=24576, vocab=100)
    dec = lb.Decoder(ctx, **cfg)
    assert dec.path() == lb.Decoder.KERNELS    # ffn above the shared-memory limit
    with pytest.raises(lb.LalbError) as e:
        dec.set_path(lb.Decoder.PERSISTENT)
    assert e.value.status == -4
    with pytest.raises(lb.LalbError) as e:
        dec.set_path(7)
    assert e.value.status == -1
    dec.close()


def test_decoder_keeps_weights_passed_as_temporaries(ctx):
    """The library holds device pointers only; the Python decoder must keep
    the tensors alive, so weights built on the fly still decode correctly
    after their names are gone and the allocator has reused freed memory."""
    cfg = dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000)
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=4242, n_vocab=cfg["vocab"])
    dec = lb.Decoder(ctx, **cfg)
    for l, w in enumerate(dl):
        dec.set_layer(l, w["wqkv"].clone(), w["wo"].clone(), w["wgu"].clone(), w["wdown"].clone())
    dec.set_lm_head(dev(lq), dev(ls))
    del dl
    junk = [torch.full((1 << 20,), 255, dtype=torch.uint8, device="cuda") for _ in range(8)]
    h_in = O.normal(cfg["hidden"], seed=5)
    ref_h, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h_in, cfg)
    h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    dec.step(dev(h_in), h_out, None, am)
    assert_fp32_parity(host(h_out), ref_h)
    assert int(host(am)[0]) == ref_am
    del junk
    dec.close()
