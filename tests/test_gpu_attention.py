"""Decode attention on the GPU against the oracle.

The oracle (oracle/lalb_oracle.c lalb_o_attention_decode) restates the
reference's apply_rope + attention_forward (runtime/lal_runtime.c:137-153,
833-882) for grouped KV heads in double, and is pinned to the reference's
own compiled functions by tests/test_oracle.py.  The GPU computes the same
double-precision arithmetic in another order, so outputs and the cache rows
it writes agree to the last float bit almost everywhere.
"""
import numpy as np
import pytest
import torch

import _oracle as O
import lalmodel_b200 as lb
from test_gpu_kernels import assert_fp32_parity, dev, host, make_decoder_weights, set_layers

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_head,n_kv,hd,pos,theta", [
    (28, 4, 128, 0, 10000.0),       # Qwen2.5-7B heads, first token
    (28, 4, 128, 1, 1e6),
    (28, 4, 128, 63, 10000.0),
    (28, 4, 128, 1000, 1e6),
    (8, 8, 64, 17, 10000.0),        # the reference's multi-head case
    (4, 1, 256, 5, 10000.0),
    (16, 2, 32, 300, 10000.0),
])
def test_attention_decode_matches_oracle(ctx, n_head, n_kv, hd, pos, theta):
    rng = np.random.default_rng(pos + 7 * n_head + hd)
    max_ctx = pos + 3
    kvr = n_kv * hd
    qkv = rng.standard_normal((n_head + 2 * n_kv) * hd).astype(np.float32)
    kc = np.zeros((max_ctx, kvr), np.float32)
    vc = np.zeros((max_ctx, kvr), np.float32)
    kc[:pos] = rng.standard_normal((pos, kvr)).astype(np.float32)
    vc[:pos] = rng.standard_normal((pos, kvr)).astype(np.float32)
    kd, vd = dev(kc), dev(vc)
    out = ctx.attention_decode(dev(qkv), n_head, n_kv, hd, pos, kd, vd, rope_theta=theta)
    ref = O.attention_decode(qkv, n_head, n_kv, hd, pos, kc, vc, theta)
    assert_fp32_parity(host(out), ref, tol=1e-6, exact_frac=0.99)
    gk, gv = host(kd), host(vd)
    assert np.array_equal(gv, vc)                          # v row stored as is
    assert np.array_equal(gk[:pos], kc[:pos]) and not gk[pos + 1:].any()
    assert_fp32_parity(gk[pos], kc[pos], tol=1e-6, exact_frac=0.99)   # rotated k


def test_attention_decode_rejects_bad_arguments(ctx):
    q = torch.zeros(1024, dtype=torch.float32, device="cuda")
    c = torch.zeros(4 * 512, dtype=torch.float32, device="cuda")
    for args, status in [((8, 3, 64, 0), -1),      # KV heads do not divide the heads
                         ((8, 2, 48, 0), -4),      # head_dim not 32/64/128/256
                         ((8, 2, 64, 4), -1)]:     # pos == max_ctx (4 rows of 2*64)
        with pytest.raises(lb.LalbError) as e:
            ctx.attention_decode(q, *args, c[:4 * 128], c[:4 * 128])
        assert e.value.status == status


ATT_CFGS = [
    dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000, head_dim=64,
         max_ctx=40),
    dict(n_layer=1, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=20000, head_dim=128,
         max_ctx=400, rope_theta=1e6),
    # the largest head: 4 heads of 256 over one KV head; from position 7 the
    # persistent kernel's 8 chunks' partials fill the merge area exactly
    dict(n_layer=1, hidden=1024, q_rows=1024, kv_rows=256, ffn=2048, vocab=3000, head_dim=256,
         max_ctx=40),
]


def run_decoder_tokens(ctx, cfg, path, start, n_tok, seed, n_rank=1):
    """Decodes n_tok tokens from position `start` (caches 0..start-1 filled
    at random) on the GPU and on the oracle; returns the per-token results."""
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=seed, n_vocab=cfg["vocab"], norms=True)
    rng = np.random.default_rng(seed)
    kv = []
    for _ in range(cfg["n_layer"]):
        kc = np.zeros((cfg["max_ctx"], cfg["kv_rows"]), np.float32)
        vc = np.zeros_like(kc)
        kc[:start] = rng.standard_normal((start, cfg["kv_rows"])).astype(np.float32)
        vc[:start] = rng.standard_normal((start, cfg["kv_rows"])).astype(np.float32)
        kv.append((kc, vc))
    kv_dev = [(dev(k), dev(v)) for k, v in kv]
    lqd, lsd = dev(lq), dev(ls)
    if n_rank == 1:
        dec = lb.Decoder(ctx, **cfg)
        dec.set_path(path)
        set_layers(dec, dl)
        dec.set_lm_head(lqd, lsd)
    else:
        from test_gpu_tp import load_shards
        dec = lb.Decoder(ctx, **cfg, n_rank=n_rank, rank=-1)
        for r in range(n_rank):
            load_shards(dec, r, cfg, dl, lqd, lsd)
    for l, (k, v) in enumerate(kv_dev):
        dec.set_kv_cache(l, k, v)
    h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    res = []
    with torch.cuda.stream(s):
        dec.set_position(start)
        for t in range(n_tok):
            h_in = O.normal(cfg["hidden"], seed=seed + 100 + t)
            ref = O.decode_chain(layers, lq, ls, h_in, cfg, kv=kv, pos=start + t)
            dec.step(dev(h_in), h_out, logits, am)
            s.synchronize()
            res.append((host(h_out).copy(), host(logits).copy(), int(host(am)[0]), ref))
    assert dec.position() == start + n_tok
    caches = [(host(k), host(v)) for k, v in kv_dev]
    dec.close()
    return res, caches, kv


@pytest.mark.parametrize("path", [lb.Decoder.KERNELS, lb.Decoder.PERSISTENT],
                         ids=["kernels", "persistent"])
@pytest.mark.parametrize("ci,start,n_tok", [(0, 0, 4), (0, 30, 2), (1, 300, 2), (2, 30, 2)],
                         ids=["small", "small-8-chunks", "qwen", "hd256-8-chunks"])
def test_decoder_with_attention_matches_oracle(ctx, path, ci, start, n_tok):
    """Tokens at consecutive positions: the attention output feeds o, the
    caches grow by one row per token; both decode paths match the oracle.
    From position 30 the persistent kernel splits each of the 8 heads over
    8 position chunks (the most it uses), whose partials one chunk merges."""
    res, caches, kv = run_decoder_tokens(ctx, ATT_CFGS[ci], path, start, n_tok, seed=3300 + ci)
    for h, logits, am, (ref_h, ref_logits, ref_am) in res:
        assert_fp32_parity(h, ref_h, exact_frac=0.99)
        assert_fp32_parity(logits, ref_logits, exact_frac=0.99)
        assert am == ref_am
    for (gk, gv), (rk, rv) in zip(caches, kv):
        assert_fp32_parity(gk, rk, exact_frac=0.99)
        assert_fp32_parity(gv, rv, exact_frac=0.99)


def test_tp_emulated_ranks_with_attention_match_oracle(ctx):
    res, caches, kv = run_decoder_tokens(ctx, ATT_CFGS[0], lb.Decoder.PERSISTENT, 5, 3,
                                         seed=3400, n_rank=2)
    for h, logits, am, (ref_h, ref_logits, ref_am) in res:
        assert_fp32_parity(h, ref_h, exact_frac=0.99)
        assert_fp32_parity(logits, ref_logits, exact_frac=0.99)
        assert am == ref_am


def test_decoder_refuses_a_full_kv_cache(ctx):
    cfg = dict(ATT_CFGS[0], max_ctx=3)
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=3500, n_vocab=cfg["vocab"])
    dec = lb.Decoder(ctx, **cfg)
    set_layers(dec, dl)
    lqd, lsd = dev(lq), dev(ls)
    dec.set_lm_head(lqd, lsd)
    bufs = [torch.zeros(3 * cfg["kv_rows"], dtype=torch.float32, device="cuda") for _ in range(4)]
    dec.set_kv_cache(0, bufs[0], bufs[1])
    with pytest.raises(lb.LalbError):      # layer 1's cache is missing
        dec.step(dev(O.normal(cfg["hidden"], seed=1)))
    dec.set_kv_cache(1, bufs[2], bufs[3])
    h = dev(O.normal(cfg["hidden"], seed=1))
    for _ in range(3):
        dec.step(h)
    assert dec.position() == 3
    with pytest.raises(lb.LalbError) as e:
        dec.step(h)
    assert e.value.status == -1
    dec.set_position(0)
    dec.step(h)
    torch.cuda.synchronize()
    assert ctx.device_status() == 0
    dec.close()
