"""Tensor-parallel decode on the GPU, against the oracle's decode chain.

* One GPU running every rank (rank=-1): the ranks are groups of CTAs of one
  cooperative launch, exchanging rows through their exchange buffers exactly
  as separate GPUs do.
* Two GPUs, one process each, peers connected with CUDA IPC (skipped when
  fewer than two GPUs are visible).
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import _oracle as O
import lalmodel_b200 as lb
from test_gpu_kernels import assert_fp32_parity, dev, host, make_decoder_weights

pytestmark = pytest.mark.gpu

CFGS = [
    dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000),
    dict(n_layer=1, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=20000),
]


def load_shards(dec, rank, cfg, dl, lqd, lsd):
    """Give `dec` rank `rank`'s row shards of the full device weights (RMSNorm
    weights, when present, whole)."""
    rows = [lb.tp_range(cfg, m, dec.n_rank, rank) for m in range(5)]
    for l, w in enumerate(dl):
        dec.set_layer_shard(rank, l, lb.shard_rows(w["wqkv"], *rows[0]),
                            lb.shard_rows(w["wo"], *rows[1]), lb.shard_rows(w["wgu"], *rows[2]),
                            lb.shard_rows(w["wdown"], *rows[3]), w.get("attn_norm"),
                            w.get("ffn_norm"))
    dec.set_lm_head_shard(rank, lb.shard_rows(lqd, *rows[4]), lb.shard_rows(lsd, *rows[4]))


@pytest.mark.parametrize("n_rank", [2, 3, 8])
@pytest.mark.parametrize("ci", [0, 1])
def test_tp_all_ranks_on_one_gpu_match_oracle(ctx, n_rank, ci):
    cfg = CFGS[ci]
    if ci == 1 and n_rank != 2:
        pytest.skip("Qwen-shape layer: two ranks suffice")
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=2000 + ci, n_vocab=cfg["vocab"],
                                              norms=(ci == 0))
    lqd, lsd = dev(lq), dev(ls)
    dec = lb.Decoder(ctx, **cfg, n_rank=n_rank, rank=-1)
    assert dec.launches_per_step() == 1
    for r in range(n_rank):
        load_shards(dec, r, cfg, dl, lqd, lsd)
    h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for tok in range(3):   # counters carry over between tokens; graph replay after the first
            h_in = O.normal(cfg["hidden"], seed=40 + tok)
            ref_h, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h_in, cfg)
            hd = dev(h_in)
            logits.zero_()
            dec.step(hd, h_out, logits, am)
            s.synchronize()
            assert_fp32_parity(host(h_out), ref_h, exact_frac=0.99)
            assert_fp32_parity(host(logits), ref_logits, exact_frac=0.99)
            assert int(host(am)[0]) == ref_am
    assert ctx.device_status() == 0
    dec.close()


def test_tp_wait_runs_out_when_a_peer_never_steps(ctx):
    """A bounded cross-GPU wait made to run out on purpose, with no fault:
    rank 0 of a two-rank decoder steps alone (rank 1's decoder exists on the
    same GPU, its exchange buffer connected, but it never launches), with a
    50 ms wait limit.  The token must end by itself within seconds, report
    the expired wait through the status word and an argmax of -1, and leave
    the context usable."""
    import time

    cfg = CFGS[0]
    layers, dl, lq, ls = make_decoder_weights(cfg, seed=2100, n_vocab=cfg["vocab"])
    lqd, lsd = dev(lq), dev(ls)
    a = lb.Decoder(ctx, **cfg, n_rank=2, rank=0)
    b = lb.Decoder(ctx, **cfg, n_rank=2, rank=1)   # connected, never steps
    load_shards(a, 0, cfg, dl, lqd, lsd)
    a.connect_local([a.exchange_buffer(), b.exchange_buffer()])
    a.set_wait_limit(0.05)
    h_in = dev(O.normal(cfg["hidden"], seed=2101))
    am = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    assert ctx.device_status() == 0
    t0 = time.perf_counter()
    with torch.cuda.stream(s):
        a.step(h_in, None, None, am)
    s.synchronize()
    dt = time.perf_counter() - t0
    assert dt < 10.0, dt
    assert ctx.device_status() == 1          # LALB_STATUS_WAIT_TIMEOUT
    assert int(am.item()) == -1
    assert ctx.device_status(reset=True) == 1
    assert ctx.device_status() == 0
    with torch.cuda.stream(s):
        a.reset()
        b.reset()
    s.synchronize()
    a.close()
    b.close()
    # the context still computes: a one-GPU decoder on the same weights
    one = lb.Decoder(ctx, **cfg)
    for l, w in enumerate(dl):
        one.set_layer(l, w["wqkv"], w["wo"], w["wgu"], w["wdown"])
    one.set_lm_head(lqd, lsd)
    h = O.normal(cfg["hidden"], seed=2102)
    _, ref_logits, ref_am = O.decode_chain(layers, lq, ls, h, cfg)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    with torch.cuda.stream(s):
        one.step(dev(h), None, logits, am)
    s.synchronize()
    assert int(am.item()) == ref_am
    assert O.normwise_rel_err(host(logits), ref_logits) < 1e-5
    assert ctx.device_status() == 0
    one.close()


def test_tp_rejects_chain_path_and_unheld_ranks(ctx):
    cfg = CFGS[0]
    dec = lb.Decoder(ctx, **cfg, n_rank=2, rank=1)
    with pytest.raises(lb.LalbError):
        dec.set_path(lb.Decoder.KERNELS)
    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(lb.LalbError):       # rank 0 lives in another process
        dec.set_layer_shard(0, 0, w, w, w, w)
    with pytest.raises(lb.LalbError):       # the whole-model call is for one rank only
        dec.set_layer(0, w, w, w, w)
    dec.close()


def _two_gpu_worker(rank, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        cfg = CFGS[0]
        layers, dl, lq, ls = make_decoder_weights(cfg, seed=3000, n_vocab=cfg["vocab"])
        lqd, lsd = dev(lq), dev(ls)
        ctx = lb.Context(rank)
        dec = lb.Decoder(ctx, **cfg, n_rank=2, rank=rank)
        load_shards(dec, rank, cfg, dl, lqd, lsd)
        dec.connect(lb.exchange_handles(dec.ipc_handle()))
        dist.barrier()
        h_out = torch.empty(cfg["hidden"], dtype=torch.float32, device="cuda")
        logits = torch.zeros(cfg["vocab"], dtype=torch.float32, device="cuda")
        am = torch.empty(1, dtype=torch.int32, device="cuda")
        r0, r1 = dec.tp_rows(rank, lb.Decoder.HEAD)
        # the oracle first: the ranks' kernels wait on each other, so keep
        # the host work between their launches alike
        toks = [O.normal(cfg["hidden"], seed=60 + tok) for tok in range(3)]
        refs = [O.decode_chain(layers, lq, ls, h_in, cfg) for h_in in toks]
        errs = []
        s = torch.cuda.Stream()
        dist.barrier()
        with torch.cuda.stream(s):
            for h_in, (ref_h, ref_logits, ref_am) in zip(toks, refs):
                dec.step(dev(h_in), h_out, logits, am)
                s.synchronize()
                errs.append((O.normwise_rel_err(host(h_out), ref_h),
                             O.normwise_rel_err(host(logits)[r0:r1], ref_logits[r0:r1]),
                             int(host(am)[0]), int(ref_am)))
        status = ctx.device_status()
        dist.barrier()   # no rank unmaps its buffer while a peer may still write to it
        dec.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, errs, status, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_two_gpus_over_nvlink_match_oracle():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, status, err in res:
        assert err is None, f"rank {rank}: {err}"
        for eh, el, am, ref_am in errs:
            assert eh < 1e-5 and el < 1e-5 and am == ref_am, (rank, errs)
        assert status == 0
