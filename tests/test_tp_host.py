"""Tensor-parallel decode: host-side logic on CPU.

Row shards (lalb_tp_rows and its Python statement: qkv and o whole on every
rank, gate/up, down and the LM head split), the reassembly of sharded
row-major weights, and the gathering of every rank's exchange-buffer
handle over a 2-rank gloo process group.  The device path is covered by the
gpu-marked tests in test_gpu_tp.py."""
import ctypes
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import lalmodel_b200 as lb
from lalmodel_b200 import _abi

QWEN = dict(n_layer=28, hidden=3584, q_rows=3584, kv_rows=512, ffn=18944, vocab=152064)
SMALL = dict(n_layer=2, hidden=512, q_rows=256, kv_rows=128, ffn=1024, vocab=3001)


def lib_rows(cfg, n, r, m):
    c = _abi.DecoderCfg(cfg["n_layer"], cfg["hidden"], cfg["q_rows"], cfg["kv_rows"],
                        cfg["ffn"], cfg["vocab"])
    r0, r1 = ctypes.c_int(), ctypes.c_int()
    st = _abi.lib().lalb_tp_rows(ctypes.byref(c), n, r, m, ctypes.byref(r0), ctypes.byref(r1))
    assert st == 0
    return r0.value, r1.value


@pytest.mark.parametrize("cfg", [QWEN, SMALL])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shards_partition_the_split_matrices(cfg, n):
    totals = [cfg["q_rows"] + 2 * cfg["kv_rows"], cfg["hidden"], 2 * cfg["ffn"], cfg["hidden"],
              cfg["vocab"]]
    for m, total in enumerate(totals):
        bounds = [lb.tp_range(cfg, m, n, r) for r in range(n)]
        assert bounds == [lib_rows(cfg, n, r, m) for r in range(n)]
        if m in (0, 1):   # qkv and o: every rank holds every row
            assert bounds == [(0, total)] * n
            continue
        assert bounds[0][0] == 0 and bounds[-1][1] == total
        for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
            assert a1 == b0 and a0 <= a1
        if m == 2:   # gate/up shards hold whole 64-row tiles (32 gate + 32 up rows)
            assert all(r0 % 64 == 0 and r1 % 64 == 0 for r0, r1 in bounds)


def test_tp_rows_rejects_bad_arguments():
    c = _abi.DecoderCfg(1, 256, 256, 0, 256, 10)
    r0, r1 = ctypes.c_int(), ctypes.c_int()
    for n, r, m in [(0, 0, 0), (9, 0, 0), (2, 2, 0), (2, -1, 0), (2, 0, 5)]:
        assert _abi.lib().lalb_tp_rows(ctypes.byref(c), n, r, m, ctypes.byref(r0),
                                       ctypes.byref(r1)) == -1


def test_row_shards_reassemble_q4k_bytes():
    rows, K = 300, 512
    w = np.random.default_rng(3).integers(0, 256, size=(rows, K // 256 * 144), dtype=np.uint8)
    t = torch.from_numpy(w)
    cfg = dict(SMALL, hidden=rows)
    parts = [lb.shard_rows(t, *lb.tp_range(cfg, 3, 3, r)) for r in range(3)]
    assert all(p.is_contiguous() for p in parts)
    assert torch.equal(torch.cat(parts), t)


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * lb.IPC_HANDLE_BYTES
        got = lb.exchange_handles(mine)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_handles_gathered_in_rank_order_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [bytes([0]) * 64, bytes([1]) * 64]
    assert results[0] == want and results[1] == want
