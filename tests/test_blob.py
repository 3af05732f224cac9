"""Weight blobs (lalb_blob_*): the file format, its writer and its loader.

CPU: tensors written as they are come back byte for byte (whole and as row
ranges), the checksum catches a changed byte, malformed files are refused.
GPU: the converter's quantization equals the library's in-memory
quantizers, device loads (whole and per tensor-parallel shard) equal the
host bytes, and a decoder loaded from a blob decodes like one built in
memory.
"""
import os

import numpy as np
import pytest

import _oracle as O
from lalmodel_b200 import blob as B


def sample_tensors(rng):
    q = O.q4k_quantize(O.normal(40 * 512, seed=3, sigma=0.02).reshape(40, 512))
    return {
        "a.f32": (B.F32, rng.standard_normal((7, 33)).astype(np.float32), None),
        "b.q4k": (B.Q4K, q, [40, 512]),
        "c.i8": (B.I8, rng.integers(-127, 128, (300, 64)).astype(np.int8), None),
        "d.vec": (B.F32, rng.standard_normal(5000).astype(np.float32), None),
        "e.bf16": (B.BF16, rng.integers(0, 65535, (3, 4, 5)).astype(np.uint16), None),
    }


def write(path, tensors):
    w = B.BlobWriter(str(path))
    for k, (dt, a, dims) in tensors.items():
        w.add(k, dt, a, dims)
    w.close()


def test_blob_round_trip_is_byte_exact(tmp_path):
    ts = sample_tensors(np.random.default_rng(1))
    p = tmp_path / "w.lq4k"
    write(p, ts)
    assert os.path.getsize(p) % 128 == 0
    b = B.Blob(str(p))
    assert b.keys() == list(ts)
    for k, (dt, a, dims) in ts.items():
        inf = b.info(k)
        assert inf["dtype"] == dt and inf["dims"] == list(dims or a.shape)
        got = b.read(k)
        assert got.tobytes() == np.ascontiguousarray(a).tobytes()
        assert b.verify(k)
        # a row range is one byte range
        n = inf["dims"][0]
        r0, r1 = n // 3, n - 1
        part = b.read(k, r0, r1)
        assert part.tobytes() == np.ascontiguousarray(a).reshape(n, -1)[r0:r1].tobytes()
    with pytest.raises(KeyError):
        b.index("missing")
    b.close()


def test_blob_refuses_malformed_files_and_catches_changed_bytes(tmp_path):
    ts = sample_tensors(np.random.default_rng(2))
    p = tmp_path / "w.lq4k"
    write(p, ts)
    raw = bytearray(open(p, "rb").read())
    # one flipped byte inside a tensor: the table still parses, the checksum fails
    b = B.Blob(str(p))
    off = 4096
    b.close()
    bad = bytearray(raw)
    bad[off + 5] ^= 0x40
    open(tmp_path / "flip", "wb").write(bad)
    b = B.Blob(str(tmp_path / "flip"))
    assert not b.verify("a.f32") and b.verify("b.q4k")
    b.close()
    for name, mutate in [("magic", lambda r: r.__setitem__(0, ord("X"))),
                         ("version", lambda r: r.__setitem__(4, 9)),
                         ("truncated", lambda r: r.__delitem__(slice(len(r) - 10, None))),
                         ("empty", lambda r: r.__delitem__(slice(0, None)))]:
        m = bytearray(raw)
        mutate(m)
        open(tmp_path / name, "wb").write(m)
        with pytest.raises(B.LalbError):
            B.Blob(str(tmp_path / name))
    # the writer refuses duplicate keys, empty keys and shapes that do not fit the dtype
    w = B.BlobWriter(str(tmp_path / "w2"))
    w.add("x", B.F32, np.zeros(4, np.float32))
    for key, dt, a, dims in [("x", B.F32, np.zeros(4, np.float32), None), ("", B.F32, np.zeros(4, np.float32), None),
                             ("q", B.Q4K, np.zeros(144, np.uint8), [1, 100])]:
        with pytest.raises(B.LalbError):
            w.add(key, dt, a, dims)
    w.close()


@pytest.mark.gpu
def test_blob_converter_and_device_loads(ctx, tmp_path):
    import torch

    rows, K = 1000, 3584
    wf = O.normal(rows * K, seed=11, sigma=0.02).reshape(rows, K)
    wbf = (wf.view(np.uint32) >> 16).astype(np.uint16)      # bf16 bits (truncated)
    p = str(tmp_path / "c.lq4k")
    w = B.BlobWriter(p)
    w.add_quantized(ctx, "q", wf, B.Q4K)
    w.add_quantized(ctx, "qb", wbf, B.Q4K)
    w.add_quantized(ctx, "h", wf, B.I8, scale_key="h.s")
    w.close()
    b = B.Blob(p)
    ref = O.q4k_quantize(wf)                                   # the GPU quantizer is bit-exact to it
    assert np.array_equal(b.read("q").reshape(-1), ref.reshape(-1))
    wb32 = (wbf.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(b.read("qb").reshape(-1), O.q4k_quantize(wb32).reshape(-1))
    hq, hs = O.q8_quantize_rows(wf)
    assert np.array_equal(b.read("h"), hq) and np.array_equal(b.read("h.s"), hs)
    for key in ("q", "h", "h.s"):
        full = b.load(ctx, key)
        torch.cuda.synchronize()
        assert full.cpu().numpy().tobytes() == b.read(key).tobytes()
        part = b.load(ctx, key, 123, 777)
        torch.cuda.synchronize()
        assert part.cpu().numpy().tobytes() == b.read(key, 123, 777).tobytes()
    b.close()


@pytest.mark.gpu
def test_decoder_from_blob_matches_decoder_from_memory(ctx, tmp_path):
    import torch

    import lalmodel_b200 as lb
    from test_gpu_kernels import host

    cfg = dict(n_layer=2, hidden=512, q_rows=512, kv_rows=128, ffn=1024, vocab=3000, rms_eps=1e-6)
    hid, qr, kv, ffn = 512, 512, 128, 1024

    def f(rows, K, s):
        return O.normal(rows * K, seed=s, sigma=0.02).reshape(rows, K)

    layers = [dict(wqkv=f(qr + 2 * kv, hid, 10 + l), wo=f(hid, qr, 20 + l), wgu=f(2 * ffn, hid, 30 + l),
                   wdown=f(hid, ffn, 40 + l), attn_norm=1 + O.normal(hid, seed=50 + l, sigma=0.1),
                   ffn_norm=1 + O.normal(hid, seed=60 + l, sigma=0.1)) for l in range(2)]
    lm = f(cfg["vocab"], hid, 70)
    out_norm = 1 + O.normal(hid, seed=71, sigma=0.1)
    p = str(tmp_path / "dec.lq4k")
    B.save_decoder(p, ctx, cfg, layers, lm, out_norm)
    b = B.Blob(p)
    got_cfg = B.cfg_of(b)
    assert all(got_cfg[k] == pytest.approx(v) for k, v in cfg.items())
    dec = B.load_decoder(ctx, b)
    qlayers = [dict(wqkv=O.q4k_quantize(lw["wqkv"]), wo=O.q4k_quantize(lw["wo"]),
                    wgu=O.q4k_quantize(lw["wgu"]), wdown=O.q4k_quantize(lw["wdown"]),
                    attn_norm=lw["attn_norm"], ffn_norm=lw["ffn_norm"]) for lw in layers]
    lq, ls = O.q8_quantize_rows(lm)
    h_in = O.normal(hid, seed=72)
    ref_h, ref_logits, ref_am = O.decode_chain(qlayers, lq, ls, h_in, cfg, out_norm)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    dec.step(torch.from_numpy(h_in).cuda(), None, logits, am)
    assert O.normwise_rel_err(host(logits), ref_logits) < 1e-5
    assert int(host(am)[0]) == ref_am
    dec.close()
    b.close()
