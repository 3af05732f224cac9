"""Weight blobs (include/lalb.h, lalb_blob_*): the file format of the
converted weights, its writer (the converter) and its loader.

A decoder's tensors are stored under these keys (a convention of this module
and of the integration notes; the format itself only knows names):

    decoder.cfg            I8: the raw bytes of lalb_decoder_cfg (little-endian)
    layer.{l}.wqkv, .wo, .wgu, .wdown     Q4K [rows, K]  (wgu: 32-row gate/up tiles)
    layer.{l}.attn_norm, .ffn_norm        F32 [hidden]   (optional)
    lm_head.w              I8 [vocab, hidden]
    lm_head.scale          F32 [vocab]
    output_norm            F32 [hidden]   (optional)
"""
import ctypes

import numpy as np

from . import _abi
from ._abi import BlobTensor, DecoderCfg, LalbError

F32, Q4K, I8, F16, BF16 = 0, 1, 2, 3, 4
_NP = {F32: np.float32, I8: np.int8, F16: np.float16, BF16: np.uint16, Q4K: np.uint8}


def _chk(name, st):
    if st:
        raise LalbError(name, st)


class BlobWriter:
    def __init__(self, path):
        h = ctypes.c_void_p()
        _chk("lalb_blob_writer_open", _abi.lib().lalb_blob_writer_open(path.encode(), ctypes.byref(h)))
        self.h = h

    def add(self, key, dtype, data, dims=None):
        """data: a numpy array of the tensor's bytes in dtype's layout; dims
        default to data.shape (for Q4K give [rows, K])."""
        data = np.ascontiguousarray(data)
        dims = list(dims if dims is not None else data.shape)
        arr = (ctypes.c_uint64 * len(dims))(*dims)
        _chk("lalb_blob_writer_add", _abi.lib().lalb_blob_writer_add(
            self.h, key.encode(), dtype, len(dims), arr, data.ctypes.data_as(ctypes.c_void_p)))

    def add_quantized(self, ctx, key, w, dtype=Q4K, scale_key=None):
        """w: host weights [rows, K], float32 or bfloat16 bits (uint16),
        quantized on ctx's GPU by the library's own quantizer."""
        w = np.ascontiguousarray(w)
        src = BF16 if w.dtype == np.uint16 else F32
        if src == F32:
            w = w.astype(np.float32, copy=False)
        rows, K = w.shape
        _chk("lalb_blob_writer_add_quantized", _abi.lib().lalb_blob_writer_add_quantized(
            ctx.h, self.h, key.encode(), scale_key.encode() if scale_key else None, dtype, src,
            w.ctypes.data_as(ctypes.c_void_p), rows, K))

    def close(self):
        if getattr(self, "h", None):
            st = _abi.lib().lalb_blob_writer_close(self.h)
            self.h = None
            _chk("lalb_blob_writer_close", st)


class Blob:
    def __init__(self, path):
        h = ctypes.c_void_p()
        _chk("lalb_blob_open", _abi.lib().lalb_blob_open(path.encode(), ctypes.byref(h)))
        self.h = h

    def keys(self):
        return [self.info(i)["key"] for i in range(_abi.lib().lalb_blob_count(self.h))]

    def index(self, key):
        i = _abi.lib().lalb_blob_find(self.h, key.encode())
        if i < 0:
            raise KeyError(key)
        return i

    def info(self, key):
        i = key if isinstance(key, int) else self.index(key)
        t = BlobTensor()
        _chk("lalb_blob_info", _abi.lib().lalb_blob_info(self.h, i, ctypes.byref(t)))
        return {"key": t.key.decode(), "dtype": t.dtype, "dims": list(t.dims[: t.ndim]),
                "bytes": t.bytes, "row_bytes": t.row_bytes}

    def __contains__(self, key):
        return _abi.lib().lalb_blob_find(self.h, key.encode()) >= 0

    def verify(self, key):
        return _abi.lib().lalb_blob_verify(self.h, self.index(key)) == 0

    def read(self, key, row0=0, row1=None):
        """Rows [row0, row1) as a numpy array (Q4K: uint8 [rows, row_bytes])."""
        inf = self.info(key)
        row1 = inf["dims"][0] if row1 is None else row1
        out = np.empty((row1 - row0) * inf["row_bytes"], np.uint8)
        _chk("lalb_blob_read_host", _abi.lib().lalb_blob_read_host(
            self.h, self.index(key), row0, row1, out.ctypes.data_as(ctypes.c_void_p)))
        out = out.view(_NP[inf["dtype"]])
        if inf["dtype"] == Q4K:
            return out.reshape(row1 - row0, inf["row_bytes"])
        return out.reshape([row1 - row0] + inf["dims"][1:])

    def load(self, ctx, key, row0=0, row1=None, out=None):
        """Rows [row0, row1) into a new (or the given) CUDA tensor."""
        import torch

        inf = self.info(key)
        row1 = inf["dims"][0] if row1 is None else row1
        n = (row1 - row0) * inf["row_bytes"]
        if out is None:
            out = torch.empty(n, dtype=torch.uint8, device=ctx.device)
        assert out.numel() * out.element_size() >= n
        _chk("lalb_blob_load", _abi.lib().lalb_blob_load(
            ctx.h, self.h, self.index(key), row0, row1, ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        if inf["dtype"] in (F32, I8, F16, BF16):
            tdt = {F32: torch.float32, I8: torch.int8, F16: torch.float16, BF16: torch.bfloat16}
            out = out[:n].view(tdt[inf["dtype"]]).view([row1 - row0] + inf["dims"][1:])
        return out

    def close(self):
        if getattr(self, "h", None):
            _abi.lib().lalb_blob_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def cfg_bytes(cfg):
    """lalb_decoder_cfg of a dict of decoder shapes, as raw bytes."""
    c = DecoderCfg(*(cfg.get(f, 0) for f, _ in DecoderCfg._fields_))
    return np.frombuffer(bytes(c), np.int8).copy()


def cfg_of(blob):
    raw = blob.read("decoder.cfg").tobytes()
    c = DecoderCfg.from_buffer_copy(raw)
    return {f: getattr(c, f) for f, _ in DecoderCfg._fields_}


def save_decoder(path, ctx, cfg, layers, lm_head, output_norm=None):
    """Converts a decoder's host weights into a blob.  layers: per layer a
    dict with fp32 (or bf16 bits) matrices wqkv [q+2kv, hidden], wo
    [hidden, q], wgu [2 ffn, hidden] (32-row gate/up tiles), wdown [hidden,
    ffn], optional attn_norm / ffn_norm [hidden]; lm_head: [vocab, hidden]."""
    w = BlobWriter(path)
    try:
        w.add("decoder.cfg", I8, cfg_bytes(cfg))
        for l, lw in enumerate(layers):
            for m in ("wqkv", "wo", "wgu", "wdown"):
                w.add_quantized(ctx, f"layer.{l}.{m}", lw[m], Q4K)
            for m in ("attn_norm", "ffn_norm"):
                if lw.get(m) is not None:
                    w.add(f"layer.{l}.{m}", F32, np.asarray(lw[m], np.float32))
        w.add_quantized(ctx, "lm_head.w", lm_head, I8, scale_key="lm_head.scale")
        if output_norm is not None:
            w.add("output_norm", F32, np.asarray(output_norm, np.float32))
    finally:
        w.close()


def load_decoder(ctx, blob, n_rank=1, rank=0):
    """A Decoder (lalmodel_b200.Decoder) with its weights loaded from the
    blob into device memory: rank `rank`'s row shards when n_rank > 1 (each
    process loads only its own rows).  The decoder keeps the tensors."""
    from . import Decoder, tp_range

    assert rank >= 0, "one rank per decoder: each process loads its own shard"
    cfg = cfg_of(blob)
    dec = Decoder(ctx, **cfg, n_rank=n_rank, rank=rank)
    rows = [tp_range(cfg, m, n_rank, rank) for m in range(5)]
    for l in range(cfg["n_layer"]):
        mats = [blob.load(ctx, f"layer.{l}.{m}", *rows[j])
                for j, m in enumerate(("wqkv", "wo", "wgu", "wdown"))]
        norms = [blob.load(ctx, f"layer.{l}.{m}") if f"layer.{l}.{m}" in blob else None
                 for m in ("attn_norm", "ffn_norm")]
        dec.set_layer_shard(rank, l, *mats, *norms)
    dec.set_lm_head_shard(rank, blob.load(ctx, "lm_head.w", *rows[4]),
                          blob.load(ctx, "lm_head.scale", *rows[4]))
    if "output_norm" in blob:
        dec.set_output_norm(blob.load(ctx, "output_norm"))
    return dec
