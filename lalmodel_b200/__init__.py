"""lalmodel_b200 -- LAL's quantized-matmul hot path, B200-native (sm_100a).

Host-side mirror of the reference engine's kernel interface, over the C ABI
declared in include/lalb.h and implemented by liblalb.so:

  lal_matmul_q4_k          Q4_K x Q8 matvec   (runtime/lal_q4k_kernel.h,
                                               README.md:130,210)
  lal_lm_head_int8_range   int8 LM head + argmax over a row range
                                              (runtime/lal_q8_kernel.h,
                                               README.md:131,211)
  unpack_scales_6bit       12 packed bytes -> 8 scales + 8 mins
                                              (README.md:212)

Device memory and streams come from PyTorch (plumbing only); every compute
call goes through liblalb.so on the caller's current CUDA stream.  Nothing
here computes on the CPU: a missing library or a non-sm_100 device raises.
"""
import ctypes

import torch

from . import _abi
from ._abi import DecoderCfg, LalbError, LayerWeights

QK_K = 256
QB = 32
Q4K_BLOCK_BYTES = 144

__all__ = ["Context", "Decoder", "LalbError", "lal_matmul_q4_k", "lal_lm_head_int8_range",
           "unpack_scales_6bit", "q4k_row_bytes", "QK_K", "QB", "Q4K_BLOCK_BYTES"]


def q4k_row_bytes(K):
    return (K // QK_K) * Q4K_BLOCK_BYTES


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def unpack_scales_6bit(scales12):
    """12 packed bytes -> 16 bytes (8 scales, then 8 mins); host-only helper."""
    src = (ctypes.c_uint8 * 12).from_buffer_copy(bytes(scales12))
    dst = (ctypes.c_uint8 * 16)()
    _abi.call(None, "lalb_unpack_scales_6bit", src, dst)
    return bytes(dst)


class Context:
    """One lalb_ctx bound to one CUDA device."""

    def __init__(self, device=0):
        self.device = torch.device("cuda", device)
        h = ctypes.c_void_p()
        st = _abi.lib().lalb_init(device, ctypes.byref(h))
        if st != 0:
            raise LalbError("lalb_init", st, "device %d" % device)
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            _abi.lib().lalb_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _call(self, name, *args):
        return _abi.call(self.h, name, *args)

    def device_status(self, reset=False):
        st = _abi.lib().lalb_device_status(self.h, 1 if reset else 0)
        if st < 0:
            raise LalbError("lalb_device_status", st, _abi.lib().lalb_last_error(self.h).decode())
        return st

    # ---- data and formats ------------------------------------------------
    def fill_normal(self, out, seed, sigma, offset=0):
        self._call("lalb_fill_normal", self.h, _p(out), out.numel(), seed, offset,
                   ctypes.c_float(sigma), _stream())
        return out

    def q4k_quantize(self, w, out=None):
        rows, K = w.shape
        if out is None:
            out = torch.empty((rows, q4k_row_bytes(K)), dtype=torch.uint8, device=w.device)
        self._call("lalb_q4k_quantize", self.h, _p(w), rows, K, _p(out), _stream())
        return out

    def q8_quantize_rows(self, w):
        rows, K = w.shape
        q = torch.empty((rows, K), dtype=torch.int8, device=w.device)
        s = torch.empty(rows, dtype=torch.float32, device=w.device)
        self._call("lalb_q8_quantize_rows", self.h, _p(w), rows, K, _p(q), _p(s), _stream())
        return q, s

    def quantize_act(self, x):
        M, K = x.shape if x.dim() == 2 else (1, x.shape[0])
        xq = torch.empty((M, K), dtype=torch.int8, device=x.device)
        sx = torch.empty((M, K // QB), dtype=torch.float32, device=x.device)
        sq = torch.empty((M, K // QB), dtype=torch.int32, device=x.device)
        self._call("lalb_quantize_act", self.h, _p(x), M, K, _p(xq), _p(sx), _p(sq), _stream())
        return xq, sx, sq

    # ---- hot path ----------------------------------------------------------
    def matmul_q4_k(self, W, x, rows, K, out=None):
        y = out if out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
        self._call("lalb_matmul_q4_k", self.h, _p(W), rows, K, _p(x), _p(y), _stream())
        return y

    def matmul_q4_k_q8(self, W, xq, sx, sumq, rows, K, want_isum=False):
        y = torch.empty(rows, dtype=torch.float32, device=xq.device)
        isum = (torch.empty((rows, K // QB), dtype=torch.int32, device=xq.device)
                if want_isum else None)
        self._call("lalb_matmul_q4_k_q8", self.h, _p(W), rows, K, _p(xq), _p(sx), _p(sumq),
                   _p(y), _p(isum), _stream())
        return y, isum

    def lm_head_int8_range(self, W, sw, x, row_begin, row_end, want_logits=True):
        K = W.shape[1]
        n = row_end - row_begin
        logits = torch.empty(n, dtype=torch.float32, device=x.device) if want_logits else None
        am = torch.empty(1, dtype=torch.int32, device=x.device)
        self._call("lalb_lm_head_int8_range", self.h, _p(W), _p(sw), K, row_begin, row_end,
                   _p(x), _p(logits), _p(am), _stream())
        return logits, am

    def attention_decode(self, qkv, n_head, n_kv_head, head_dim, pos, k_cache, v_cache,
                         rope_theta=10000.0, out=None):
        """One layer's decode attention at position pos (lalb_attention_decode):
        writes row pos of the caches (float32 [max_ctx][n_kv_head*head_dim])
        and returns out [n_head*head_dim]."""
        max_ctx = k_cache.numel() // (n_kv_head * head_dim)
        if out is None:
            out = torch.empty(n_head * head_dim, dtype=torch.float32, device=qkv.device)
        self._call("lalb_attention_decode", self.h, _p(qkv), n_head, n_kv_head, head_dim, pos,
                   max_ctx, ctypes.c_float(rope_theta), _p(k_cache), _p(v_cache), _p(out),
                   _stream())
        return out

    def sample(self, logits, history=None, temperature=0.0, top_k=1, top_p=0.9,
               rep_penalty=1.0, no_repeat_ngram=0, n_masked_low_ids=0, u=None, want_topk=False):
        """Next token from device logits (lalb_sample).  history: int32 CUDA
        tensor of earlier tokens (or None); u: float32 CUDA tensor [1] with
        the draw in [0, 1) (needed above temperature 0.01).  Returns the
        token tensor [1] (and the ranked ids and p_j with want_topk)."""
        vocab = logits.numel()
        n = ctypes.c_size_t()
        st = _abi.lib().lalb_sample_ws_bytes(vocab, top_k, ctypes.byref(n))
        if st:
            raise LalbError("lalb_sample_ws_bytes", st)
        ws = torch.empty(max(n.value, 8), dtype=torch.uint8, device=logits.device)
        tok = torch.empty(1, dtype=torch.int32, device=logits.device)
        k = min(top_k, vocab)
        tid = torch.empty(k, dtype=torch.int32, device=logits.device) if want_topk else None
        tpr = torch.empty(k, dtype=torch.float32, device=logits.device) if want_topk else None
        p = _abi.Sampling(temperature, top_k, top_p, rep_penalty, no_repeat_ngram, n_masked_low_ids)
        nh = 0 if history is None else history.numel()
        self._call("lalb_sample", self.h, _p(logits), vocab, _p(history), nh, ctypes.byref(p),
                   _p(u), _p(ws), _p(tok), _p(tid), _p(tpr), _stream())
        return (tok, tid, tpr) if want_topk else tok

    def lm_head_int8_q8(self, W, sw, xq, sx, row_begin, row_end, want_isum=False):
        K = W.shape[1]
        n = row_end - row_begin
        logits = torch.empty(n, dtype=torch.float32, device=xq.device)
        isum = torch.empty((n, K // QB), dtype=torch.int32, device=xq.device) if want_isum else None
        am = torch.empty(1, dtype=torch.int32, device=xq.device)
        self._call("lalb_lm_head_int8_q8", self.h, _p(W), _p(sw), K, row_begin, row_end, _p(xq),
                   _p(sx), _p(logits), _p(isum), _p(am), _stream())
        return logits, isum, am

    def measure_mma_peak(self, kind):
        """Back-to-back tcgen05.mma throughput on every SM (TFLOP/s for
        MMA_F16, TOPS for MMA_I8)."""
        v = ctypes.c_double()
        self._call("lalb_measure_mma_peak", self.h, kind, ctypes.byref(v))
        return v.value

    # ---- prefill: T tokens at once on the tensor cores ----------------------
    def matmul_q4_k_prefill(self, W, rows, K, X, ws=None, out=None):
        """Y [T][rows] = the Q4_K x Q8 matmul of each token row of X [T][K],
        straight from the Q4_K rows W (as for matmul_q4_k)."""
        T = X.shape[0]
        if ws is None:
            ws = torch.empty(prefill_ws_bytes(rows, K, T), dtype=torch.uint8, device=X.device)
        Y = out if out is not None else torch.empty((T, rows), dtype=torch.float32, device=X.device)
        self._call("lalb_matmul_q4_k_prefill", self.h, _p(W), rows, K, _p(X), T, _p(ws), _p(Y), _stream())
        return Y


MMA_F16, MMA_I8 = 0, 1   # LALB_MMA_F16, LALB_MMA_I8


def prefill_ws_bytes(rows, K, T):
    """Workspace bytes of a prefill call (the prepared tokens, split-K partial sums)."""
    ws = ctypes.c_size_t()
    st = _abi.lib().lalb_prefill_ws_bytes(rows, K, T, ctypes.byref(ws))
    if st != 0:
        raise LalbError("lalb_prefill_ws_bytes", st, "rows=%d K=%d T=%d" % (rows, K, T))
    return ws.value


IPC_HANDLE_BYTES = 64   # LALB_IPC_HANDLE_BYTES


def tp_range(cfg, matrix, n_rank, rank):
    """Pure-Python statement of lalb_tp_rows (rows [r0, r1) of `matrix` that
    `rank` of `n_rank` holds; cfg is a dict of the decoder shapes).  qkv (0)
    and o (1) are held whole by every rank; gate/up (2, whole 64-row tiles),
    down (3) and the LM head (4) are split."""
    if matrix == 0:   # qkv and o: every rank holds all rows
        return 0, cfg["q_rows"] + 2 * cfg["kv_rows"]
    if matrix == 1:
        return 0, cfg["hidden"]
    if matrix == 3:
        units, unit = cfg["hidden"], 1
    elif matrix == 2:
        units, unit = 2 * cfg["ffn"] // 64, 64
    else:
        units, unit = cfg["vocab"], 1
    return rank * units // n_rank * unit, (rank + 1) * units // n_rank * unit


def exchange_handles(handle, group=None):
    """Every rank's exchange-buffer handle in rank order, gathered over a
    torch.distributed process group (any backend)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def shard_rows(t, r0, r1):
    """Rows [r0, r1) of a row-major weight tensor (Q4_K bytes [rows][K/256*144],
    int8 [rows][K] or per-row scales [rows]) as a contiguous view."""
    return t[r0:r1]


class Decoder:
    """The Qwen2.5-shape decode matmul set (include/lalb.h, lalb_decoder_*)."""

    def __init__(self, ctx, n_layer, hidden, q_rows, kv_rows, ffn, vocab, n_rank=1, rank=0,
                 rms_eps=0.0, head_dim=0, max_ctx=0, rope_theta=0.0):
        """n_rank > 1: tensor-parallel decoder holding rank `rank` (one GPU
        per rank, peers connected with ipc_handle()/connect()), or every rank
        on this GPU with rank=-1.  rms_eps 0 selects 1e-5.  head_dim > 0
        turns the decode attention on (KV caches of max_ctx positions, set per
        layer with set_kv_cache; rope_theta 0 selects 10000)."""
        self.ctx = ctx
        self.cfg = DecoderCfg(n_layer, hidden, q_rows, kv_rows, ffn, vocab, rms_eps, head_dim,
                              max_ctx, rope_theta)
        self.n_rank, self.rank = n_rank, rank
        # the library keeps only device pointers: hold the weight tensors (a
        # shard built on the fly would otherwise be freed while still in use)
        self._keep = {}
        h = ctypes.c_void_p()
        ctx._call("lalb_decoder_create_tp", ctx.h, ctypes.byref(self.cfg), n_rank, rank,
                  ctypes.byref(h))
        self.h = h

    # matrices of lalb_tp_rows
    QKV, O, GU, DOWN, HEAD = 0, 1, 2, 3, 4

    def tp_rows(self, rank, matrix):
        """Rows [r0, r1) of `matrix` that `rank` holds (include/lalb.h)."""
        r0, r1 = ctypes.c_int(), ctypes.c_int()
        st = _abi.lib().lalb_tp_rows(ctypes.byref(self.cfg), self.n_rank, rank, matrix,
                                     ctypes.byref(r0), ctypes.byref(r1))
        if st:
            raise LalbError("lalb_tp_rows", st)
        return r0.value, r1.value

    def set_layer_shard(self, rank, layer, wqkv, wo, wgu, wdown, attn_norm=None, ffn_norm=None):
        """attn_norm / ffn_norm: RMSNorm weights [hidden] (None: unit)."""
        lw = LayerWeights(wqkv.data_ptr(), wo.data_ptr(), wgu.data_ptr(), wdown.data_ptr(),
                          _p(attn_norm), _p(ffn_norm))
        self.ctx._call("lalb_decoder_set_layer_shard", self.h, rank, layer, ctypes.byref(lw))
        self._keep[("layer", rank, layer)] = (wqkv, wo, wgu, wdown, attn_norm, ffn_norm)

    def set_lm_head_shard(self, rank, w, sw):
        self.ctx._call("lalb_decoder_set_lm_head_shard", self.h, rank, _p(w), _p(sw))
        self._keep[("head", rank)] = (w, sw)

    def ipc_handle(self):
        """This rank's exchange-buffer handle (bytes) for the other ranks."""
        buf = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
        self.ctx._call("lalb_decoder_ipc_handle", self.h, buf)
        return bytes(buf)

    def connect(self, handles):
        """handles: every rank's ipc_handle() bytes, in rank order."""
        blob = b"".join(handles)
        assert len(blob) == IPC_HANDLE_BYTES * self.n_rank
        buf = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
        self.ctx._call("lalb_decoder_connect", self.h, buf)

    def exchange_buffer(self):
        """Device address of this rank's exchange buffer (int)."""
        out = ctypes.c_void_p()
        self.ctx._call("lalb_decoder_exchange_buffer", self.h, ctypes.byref(out))
        return out.value

    def connect_local(self, bufs):
        """bufs: every rank's exchange_buffer() address, in rank order (all
        ranks in this process)."""
        arr = (ctypes.c_void_p * len(bufs))(*bufs)
        self.ctx._call("lalb_decoder_connect_local", self.h, arr)

    def set_wait_limit(self, seconds):
        self.ctx._call("lalb_decoder_set_wait_limit", self.h, ctypes.c_double(seconds))

    def reset(self):
        self.ctx._call("lalb_decoder_reset", self.h, _stream())

    def set_layer(self, layer, wqkv, wo, wgu, wdown, attn_norm=None, ffn_norm=None):
        lw = LayerWeights(wqkv.data_ptr(), wo.data_ptr(), wgu.data_ptr(), wdown.data_ptr(),
                          _p(attn_norm), _p(ffn_norm))
        self.ctx._call("lalb_decoder_set_layer", self.h, layer, ctypes.byref(lw))
        self._keep[("layer", 0, layer)] = (wqkv, wo, wgu, wdown, attn_norm, ffn_norm)

    def set_kv_cache(self, layer, k_cache, v_cache):
        """Layer `layer`'s caches: float32 CUDA tensors of max_ctx * kv_rows."""
        self.ctx._call("lalb_decoder_set_kv_cache", self.h, layer, _p(k_cache), _p(v_cache))
        self._keep[("kv", layer)] = (k_cache, v_cache)

    def set_position(self, pos):
        self.ctx._call("lalb_decoder_set_position", self.h, pos, _stream())

    def position(self):
        return _abi.lib().lalb_decoder_position(self.h)

    def set_output_norm(self, w):
        """RMSNorm weights [hidden] before the LM head (None: unit)."""
        self.ctx._call("lalb_decoder_set_output_norm", self.h, _p(w))
        self._keep[("out_norm",)] = w

    def set_lm_head(self, w, sw):
        self.ctx._call("lalb_decoder_set_lm_head", self.h, _p(w), _p(sw))
        self._keep[("head", 0)] = (w, sw)

    def step(self, h_in, h_out=None, logits=None, argmax=None):
        self.ctx._call("lalb_decoder_step", self.h, _p(h_in), _p(h_out), _p(logits),
                       _p(argmax), _stream())

    def step_host(self, h_in_host):
        """h_in_host: pinned CPU float32 tensor; returns the argmax (int)."""
        out = ctypes.c_int32(0)
        self.ctx._call("lalb_decoder_step_host", self.h, _p(h_in_host), ctypes.byref(out),
                       _stream())
        return out.value

    def phases_per_layer(self):
        return 5 if self.cfg.head_dim > 0 else 4

    def profile_step(self, h_in):
        """Per-kernel durations (microseconds) of one token on the per-phase
        kernel chain, in launch order (phases_per_layer() * n_layer + 1)."""
        n = self.phases_per_layer() * self.cfg.n_layer + 1
        buf = (ctypes.c_float * n)()
        self.ctx._call("lalb_decoder_profile_step", self.h, _p(h_in), buf, _stream())
        return list(buf)

    def trace_step(self, h_in, max_cta=1024):
        """Phase timeline of one persistent-path token: an int64 array
        [n_cta, 4*n_layer + 1, 8] per CTA and phase: GPU global-timer ns
        (work done, barrier left, prologue done, consumer-0 wait, consumer-0
        compute, producer done issuing), then the producer's and consumer 0's
        mbarrier polls."""
        import numpy as np
        n_phase = self.phases_per_layer() * self.cfg.n_layer + 1
        n = max_cta * n_phase * 8
        buf = (ctypes.c_ulonglong * n)()
        n_cta = ctypes.c_int(0)
        self.ctx._call("lalb_decoder_trace_step", self.h, _p(h_in), buf, n, ctypes.byref(n_cta),
                       _stream())
        arr = np.frombuffer(buf, dtype=np.uint64, count=n_cta.value * n_phase * 8)
        return arr.reshape(n_cta.value, n_phase, 8).astype(np.int64)

    AUTO, KERNELS, PERSISTENT = 0, 1, 2

    def set_path(self, path):
        """AUTO (persistent kernel when the shapes fit), KERNELS or PERSISTENT."""
        self.ctx._call("lalb_decoder_set_path", self.h, path)

    def path(self):
        """The path step() takes: Decoder.KERNELS or Decoder.PERSISTENT."""
        return _abi.lib().lalb_decoder_path(self.h)

    def launches_per_step(self):
        return _abi.lib().lalb_decoder_launches_per_step(self.h)

    def close(self):
        if getattr(self, "h", None):
            _abi.lib().lalb_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BinLayer:
    """The seed STE model's logic-masked layer on tensor cores (include/lalb.h,
    lalb_binlayer_*): W [out][in] fp32, bias [out] or None, mask [out] uint8
    (0 CORE, 1 BINARY, 2 PRUNE), all CUDA tensors."""

    def __init__(self, ctx, W, bias, mask, alpha_repack=False, binary_scale=0.25, max_rows=1024):
        self.ctx = ctx
        self.out_dim, self.in_dim = W.shape
        h = ctypes.c_void_p()
        ctx._call("lalb_binlayer_create", ctx.h, _p(W), _p(bias), _p(mask), self.in_dim,
                  self.out_dim, int(alpha_repack), ctypes.c_float(binary_scale), max_rows,
                  ctypes.byref(h))
        self.h = h

    def forward(self, X, mode=0, Y=None):
        """mode 0: bin_forward; mode 1: bin_forward_pure_float."""
        M = X.shape[0]
        if Y is None:
            Y = torch.empty((M, self.out_dim), dtype=torch.float32, device=X.device)
        self.ctx._call("lalb_binlayer_forward", self.h, _p(X), M, _p(Y), mode, _stream())
        return Y

    def alpha(self):
        a = torch.empty(self.out_dim, dtype=torch.float32, device="cuda")
        self.ctx._call("lalb_binlayer_alpha", self.h, _p(a), _stream())
        return a

    def close(self):
        if getattr(self, "h", None):
            _abi.lib().lalb_binlayer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LogicLayer:
    """Per-element CORE/BINARY/PRUNE weights as int8 codes with a per-row
    scale (lalb_logic_*).  The layer keeps references to srow and bias."""

    def __init__(self, ctx, codes, srow, bias=None, max_rows=1024):
        self.ctx = ctx
        self.rows, self.K = codes.shape
        self._keep = (codes, srow, bias)
        h = ctypes.c_void_p()
        ctx._call("lalb_logic_layer_create", ctx.h, _p(codes), _p(srow), _p(bias), self.rows,
                  self.K, max_rows, ctypes.byref(h))
        self.h = h

    @staticmethod
    def pack(ctx, W, state):
        rows, K = W.shape
        codes = torch.empty((rows, K), dtype=torch.int8, device=W.device)
        srow = torch.empty(rows, dtype=torch.float32, device=W.device)
        ctx._call("lalb_logic_pack", ctx.h, _p(W), _p(state), rows, K, _p(codes), _p(srow),
                  _stream())
        return codes, srow

    def forward(self, X, Y=None):
        M = X.shape[0]
        if Y is None:
            Y = torch.empty((M, self.rows), dtype=torch.float32, device=X.device)
        self.ctx._call("lalb_logic_layer_forward", self.h, _p(X), M, _p(Y), _stream())
        return Y

    def close(self):
        if getattr(self, "h", None):
            _abi.lib().lalb_logic_layer_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx = {}


def _ctx_for(t):
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if dev not in _default_ctx:
        _default_ctx[dev] = Context(dev)
    return _default_ctx[dev]


def lal_matmul_q4_k(W, x, rows, K, ctx=None):
    """y = W . x for a Q4_K matrix W [rows][K/256 blocks] and fp32 x [K]."""
    ctx = ctx or _ctx_for(x)
    return ctx.matmul_q4_k(W, x, rows, K)


def lal_lm_head_int8_range(W, sw, x, row_begin, row_end, ctx=None):
    """logits for rows [row_begin, row_end) of the int8 head, and the argmax row."""
    ctx = ctx or _ctx_for(x)
    return ctx.lm_head_int8_range(W, sw, x, row_begin, row_end)
