"""numpy-facing wrapper of the CPU oracle (oracle/liblalb_oracle.so).

Test infrastructure: the checker that the GPU results are compared with.
Builds the oracle with `make -C oracle` when the library is missing or older
than its sources.
"""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
SO = os.path.join(ORACLE_DIR, "liblalb_oracle.so")
P = ctypes.c_void_p
c_int, c_float, c_size_t, c_u64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_uint64

_SIG = {
    "lalb_o_mix64": (c_u64, [c_u64]),
    "lalb_o_fill_normal": (None, [P, c_size_t, c_u64, c_u64, c_float]),
    "lalb_o_f32_to_f16": (ctypes.c_uint16, [c_float]),
    "lalb_o_f16_to_f32": (c_float, [ctypes.c_uint16]),
    "lalb_o_unpack_scales_6bit": (None, [P, P]),
    "lalb_o_q4k_quantize": (None, [P, c_int, c_int, P]),
    "lalb_o_q4k_dequantize": (None, [P, c_int, c_int, P]),
    "lalb_o_quantize_act": (None, [P, c_int, c_int, P, P, P]),
    "lalb_o_q4k_matmul": (None, [P, c_int, c_int, P, P, P, c_int, P, P]),
    "lalb_o_q8_quantize_rows": (None, [P, c_int, c_int, P, P]),
    "lalb_o_q8_lmhead_range": (c_int, [P, P, c_int, c_int, c_int, P, P, P, P]),
    "lalb_o_argmax": (c_int, [P, c_int]),
    "lalb_o_swiglu": (None, [P, P, c_int, P]),
    "lalb_o_rms_norm": (None, [P, P, c_int, c_float, P]),
    "lalb_o_attention_decode": (None, [P, c_int, c_int, c_int, c_int, c_float, P, P, P]),
    "lalb_o_sample": (c_int, [P, c_int, P, c_int, c_float, c_int, c_float, c_float, c_int, c_int,
                              c_float, c_int, P, P]),
    "lalb_o_logic_state": (None, [c_u64, c_size_t, c_float, c_float, P]),
    "lalb_o_logic_pack": (None, [P, P, c_int, c_int, P, P]),
    "lalb_o_logic_forward": (None, [P, P, P, c_int, c_int, P, c_int, P]),
    "lalb_o_binlayer_forward": (None, [P, P, P, c_int, c_int, P, c_int, P, c_int, c_int,
                                       c_float, P]),
    "lalb_cpu_threads": (c_int, []),
    "lalb_cpu_set_threads": (None, [c_int]),
    "lalb_cpu_quantize_act": (None, [P, c_int, c_int, P, P, P]),
    "lalb_cpu_q4k_gemv": (None, [P, c_int, c_int, P, P, P, P]),
    "lalb_cpu_q8_lmhead": (c_int, [P, P, c_int, c_int, P, P, P]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(ORACLE_DIR, f) for f in ("lalb_oracle.c", "lalb_oracle.h",
                                                      "lalb_cpu_baseline.c")]
        if not os.path.exists(SO) or any(os.path.getmtime(f) > os.path.getmtime(SO) for f in srcs):
            subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
        L = ctypes.CDLL(SO)
        for k, (r, a) in _SIG.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def normal(n, seed, sigma=1.0, offset=0):
    out = np.empty(n, np.float32)
    lib().lalb_o_fill_normal(_p(out), n, seed, offset, sigma)
    return out


def q4k_quantize(w):
    rows, K = w.shape
    out = np.empty((rows, K // 256 * 144), np.uint8)
    lib().lalb_o_q4k_quantize(_p(np.ascontiguousarray(w, np.float32)), rows, K, _p(out))
    return out


def q4k_dequantize(blocks, rows, K):
    out = np.empty((rows, K), np.float32)
    lib().lalb_o_q4k_dequantize(_p(np.ascontiguousarray(blocks)), rows, K, _p(out))
    return out


def unpack_scales(s12):
    out = np.empty(16, np.uint8)
    lib().lalb_o_unpack_scales_6bit(_p(np.ascontiguousarray(s12, np.uint8)), _p(out))
    return out


def quantize_act(x):
    x = np.ascontiguousarray(x, np.float32)
    M, K = (1, x.size) if x.ndim == 1 else x.shape
    xq = np.empty((M, K), np.int8)
    sx = np.empty((M, K // 32), np.float32)
    sq = np.empty((M, K // 32), np.int32)
    lib().lalb_o_quantize_act(_p(x), M, K, _p(xq), _p(sx), _p(sq))
    return xq, sx, sq


def q4k_matmul(W, rows, K, xq, sx, sq, want_isum=False):
    M = xq.shape[0] if xq.ndim == 2 else 1
    y = np.empty((M, rows), np.float32)
    isum = np.empty((M, rows, K // 32), np.int32) if want_isum else None
    lib().lalb_o_q4k_matmul(_p(np.ascontiguousarray(W)), rows, K, _p(np.ascontiguousarray(xq)),
                            _p(np.ascontiguousarray(sx)), _p(np.ascontiguousarray(sq)), M,
                            _p(y), _p(isum))
    return y, isum


def q8_quantize_rows(w):
    rows, K = w.shape
    q = np.empty((rows, K), np.int8)
    s = np.empty(rows, np.float32)
    lib().lalb_o_q8_quantize_rows(_p(np.ascontiguousarray(w, np.float32)), rows, K, _p(q), _p(s))
    return q, s


def q8_lmhead(Wq, sw, xq, sx, r0, r1, want_isum=False):
    K = Wq.shape[1]
    logits = np.empty(r1 - r0, np.float32)
    isum = np.empty((r1 - r0, K // 32), np.int32) if want_isum else None
    am = lib().lalb_o_q8_lmhead_range(_p(Wq), _p(sw), K, r0, r1,
                                      _p(np.ascontiguousarray(xq).reshape(-1)),
                                      _p(np.ascontiguousarray(sx).reshape(-1)), _p(logits),
                                      _p(isum))
    return logits, isum, am


def swiglu(gate, up):
    act = np.empty_like(gate, dtype=np.float32)
    lib().lalb_o_swiglu(_p(np.ascontiguousarray(gate, np.float32)),
                        _p(np.ascontiguousarray(up, np.float32)), gate.size, _p(act))
    return act


def rms_normalise(x, w=None, eps=1e-5):
    """rms_norm (runtime/lal_runtime.c:82-87) through the C oracle:
    (x * s) * w with s = (float)(1/sqrt(mean(x^2) + eps)) in double."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    out = np.empty_like(x)
    wc = None if w is None else np.ascontiguousarray(w, np.float32).reshape(-1)
    lib().lalb_o_rms_norm(_p(x), _p(wc), x.size, eps, _p(out))
    return out


def attention_decode(qkv, n_head, n_kv, hd, pos, k_cache, v_cache, theta=10000.0):
    """One layer's decode attention at position pos (C oracle,
    lalb_o_attention_decode): writes row pos of the caches (float32 arrays
    [max_ctx][n_kv*hd], modified in place) and returns out [n_head*hd]."""
    qkv = np.ascontiguousarray(qkv, np.float32).reshape(-1)
    assert k_cache.flags.c_contiguous and v_cache.flags.c_contiguous
    assert k_cache.dtype == np.float32 and v_cache.dtype == np.float32
    out = np.empty(n_head * hd, np.float32)
    lib().lalb_o_attention_decode(_p(qkv), n_head, n_kv, hd, pos, theta, _p(k_cache),
                                  _p(v_cache), _p(out))
    return out


def sample(logits, history=(), temperature=0.0, top_k=1, top_p=0.9, rep_penalty=1.0,
           no_repeat_ngram=0, n_masked_low_ids=0, u=0.0, tie_rule=0):
    """generate_text's sampling on the CPU (lalb_o_sample): returns (token,
    ranked ids, p_j); tie_rule 1 is the reference's selection sort."""
    logits = np.ascontiguousarray(logits, np.float32).reshape(-1)
    hist = np.ascontiguousarray(np.asarray(history, np.int32).reshape(-1))
    k = min(top_k, logits.size)
    idx = np.empty(k, np.int32)
    prob = np.empty(k, np.float32)
    tok = lib().lalb_o_sample(_p(logits), logits.size, _p(hist) if hist.size else None, hist.size,
                              temperature, top_k, top_p, rep_penalty, no_repeat_ngram,
                              n_masked_low_ids, u, tie_rule, _p(idx), _p(prob))
    return tok, idx, prob


def decode_chain(layers, lm_q, lm_s, h_in, cfg, out_norm=None, kv=None, pos=0):
    """The decoder's per-token math on the CPU (see include/lalb.h).

    layers: list of dicts with Q4_K byte arrays wqkv, wo, wgu, wdown and
    optional RMSNorm weights attn_norm, ffn_norm; cfg["rms_eps"] (default
    1e-5) is the norm epsilon.  With cfg["head_dim"] > 0 the attention runs
    at position pos over kv, a list of per-layer (k_cache, v_cache) float32
    arrays [max_ctx][kv_rows] that are updated in place (row pos).
    Returns (h_final, logits, argmax)."""
    hid, q_rows, kvr, ffn = cfg["hidden"], cfg["q_rows"], cfg["kv_rows"], cfg["ffn"]
    eps = cfg.get("rms_eps", 0.0) or 1e-5
    hd = cfg.get("head_dim", 0)
    theta = cfg.get("rope_theta", 0.0) or 10000.0
    h = np.array(h_in, np.float32)
    for li, lw in enumerate(layers):
        xq, sx, sq = quantize_act(rms_normalise(h, lw.get("attn_norm"), eps))
        qkv, _ = q4k_matmul(lw["wqkv"], q_rows + 2 * kvr, hid, xq, sx, sq)
        if hd > 0:
            kc, vc = kv[li]
            q = attention_decode(qkv[0], q_rows // hd, kvr // hd, hd, pos, kc, vc, theta)
        else:
            q = qkv[0, :q_rows]
        xq, sx, sq = quantize_act(q)
        o, _ = q4k_matmul(lw["wo"], hid, q_rows, xq, sx, sq)
        h = (h + o[0]).astype(np.float32)
        xq, sx, sq = quantize_act(rms_normalise(h, lw.get("ffn_norm"), eps))
        gu, _ = q4k_matmul(lw["wgu"], 2 * ffn, hid, xq, sx, sq)
        gu = gu[0].reshape(-1, 2, 32)          # 32-row gate/up tiles
        act = swiglu(gu[:, 0, :].reshape(-1), gu[:, 1, :].reshape(-1))
        xq, sx, sq = quantize_act(act)
        d, _ = q4k_matmul(lw["wdown"], hid, ffn, xq, sx, sq)
        h = (h + d[0]).astype(np.float32)
    xq, sx, _ = quantize_act(rms_normalise(h, out_norm, eps))
    logits, _, am = q8_lmhead(lm_q, lm_s, xq, sx, 0, lm_q.shape[0])
    return h, logits, am


def normwise_rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / (den if den > 0 else 1.0))


def binlayer_forward(W, bias, mask, X, mode, repack=False, binary_scale=0.25):
    """The reference's logic-masked BinLayer forward (double, one rounding)."""
    W = np.ascontiguousarray(W, np.float32)
    X = np.ascontiguousarray(X, np.float32)
    mask = np.ascontiguousarray(mask, np.uint8)
    out_dim, in_dim = W.shape
    M = X.shape[0]
    Y = np.zeros((M, out_dim), np.float32)
    alpha = np.zeros(out_dim, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().lalb_o_binlayer_forward(_p(W), _p(b), _p(mask), in_dim, out_dim, _p(X), M, _p(Y), mode,
                                int(repack), binary_scale, _p(alpha))
    return Y, alpha


def logic_state(seed, n, p_core, p_binary):
    st = np.zeros(n, np.uint8)
    lib().lalb_o_logic_state(seed, n, p_core, p_binary, _p(st))
    return st


def logic_pack(W, state):
    W = np.ascontiguousarray(W, np.float32)
    rows, K = W.shape
    codes = np.zeros((rows, K), np.int8)
    srow = np.zeros(rows, np.float32)
    lib().lalb_o_logic_pack(_p(W), _p(np.ascontiguousarray(state, np.uint8)), rows, K, _p(codes),
                          _p(srow))
    return codes, srow


def logic_forward(codes, srow, bias, X):
    rows, K = codes.shape
    X = np.ascontiguousarray(X, np.float32)
    M = X.shape[0]
    Y = np.zeros((M, rows), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().lalb_o_logic_forward(_p(np.ascontiguousarray(codes)), _p(srow), _p(b), rows, K, _p(X), M,
                             _p(Y))
    return Y
