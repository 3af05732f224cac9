"""ctypes binding of include/lalb.h (liblalb.so, built in-tree).

Every C entry point is declared here with its exact argument types; `call`
raises LalbError on a nonzero status with the context's last error text.
There is no fallback: if the shared library is missing, lib() raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblalb.so")

c_int, c_float, c_size_t, c_uint64 = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_uint64
P = ctypes.c_void_p

STATUS = {0: "LALB_OK", -1: "LALB_ERR_INVALID", -2: "LALB_ERR_CUDA", -3: "LALB_ERR_NOMEM",
          -4: "LALB_ERR_UNSUPPORTED", -5: "LALB_ERR_TIMEOUT", -6: "LALB_ERR_COMM",
          -7: "LALB_ERR_DEVICE"}


class DecoderCfg(ctypes.Structure):
    _fields_ = [("n_layer", c_int), ("hidden", c_int), ("q_rows", c_int),
                ("kv_rows", c_int), ("ffn", c_int), ("vocab", c_int), ("rms_eps", c_float),
                ("head_dim", c_int), ("max_ctx", c_int), ("rope_theta", c_float)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("wqkv", P), ("wo", P), ("wgu", P), ("wdown", P), ("attn_norm", P),
                ("ffn_norm", P)]


class BlobTensor(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char * 72), ("dtype", c_int), ("ndim", c_int),
                ("dims", c_uint64 * 3), ("bytes", c_uint64), ("row_bytes", c_uint64)]


class Sampling(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_k", c_int), ("top_p", c_float),
                ("rep_penalty", c_float), ("no_repeat_ngram", c_int), ("n_masked_low_ids", c_int)]


# name -> (restype, argtypes); mirrors include/lalb.h one to one
SIGNATURES = {
    "lalb_abi_version": (c_int, []),
    "lalb_status_string": (ctypes.c_char_p, [c_int]),
    "lalb_init": (c_int, [c_int, ctypes.POINTER(P)]),
    "lalb_destroy": (c_int, [P]),
    "lalb_last_error": (ctypes.c_char_p, [P]),
    "lalb_device_status": (c_int, [P, c_int]),
    "lalb_unpack_scales_6bit": (c_int, [P, P]),
    "lalb_fill_normal": (c_int, [P, P, c_size_t, c_uint64, c_uint64, c_float, P]),
    "lalb_q4k_quantize": (c_int, [P, P, c_int, c_int, P, P]),
    "lalb_q8_quantize_rows": (c_int, [P, P, c_int, c_int, P, P, P]),
    "lalb_quantize_act": (c_int, [P, P, c_int, c_int, P, P, P, P]),
    "lalb_matmul_q4_k": (c_int, [P, P, c_int, c_int, P, P, P]),
    "lalb_matmul_q4_k_q8": (c_int, [P, P, c_int, c_int, P, P, P, P, P, P]),
    "lalb_lm_head_int8_range": (c_int, [P, P, P, c_int, c_int, c_int, P, P, P, P]),
    "lalb_lm_head_int8_q8": (c_int, [P, P, P, c_int, c_int, c_int, P, P, P, P, P, P]),
    "lalb_lm_head_int8_range_noalloc": (c_int, [P, P, c_int, c_int, c_int, P, P, P, P]),
    "lalb_decoder_create": (c_int, [P, ctypes.POINTER(DecoderCfg), ctypes.POINTER(P)]),
    "lalb_decoder_set_layer": (c_int, [P, c_int, ctypes.POINTER(LayerWeights)]),
    "lalb_decoder_set_lm_head": (c_int, [P, P, P]),
    "lalb_decoder_set_output_norm": (c_int, [P, P]),
    "lalb_decoder_set_kv_cache": (c_int, [P, c_int, P, P]),
    "lalb_decoder_set_position": (c_int, [P, c_int, P]),
    "lalb_decoder_position": (c_int, [P]),
    "lalb_attention_decode": (c_int, [P, P, c_int, c_int, c_int, c_int, c_int, c_float, P, P, P, P]),
    "lalb_sample_ws_bytes": (c_int, [c_int, c_int, ctypes.POINTER(c_size_t)]),
    "lalb_blob_writer_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(P)]),
    "lalb_blob_writer_add": (c_int, [P, ctypes.c_char_p, c_int, c_int, ctypes.POINTER(c_uint64), P]),
    "lalb_blob_writer_add_quantized": (c_int, [P, P, ctypes.c_char_p, ctypes.c_char_p, c_int, c_int,
                                               P, c_int, c_int]),
    "lalb_blob_writer_close": (c_int, [P]),
    "lalb_blob_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(P)]),
    "lalb_blob_close": (c_int, [P]),
    "lalb_blob_count": (c_int, [P]),
    "lalb_blob_find": (c_int, [P, ctypes.c_char_p]),
    "lalb_blob_info": (c_int, [P, c_int, ctypes.POINTER(BlobTensor)]),
    "lalb_blob_verify": (c_int, [P, c_int]),
    "lalb_blob_read_host": (c_int, [P, c_int, c_uint64, c_uint64, P]),
    "lalb_blob_load": (c_int, [P, P, c_int, c_uint64, c_uint64, P, P]),
    "lalb_sample": (c_int, [P, P, c_int, P, c_int, ctypes.POINTER(Sampling), P, P, P, P, P, P]),
    "lalb_decoder_step": (c_int, [P, P, P, P, P, P]),
    "lalb_decoder_step_host": (c_int, [P, P, P, P]),
    "lalb_decoder_profile_step": (c_int, [P, P, P, P]),
    "lalb_decoder_trace_step": (c_int, [P, P, P, c_int, P, P]),
    "lalb_tp_rows": (c_int, [ctypes.POINTER(DecoderCfg), c_int, c_int, c_int, P, P]),
    "lalb_decoder_create_tp": (c_int, [P, ctypes.POINTER(DecoderCfg), c_int, c_int, ctypes.POINTER(P)]),
    "lalb_decoder_set_layer_shard": (c_int, [P, c_int, c_int, ctypes.POINTER(LayerWeights)]),
    "lalb_decoder_set_lm_head_shard": (c_int, [P, c_int, P, P]),
    "lalb_decoder_ipc_handle": (c_int, [P, P]),
    "lalb_decoder_connect": (c_int, [P, P]),
    "lalb_decoder_exchange_buffer": (c_int, [P, ctypes.POINTER(P)]),
    "lalb_decoder_connect_local": (c_int, [P, P]),
    "lalb_decoder_set_wait_limit": (c_int, [P, ctypes.c_double]),
    "lalb_decoder_reset": (c_int, [P, P]),
    "lalb_decoder_set_path": (c_int, [P, c_int]),
    "lalb_prefill_ws_bytes": (c_int, [c_int, c_int, c_int, ctypes.POINTER(ctypes.c_size_t)]),
    "lalb_measure_mma_peak": (c_int, [P, c_int, ctypes.POINTER(ctypes.c_double)]),
    "lalb_matmul_q4_k_prefill": (c_int, [P, P, c_int, c_int, P, c_int, P, P, P]),
    "lalb_binlayer_create": (c_int, [P, P, P, P, c_int, c_int, c_int, ctypes.c_float, c_int,
                                     ctypes.POINTER(P)]),
    "lalb_binlayer_forward": (c_int, [P, P, c_int, P, c_int, P]),
    "lalb_binlayer_alpha": (c_int, [P, P, P]),
    "lalb_binlayer_destroy": (c_int, [P]),
    "lalb_logic_pack": (c_int, [P, P, P, c_int, c_int, P, P, P]),
    "lalb_logic_layer_create": (c_int, [P, P, P, P, c_int, c_int, c_int, ctypes.POINTER(P)]),
    "lalb_logic_layer_forward": (c_int, [P, P, c_int, P, P]),
    "lalb_logic_layer_destroy": (c_int, [P]),
    "lalb_decoder_path": (c_int, [P]),
    "lalb_decoder_launches_per_step": (c_int, [P]),
    "lalb_decoder_destroy": (c_int, [P]),
}

_lib = None


class LalbError(RuntimeError):
    def __init__(self, fn, status, detail=""):
        self.status = status
        super().__init__(f"{fn} -> {STATUS.get(status, status)}: {detail}")


def lib():
    """Load liblalb.so and declare every entry point (raises if absent)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run `python -m lalmodel_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def call(ctx, name, *args):
    """Call `name`; raise LalbError (with lalb_last_error text) on failure."""
    st = getattr(lib(), name)(*args)
    if st != 0:
        detail = lib().lalb_last_error(ctx).decode() if ctx else ""
        raise LalbError(name, st, detail)
    return st
