"""Generate the golden fixtures under tests/golden/ (run once, output committed).

Sources of truth, in this container only (neither travels to the GPU box):
  * gguf 0.19.0 (llama.cpp's own Python package, gguf/quants.py):
      - Q4_K.dequantize_blocks pins the 144-byte Q4_K super-block layout,
        the 6-bit scale/min packing and w = d*sc*q - dmin*m;
      - Q8_0.quantize_blocks pins the per-32-block int8 activation rounding
        (amax/127, round half away from zero).
  * the reference's own seed-model BinLayer code, runtime/lal_runtime.c
    (bin_layer_init_logic :1567, bin_layer_repack :1703, bin_forward :1852,
    bin_forward_pure_float :543), compiled from its source tree by
    `make -C oracle ref` into oracle/_ref/liblal_ref.so.
  * numpy's float32 -> float16 cast (IEEE round-to-nearest-even).
  * the reference's decode-step pieces from the same library: rms_norm,
    apply_rope and attention_forward (decode_ref.npz).

    python tests/golden/gen_golden.py [formats] [binlayer] [decode]

Inputs are seeded; nothing here reads a dataset.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
P = ctypes.c_void_p


def ptr(a):
    return a.ctypes.data_as(P)


def q4k_fixture(rng):
    from gguf.quants import Q4_K

    # (a) arbitrary bytes: every bit pattern of the scale bytes is legal
    raw = rng.integers(0, 256, size=(96, 144), dtype=np.uint8)
    # keep d/dmin finite and moderate: fp16 exponent field < 31
    d = rng.uniform(1e-4, 5e-3, size=96).astype(np.float16)
    m = rng.uniform(0.0, 5e-3, size=96).astype(np.float16)
    raw[:, 0:2] = d.view(np.uint8).reshape(96, 2)
    raw[:, 2:4] = m.view(np.uint8).reshape(96, 2)
    # edge rows: all-zero scales, all-max scales, zero d
    raw[0, 4:16] = 0
    raw[1, 4:16] = 0xFF
    raw[2, 0:2] = 0
    raw[3, 16:] = 0xFF
    deq = Q4_K.dequantize_blocks(raw.copy()).astype(np.float32)
    sc, mn = Q4_K.get_scale_min(raw[:, 4:16].copy())
    return dict(q4k_raw=raw, q4k_raw_deq=deq,
                q4k_raw_sc=sc.astype(np.uint8), q4k_raw_min=mn.astype(np.uint8))


def q8_fixture(rng):
    from gguf.quants import Q8_0

    x = rng.standard_normal((64, 32)).astype(np.float32)
    x[0] = 0.0                                     # all-zero block
    x[1] = 0.0
    x[1, 7] = -3.5                                 # single value
    x[2] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[3] = (np.arange(32, dtype=np.float32) - 15.5) * (127.0 / 15.5) / 127.0
    x[4] = np.float32(1e-30) * rng.standard_normal(32).astype(np.float32)
    blocks = Q8_0.quantize_blocks(x.copy())
    q = blocks[:, 2:].copy().view(np.int8)
    d = (np.abs(x).max(axis=1) / 127).astype(np.float32)
    return dict(q8_x=x, q8_q=q, q8_d=d)


def fp16_fixture(rng):
    f = np.concatenate([
        rng.standard_normal(2000).astype(np.float32) * np.float32(1e-3),
        (rng.standard_normal(2000) * 1e-6).astype(np.float32),  # subnormals
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, 2.0 ** -24,
                  2.0 ** -25, 3.0 * 2.0 ** -26, 6.1035156e-05], np.float32),
    ])
    with np.errstate(over="ignore"):
        h = f.astype(np.float16).view(np.uint16)
    return dict(f16_in=f, f16_out=h)


def binlayer_fixture(rng):
    so = os.path.join(ROOT, "oracle", "_ref", "liblal_ref.so")
    if not os.path.exists(so):
        sys.exit("build the reference harness first: make -C oracle ref")
    L = ctypes.CDLL(so)
    L.lalref_binlayer_forward.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int,
                                          P, ctypes.c_int, P, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_float, P]
    out = {}
    cases = [(448, 64, 4), (1792, 16, 2), (100, 24, 2)]   # (in, out, M)
    for ci, (K, N, M) in enumerate(cases):
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)  # [out, in]
        b = (rng.standard_normal(N) * 0.01).astype(np.float32)
        mask = rng.choice(np.array([0, 1, 2], np.uint8), size=N, p=[0.15, 0.6, 0.25])
        mask[0], mask[1], mask[2] = 0, 1, 2
        X = rng.standard_normal((M, K)).astype(np.float32)
        for mode in (0, 1):
            for repack in (0, 1):
                Y = np.zeros((M, N), np.float32)
                alpha = np.zeros(N, np.float32)
                L.lalref_binlayer_forward(ptr(W), ptr(b), ptr(mask), K, N, ptr(X),
                                          M, ptr(Y), mode, repack,
                                          ctypes.c_float(0.25), ptr(alpha))
                out[f"bl{ci}_m{mode}_r{repack}_Y"] = Y
                out[f"bl{ci}_m{mode}_r{repack}_alpha"] = alpha
        out[f"bl{ci}_W"], out[f"bl{ci}_b"] = W, b
        out[f"bl{ci}_mask"], out[f"bl{ci}_X"] = mask, X
    return out


def _ref_lib():
    so = os.path.join(ROOT, "oracle", "_ref", "liblal_ref.so")
    if not os.path.exists(so):
        sys.exit("build the reference harness first: make -C oracle ref")
    return ctypes.CDLL(so)


def decode_ref_fixture(rng):
    """The reference's own decode-step pieces from runtime/lal_runtime.c:
    rms_norm (:82-87), apply_rope (:137-153) and attention_forward
    (:833-882), called as the layer forward calls them (:310-311, :320-327):
    RoPE on q and k at position seq_pos, then the causal attention, which
    stores k and v at seq_pos in the layer's caches and attends 0..seq_pos."""
    L = _ref_lib()
    ci, f = ctypes.c_int, ctypes.c_float
    L.rms_norm.argtypes = [P, P, P, ci]
    L.apply_rope.argtypes = [P, P, ci, ci, ci, ci]
    L.attention_forward.argtypes = [P, P, ci, ci, ci, P, P]
    out = {}
    for i, (n, scale) in enumerate([(3584, 1.0), (512, 30.0), (96, 1e-3), (3584, 1e3)]):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        y = np.zeros(n, np.float32)
        L.rms_norm(ptr(y), ptr(x), ptr(w), n)
        out[f"rms{i}_x"], out[f"rms{i}_w"], out[f"rms{i}_y"] = x, w, y
    cases = [(256, 2, 0), (256, 2, 5), (512, 4, 37), (64, 4, 11), (256, 2, 130)]
    for i, (n_embd, n_head, pos) in enumerate(cases):
        hd = n_embd // n_head
        qkv = rng.standard_normal(3 * n_embd).astype(np.float32)
        kc = np.zeros((pos + 1, n_embd), np.float32)
        vc = np.zeros((pos + 1, n_embd), np.float32)
        kc[:pos] = rng.standard_normal((pos, n_embd)).astype(np.float32)
        vc[:pos] = rng.standard_normal((pos, n_embd)).astype(np.float32)
        out[f"att{i}_qkv"], out[f"att{i}_k_in"], out[f"att{i}_v_in"] = qkv.copy(), kc.copy(), vc.copy()
        out[f"att{i}_shape"] = np.array([n_embd, n_head, pos], np.int32)
        q = qkv.copy()
        L.apply_rope(ptr(q[:n_embd]), ptr(q[n_embd:2 * n_embd]), pos, n_head, hd, n_embd)
        out[f"att{i}_qkv_rope"] = q.copy()
        o = np.zeros(n_embd, np.float32)
        L.attention_forward(ptr(o), ptr(q), n_embd, n_head, pos, ptr(kc), ptr(vc))
        # the caches change only at row pos
        assert np.array_equal(kc[:pos], out[f"att{i}_k_in"][:pos])
        out[f"att{i}_out"], out[f"att{i}_k_row"], out[f"att{i}_v_row"] = o, kc[pos], vc[pos]
    return out


def main(which=("formats", "binlayer", "decode")):
    if "formats" in which or "binlayer" in which:
        rng = np.random.default_rng(20261201)
        fx = {}
        fx.update(q4k_fixture(rng))
        fx.update(q8_fixture(rng))
        fx.update(fp16_fixture(rng))
        if "formats" in which:
            np.savez_compressed(os.path.join(HERE, "formats_gguf.npz"), **fx)
        bl = binlayer_fixture(rng)
        if "binlayer" in which:
            np.savez_compressed(os.path.join(HERE, "binlayer_ref.npz"), **bl)
    if "decode" in which:
        np.savez_compressed(os.path.join(HERE, "decode_ref.npz"),
                            **decode_ref_fixture(np.random.default_rng(20261202)))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    # no argument: every fixture; else a subset, e.g. `decode`
    main(tuple(sys.argv[1:]) or ("formats", "binlayer", "decode"))
