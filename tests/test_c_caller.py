"""The C ABI driven from plain C99, as the reference engine's C sources would
drive it: tests/c_caller/lalb_c_caller.c includes include/lalb.h, is built
with gcc -std=c99 -pedantic -Werror and linked against liblalb.so.

CPU: the program compiles, links, and its host-only calls work (a missing
sm_100 device is reported as LALB_ERR_DEVICE, not a crash).
GPU: one Q4_K matvec and one LM-head call through the C program, checked
against the oracle.
"""
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

import _oracle as O
from lalmodel_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_caller", "lalb_c_caller.c")
CUDA = "/usr/local/cuda"


def build_caller(outdir):
    exe = os.path.join(outdir, "lalb_c_caller")
    libdir = os.path.dirname(_abi.LIB_PATH)
    cmd = [shutil.which("gcc") or "gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror",
           "-O2", "-I", os.path.join(ROOT, "include"), "-isystem", os.path.join(CUDA, "include"), SRC,
           "-o", exe, _abi.LIB_PATH, "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           "-Wl,-rpath," + libdir + ":" + os.path.join(CUDA, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c99_caller_builds_and_runs_host_calls(tmp_path):
    _abi.lib()   # builds liblalb.so when missing
    exe = build_caller(str(tmp_path))
    r = subprocess.run([exe, "--abi-only"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "abi ok" in r.stdout


@pytest.mark.gpu
def test_c99_caller_matches_oracle_on_gpu(tmp_path):
    exe = build_caller(str(tmp_path))
    rows, K, hrows, hK = 1000, 3584, 7000, 3584
    W = O.q4k_quantize(O.normal(rows * K, seed=71, sigma=0.02).reshape(rows, K))
    x = O.normal(K, seed=72)
    Hq, Hs = O.q8_quantize_rows(O.normal(hrows * hK, seed=73, sigma=0.02).reshape(hrows, hK))
    xh = O.normal(hK, seed=74)
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        f.write(struct.pack("<4i", rows, K, hrows, hK))
        for a in (W, x, Hq, Hs, xh):
            f.write(np.ascontiguousarray(a).tobytes())
    out = tmp_path / "out.bin"
    r = subprocess.run([exe, str(inp), str(out)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    raw = np.fromfile(out, dtype=np.uint8)
    y = raw[: 4 * rows].view(np.float32)
    logits = raw[4 * rows: 4 * (rows + hrows)].view(np.float32)
    am = int(raw[4 * (rows + hrows):].view(np.int32)[0])
    xq, sx, sq = O.quantize_act(x)
    ref_y, _ = O.q4k_matmul(W, rows, K, xq, sx, sq)
    assert O.normwise_rel_err(y, ref_y[0]) < 1e-5
    hq, hs, _ = O.quantize_act(xh)
    ref_l, _, ref_am = O.q8_lmhead(Hq, Hs, hq, hs, 0, hrows)
    assert O.normwise_rel_err(logits, ref_l) < 1e-5
    assert am == ref_am
