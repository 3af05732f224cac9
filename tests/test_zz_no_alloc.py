"""The allocation-free LM head, checked against the regular entry point.

lalb_lm_head_int8_range_noalloc exists for callers that cannot call
cudaMalloc: an engine whose own memory pool owns the device, or code that
cannot create a lalb_ctx because creating one allocates.  It keeps its argmax
reduction state in a static device array shared by every call, so two calls
in a row must each start from a cleared state and give the same logits and
argmax as lalb_lm_head_int8_range.  This file sorts last so that a run that
stops at the first failure has run every other test before it.
"""
import ctypes

import numpy as np
import pytest
import torch

import _oracle as O
import lalmodel_b200 as lb
from lalmodel_b200 import _abi

pytestmark = pytest.mark.gpu
TOL = 1e-5


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def noalloc(W, sw, K, r0, r1, x, logits, argmax):
    """Calls the C entry point directly (no context, no allocation)."""
    return _abi.lib().lalb_lm_head_int8_range_noalloc(
        lb._p(W), lb._p(sw), K, r0, r1, lb._p(x), lb._p(logits), lb._p(argmax), lb._stream())


def test_noalloc_lm_head_matches_regular_entry_point_twice(ctx):
    rows, K = 40000, 3584
    q, s = O.q8_quantize_rows(O.normal(rows * K, seed=901, sigma=0.02).reshape(rows, K))
    qd, sd = dev(q), dev(s)
    # two different activations, one call each, back to back: the second
    # call must not see the first call's argmax state
    for seed, (r0, r1) in ((902, (0, rows)), (903, (123, rows - 77))):
        x = O.normal(K, seed=seed)
        xd = dev(x)
        ref_logits, ref_am = ctx.lm_head_int8_range(qd, sd, xd, r0, r1)
        logits = torch.empty(r1 - r0, dtype=torch.float32, device="cuda")
        am = torch.full((1,), -2, dtype=torch.int32, device="cuda")
        assert noalloc(qd, sd, K, r0, r1, xd, logits, am) == 0
        torch.cuda.synchronize()
        got, ref = logits.cpu().numpy(), ref_logits.cpu().numpy()
        assert O.normwise_rel_err(got, ref) < TOL
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert int(am.item()) == int(ref_am.item())
        xq, sx, _ = O.quantize_act(x)
        _, _, oracle_am = O.q8_lmhead(q, s, xq, sx, r0, r1)
        assert int(am.item()) == oracle_am


def test_noalloc_and_regular_calls_mix_in_any_order(ctx):
    """Allocation-free call at a large K, then a regular call at a small K,
    then the allocation-free call again: the regular call must not shrink the
    kernel's shared-memory limit under the next allocation-free launch.  (In
    a fresh process the regular call below is the kernel's first regular
    launch, the order in which that could happen.)"""
    rows, K, Ks = 5000, 3584, 512
    q, s = O.q8_quantize_rows(O.normal(rows * K, seed=911, sigma=0.02).reshape(rows, K))
    qs, ss = O.q8_quantize_rows(O.normal(rows * Ks, seed=912, sigma=0.02).reshape(rows, Ks))
    qd, sd, qsd, ssd = dev(q), dev(s), dev(qs), dev(ss)
    x, xs = O.normal(K, seed=913), O.normal(Ks, seed=914)
    xd, xsd = dev(x), dev(xs)
    xq, sx, _ = O.quantize_act(x)
    oracle_logits, _, oracle_am = O.q8_lmhead(q, s, xq, sx, 0, rows)
    xqs, sxs, _ = O.quantize_act(xs)
    _, _, oracle_small = O.q8_lmhead(qs, ss, xqs, sxs, 0, rows)
    got = []
    for _ in range(2):
        logits = torch.empty(rows, dtype=torch.float32, device="cuda")
        am = torch.full((1,), -2, dtype=torch.int32, device="cuda")
        assert noalloc(qd, sd, K, 0, rows, xd, logits, am) == 0
        torch.cuda.synchronize()
        assert O.normwise_rel_err(logits.cpu().numpy(), oracle_logits) < TOL
        assert int(am.item()) == oracle_am
        got.append(logits.cpu().numpy())
        # the regular entry point at a small K in between
        _, small_am = ctx.lm_head_int8_range(qsd, ssd, xsd, 0, rows)
        torch.cuda.synchronize()
        assert int(small_am.item()) == oracle_small
    ref_logits, ref_am = ctx.lm_head_int8_range(qd, sd, xd, 0, rows)
    torch.cuda.synchronize()
    for g in got:
        assert np.array_equal(g.view(np.uint32), ref_logits.cpu().numpy().view(np.uint32))
    assert int(ref_am.item()) == oracle_am


def test_noalloc_lm_head_rejects_what_the_kernel_cannot_do(ctx):
    q = torch.zeros((4, 4128), dtype=torch.int8, device="cuda")
    s = torch.ones(4, dtype=torch.float32, device="cuda")
    x = torch.ones(4128, dtype=torch.float32, device="cuda")
    out = torch.empty(4, dtype=torch.float32, device="cuda")
    am = torch.empty(1, dtype=torch.int32, device="cuda")
    assert noalloc(q, s, 4128, 0, 4, x, out, am) == -4      # K > 4096: unsupported
    assert noalloc(q, s, 48, 0, 4, x, out, am) == -1        # K not a multiple of 32
    assert noalloc(q, s, 64, 3, 2, x, out, am) == -1        # inverted row range
