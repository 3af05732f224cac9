"""Next-token sampling on the GPU (lalb_sample) against the oracle's
restatement of the reference's generate_text sampling."""
import numpy as np
import pytest
import torch

import _oracle as O
from test_gpu_kernels import dev, host

pytestmark = pytest.mark.gpu

VOCAB = 152064


def draw(u):
    return torch.tensor([u], dtype=torch.float32, device="cuda")


@pytest.mark.parametrize("params", [
    dict(temperature=0.0, top_k=1),
    dict(temperature=0.0, top_k=1, rep_penalty=1.5, no_repeat_ngram=3, n_masked_low_ids=3),
    dict(temperature=0.4, top_k=8, top_p=0.9, rep_penalty=1.5, no_repeat_ngram=3,
         n_masked_low_ids=3),                 # the reference trainer's defaults
    dict(temperature=1.0, top_k=64, top_p=0.95),
    dict(temperature=0.7, top_k=256, top_p=0.5, rep_penalty=1.3),
    dict(temperature=2.0, top_k=40, top_p=1.0, no_repeat_ngram=2),
])
def test_sample_matches_oracle(ctx, params):
    rng = np.random.default_rng(params["top_k"] + int(10 * params["temperature"]))
    logits = (rng.standard_normal(VOCAB) * 2).astype(np.float32)
    # make the history matter: its tokens among the largest logits
    top = np.argsort(-logits)[:50]
    history = np.concatenate([top[:20], rng.integers(0, VOCAB, 150), top[:2], top[5:7],
                              top[:1]]).astype(np.int32)
    ld, hd = dev(logits), dev(history)
    for u in (0.0, 0.137, 0.5, 0.93):
        tok, ids, prob = ctx.sample(ld, hd, u=draw(u), want_topk=True, **params)
        ref_tok, ref_ids, ref_prob = O.sample(logits, history, u=u, **params)
        assert np.array_equal(host(ids), ref_ids)
        assert np.array_equal(host(prob), ref_prob)
        assert int(host(tok)[0]) == ref_tok


def test_sample_edge_cases(ctx):
    # ties go to the lower id; a vocabulary smaller than top_k
    lg = np.array([5, 9, 5, 9, 1], np.float32)
    tok, ids, _ = ctx.sample(dev(lg), None, temperature=1.0, top_k=64, u=draw(0.0), want_topk=True)
    assert list(host(ids)) == [1, 3, 0, 2, 4] and int(host(tok)[0]) == 1
    # every id banned or masked but one
    lg = np.zeros(1000, np.float32)
    lg[999] = -5.0
    tok = ctx.sample(dev(lg), dev(np.array([7, 8, 9, 7, 8], np.int32)), temperature=0.0,
                     top_k=1, no_repeat_ngram=3, n_masked_low_ids=999)
    assert int(host(tok)[0]) == 999
    # greedy needs no draw
    tok = ctx.sample(dev(np.arange(300000, dtype=np.float32)), None)
    assert int(host(tok)[0]) == 299999
