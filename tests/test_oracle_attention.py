"""The oracle's decoder cross-attention (cpp/src/network_graph.cpp:235-244 `attend`
over the cross-K/V cache of :401-404) against an independent float64 restatement
with torch: half(q*c), half(k*c), fp16 scores, softmax rounded to fp16, fp16 output."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import halves


def _reference(q, k, v, queries):
    import torch

    streams, heads, keys, dim = k.shape
    c = np.float16(dim ** -0.25)
    qs = (q.astype(np.float32) * np.float32(c)).astype(np.float16).astype(np.float64)
    qs = qs.reshape(streams, queries, heads, dim).transpose(0, 2, 1, 3)
    ks = (k.astype(np.float32) * np.float32(c)).astype(np.float16).astype(np.float64)
    scores = np.einsum("shtd,shjd->shtj", qs, ks).astype(np.float16).astype(np.float64)
    p = torch.softmax(torch.from_numpy(scores), -1).numpy().astype(np.float16).astype(np.float64)
    out = np.einsum("shtj,shjd->shtd", p, v.astype(np.float64)).astype(np.float16)
    return out.transpose(0, 2, 1, 3).reshape(streams * queries, heads * dim)


@pytest.mark.parametrize("streams,queries,heads,keys", [(1, 1, 2, 7), (2, 5, 3, 130), (1, 16, 1, 257)])
def test_cross_attention_matches_float64_restatement(oracle, streams, queries, heads, keys):
    rng = np.random.default_rng(streams * 100 + keys)
    q = halves(rng, (streams * queries, heads * 64))
    k = halves(rng, (streams, heads, keys, 64))
    v = halves(rng, (streams, heads, keys, 64))
    out, codes = oracle.cross_attention(q, k, v, queries, code_scale=0.004)
    np.testing.assert_array_equal(out, _reference(q, k, v, queries).view(np.uint16))
    np.testing.assert_array_equal(codes, oracle.quantize(out, np.float32(0.004)))


def test_uniform_scores_average_the_values(oracle):
    """Identical keys give equal probabilities: the output is the mean of v (here
    all v rows equal, so out = v exactly)."""
    q = np.ones((1, 64), np.float16)
    k = np.ones((1, 1, 10, 64), np.float16)
    v = np.tile(np.linspace(-2, 2, 64, dtype=np.float16), (1, 1, 10, 1))
    out, _ = oracle.cross_attention(q, k, v, 1)
    # p = half(1/10) each; sum of 10 * half(0.1) * v differs from v by the rounding of 0.1
    expected = (np.float64(np.float16(0.1)) * 10 * v[0, 0, 0].astype(np.float64)).astype(np.float16)
    np.testing.assert_array_equal(out[0], expected.view(np.uint16))


@pytest.mark.parametrize("streams,tokens,heads", [(1, 1, 1), (2, 70, 3), (1, 129, 2)])
def test_self_attention_matches_float64_restatement(oracle, streams, tokens, heads):
    """Encoder self-attention (network_graph.cpp:235-247) on a fused QKV output."""
    import torch

    rng = np.random.default_rng(streams * 10 + tokens)
    width = heads * 64
    qkv = halves(rng, (streams * tokens, 3 * width))
    out, codes = oracle.self_attention(qkv, streams, heads, code_scale=0.004)
    q, k, v = qkv[:, :width], qkv[:, width:2 * width], qkv[:, 2 * width:]
    c = np.float16(64 ** -0.25)
    split = lambda a: a.reshape(streams, tokens, heads, 64).transpose(0, 2, 1, 3)
    qs = split((q.astype(np.float32) * np.float32(c)).astype(np.float16).astype(np.float64))
    ks = split((k.astype(np.float32) * np.float32(c)).astype(np.float16).astype(np.float64))
    scores = np.einsum("shid,shjd->shij", qs, ks).astype(np.float16).astype(np.float64)
    p = torch.softmax(torch.from_numpy(scores), -1).numpy().astype(np.float16).astype(np.float64)
    want = np.einsum("shij,shjd->shid", p, split(v.astype(np.float64))).astype(np.float16)
    want = want.transpose(0, 2, 1, 3).reshape(streams * tokens, width)
    np.testing.assert_array_equal(out, want.view(np.uint16))
    np.testing.assert_array_equal(codes, oracle.quantize(out, np.float32(0.004)))


def test_score_flip_slack_bounds_one_ulp_score_changes():
    """The self-attention GPU test allows, beyond the fixed bound, the first-order
    effect of scores that land one fp16 ulp away (_score_flip_slack).  Check that
    slack on the CPU: move every score of a small case by -1, 0 or +1 fp16 ulp at
    random, redo the softmax and P.V exactly, and the output moves by no more than
    the slack says."""
    from test_gpu_attention import _score_flip_slack

    streams, tokens, heads, d = 2, 96, 2, 64
    rng = np.random.default_rng(11)
    qkv = halves(rng, (streams * tokens, 3 * heads * d), std=2.0)
    c = float(np.float16(d ** -0.25))
    x = qkv.astype(np.float64)
    exact = np.zeros((streams * tokens, heads * d))
    moved = np.zeros_like(exact)
    for st in range(streams):
        blk = slice(st * tokens, (st + 1) * tokens)
        for h in range(heads):
            q = (x[blk, h * d:(h + 1) * d] * c).astype(np.float16).astype(np.float64)
            k = (x[blk, (heads + h) * d:(heads + h + 1) * d] * c).astype(np.float16).astype(np.float64)
            v = x[blk, (2 * heads + h) * d:(2 * heads + h + 1) * d]
            s16 = (q @ k.T).astype(np.float16)
            step = rng.integers(-1, 2, size=s16.shape)
            step[s16 == 0] = 0  # +-0 would step to a NaN bit pattern
            bits = s16.view(np.int16).astype(np.int32)
            # one ulp up or down in magnitude: +-1 on the bit pattern of a nonzero finite fp16
            s_moved = np.where(step == 0, s16, (bits + step).astype(np.int16).view(np.float16))
            for s, dst in ((s16.astype(np.float64), exact), (s_moved.astype(np.float64), moved)):
                p = np.exp(s - s.max(axis=1, keepdims=True))
                p /= p.sum(axis=1, keepdims=True)
                dst[blk, h * d:(h + 1) * d] = p @ v
    slack = _score_flip_slack(qkv, streams, heads, exact)
    change = np.abs(moved - exact)
    assert change.max() > 0
    # first order in ulp(s) <= 2^-8 for these scores; allow 10% for the second order
    assert np.all(change <= 1.1 * slack + 1e-12), float((change / (slack + 1e-30)).max())


def _one_pass_model(s16, v, tile=128, lazy=8.0):
    """The self-attention kernel's one-pass softmax in exact arithmetic: per tile of
    `tile` keys the running maximum m is raised (first tile, or when the tile's
    maximum exceeds it by more than 2^lazy in exp) and what was summed is rescaled;
    P = half(exp(s - m)) feeds P.V, the row sum takes the unrounded exponentials,
    and out = half(O / sum)."""
    s = s16.astype(np.float64)
    rows, keys = s.shape
    out = np.zeros((rows, v.shape[1]))
    for r in range(rows):
        m, l, o = -np.inf, 0.0, np.zeros(v.shape[1])
        for c0 in range(0, keys, tile):
            blk = s[r, c0:c0 + tile]
            tm = blk.max()
            if m == -np.inf or (tm - m) * np.log2(np.e) > lazy:
                alpha = 0.0 if m == -np.inf else np.exp(m - tm)
                l, o, m = l * alpha, o * alpha, tm
            e = np.exp(blk - m)
            l += e.sum()
            o += e.astype(np.float16).astype(np.float64) @ v[c0:c0 + tile]
        out[r] = o / l
    return out.astype(np.float16).astype(np.float64)


@pytest.mark.parametrize("std,tokens", [(1.0, 300), (2.0, 300), (3.0, 260), (6.0, 200)])
def test_one_pass_softmax_within_slack(oracle, std, tokens):
    """The self-attention GPU test allows the one-pass softmax's probability rounding
    (2^-10 sum_j p_j |v_j| + 2^-25 sum_j |v_j|, _score_flip_slack(one_pass=True)) on
    top of the fixed bound.  Check that term on the CPU: the exact model of the
    kernel's arithmetic (_one_pass_model) stays within the fixed bound plus that term
    of the oracle's exact two-pass output, on score scales from mild to peaked (std 6
    raises the running maximum mid-row, exercising the rescale)."""
    from test_gpu_attention import ATOL, RTOL, _score_flip_slack

    streams, heads, d = 1, 2, 64
    rng = np.random.default_rng(int(std * 100) + tokens)
    qkv = halves(rng, (streams * tokens, 3 * heads * d), std=std)
    want, _ = oracle.self_attention(qkv, streams, heads)
    ref = want.view(np.float16).astype(np.float64)
    c = float(np.float16(d ** -0.25))
    x = qkv.astype(np.float64)
    got = np.zeros_like(ref)
    for h in range(heads):
        q = (x[:, h * d:(h + 1) * d] * c).astype(np.float16).astype(np.float64)
        k = (x[:, (heads + h) * d:(heads + h + 1) * d] * c).astype(np.float16).astype(np.float64)
        v = x[:, (2 * heads + h) * d:(2 * heads + h + 1) * d]
        got[:, h * d:(h + 1) * d] = _one_pass_model((q @ k.T).astype(np.float16), v)
    full = _score_flip_slack(qkv, streams, heads, ref, one_pass=True)
    flips = _score_flip_slack(qkv, streams, heads, ref)
    err = np.abs(got - ref)
    assert err.max() > 0
    assert np.all(err <= ATOL + RTOL * np.abs(ref) + (full - flips))
