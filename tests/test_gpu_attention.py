"""Decoder cross-attention on the GPU (cpp/src/network_graph.cpp:235-244 `attend`
over the cross-K/V cache of :401-404) against the CPU oracle.

The oracle sums exactly and rounds each fp16 edge once; the GPU accumulates the
scores and P.V in fp32 (tensor-core MMAs) and evaluates the softmax in fp32, as
TensorRT's graph does.  A score can therefore land one fp16 ulp away, which moves
a probability by about one fp16 ulp.  The output, a convex combination of the v
rows, stays within the linear's bound 2^-11 + 2^-10 |ref| of the oracle for inputs
~N(0, 1): about one fp16 ulp of the output.  The E4M3 codes are bit-exact against Q
of the GPU's own fp16 output."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import halves

pytestmark = pytest.mark.gpu
ATOL = 2.0**-11
RTOL = 2.0**-10


def _within(got, want_bits):
    want = want_bits.view(np.float16).astype(np.float64)
    err = np.abs(got.astype(np.float64) - want)
    return err, bool(np.all(err <= ATOL + RTOL * np.abs(want)))


def _data(rng, streams, queries, heads, keys):
    q = halves(rng, (streams * queries, heads * 64))
    k = halves(rng, (streams, heads, keys, 64))
    v = halves(rng, (streams, heads, keys, 64))
    return q, k, v


@pytest.mark.parametrize("streams,queries,heads,keys", [
    # 1, 2, 4 and 8 CTAs per (stream, head) split the keys; ragged key counts and
    # every query count up to the MMA's 16 rows
    (1, 1, 1, 1), (1, 1, 20, 1500), (4, 5, 20, 1500), (2, 16, 3, 4096), (3, 2, 4, 130), (1, 7, 2, 129),
    (2, 3, 5, 257), (1, 9, 1, 128), (2, 5, 20, 700), (16, 1, 20, 1500),
])
def test_cross_attention_matches_oracle(cuda, fp8, oracle, native, streams, queries, heads, keys):
    import torch

    rng = np.random.default_rng(streams * 1000 + queries * 100 + keys)
    q, k, v = _data(rng, streams, queries, heads, keys)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out, codes = fp8.cross_attention(dev(q), dev(k), dev(v), queries, code_scale=0.004)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    want, _ = oracle.cross_attention(q, k, v, queries)
    got = out.cpu().numpy()
    err, ok = _within(got, want)
    print(f"s={streams} q={queries} h={heads} keys={keys}: max_abs={err.max():.3g} "
          f"exact={(got.view(np.uint16) == want).mean():.4f}")
    assert ok
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(got.view(np.uint16), np.float32(0.004)))


def test_cross_attention_outputs_and_scale_pointer(cuda, fp8):
    """Codes only, output only, and a device-resident code scale agree bit for bit."""
    import torch

    rng = np.random.default_rng(3)
    q, k, v = _data(rng, 2, 5, 4, 700)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out, codes = fp8.cross_attention(qd, kd, vd, 5, code_scale=0.01)
    _, codes_only = fp8.cross_attention(qd, kd, vd, 5, code_scale=0.01, want_out=False)
    out_only, none = fp8.cross_attention(qd, kd, vd, 5)
    scale = torch.tensor([0.01], dtype=torch.float32, device=cuda)
    _, dyn = fp8.cross_attention(qd, kd, vd, 5, code_scale=scale, want_out=False)
    torch.cuda.synchronize()
    assert none is None
    assert torch.equal(out, out_only)
    assert torch.equal(codes, codes_only) and torch.equal(codes, dyn)


def test_cross_attention_identical_keys_average_values(cuda, fp8, oracle):
    """All keys equal: every probability is half(1/keys); the output matches the
    oracle exactly (no score rounding can differ)."""
    import torch

    keys = 300
    q = np.ones((2, 64), np.float16)
    k = np.ones((1, 1, keys, 64), np.float16)
    v = halves(np.random.default_rng(4), (1, 1, keys, 64))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    out, _ = fp8.cross_attention(dev(q), dev(k), dev(v), 2)
    torch.cuda.synchronize()
    want, _ = oracle.cross_attention(q, k, v, 2)
    err = np.abs(out.cpu().numpy().astype(np.float64) - want.view(np.float16).astype(np.float64))
    assert err.max() <= 2.0**-11


@pytest.mark.parametrize("streams,tokens,heads", [
    # one and several 128-row query blocks and 128-key tiles, ragged tails (the
    # last tile's rows belong to the next stream), exact tile multiples, a key
    # count at or below one 32- or 64-column softmax part, the C2 head count
    (1, 1, 1), (1, 64, 2), (2, 130, 3), (1, 1500, 2), (3, 257, 4), (8, 100, 20),
    (2, 127, 2), (2, 128, 2), (3, 129, 1), (1, 256, 3), (2, 33, 2), (1, 2048, 1),
])
def test_self_attention_matches_oracle(cuda, fp8, oracle, native, streams, tokens, heads):
    """Encoder self-attention on the fused QKV output, same bound as above."""
    import torch

    rng = np.random.default_rng(streams * 1000 + tokens + heads)
    qkv = halves(rng, (streams * tokens, 3 * heads * 64))
    out, codes = fp8.self_attention(torch.from_numpy(qkv).to(cuda), streams, heads, code_scale=0.004)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    want, _ = oracle.self_attention(qkv, streams, heads)
    got = out.cpu().numpy()
    err, ok = _within(got, want)
    print(f"self s={streams} t={tokens} h={heads}: max_abs={err.max():.3g} "
          f"exact={(got.view(np.uint16) == want).mean():.4f}")
    assert ok
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(got.view(np.uint16), np.float32(0.004)))
