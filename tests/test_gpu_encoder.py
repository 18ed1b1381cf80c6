"""The encoder front end (log-mel frames, the two convolutions with GELU and the
positional add), the head-split cross-K/V linear, and the composed encoder
forward (encoder.py) against the oracle.

The composed forward is checked stage by stage: every launch of the plan runs
alone, and its output is compared with the oracle applied to the GPU's own
inputs of that stage (so each stage is held to its own bound and every hand-off
-- scales, residual wiring, in-place q/k/v windows, padded conv rows, the
head-split layout -- is exercised).  A whole forward is then compared end to end
with the oracle's own composition, where rounding differences compound."""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PACKAGE
from helpers import ATOL, RTOL, compare_halves, halves
from test_gpu_attention import _score_flip_slack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def enc(lffw):
    return importlib.import_module(PACKAGE + ".encoder")


def _f16(bits):
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float64)


def conv_bound(frames_bits, weight, act_bits, out_bits, positions):
    """ATOL + RTOL |out| (+ 2 RTOL |GELU| before a positional add) + 1.13 K 2^-24 sum|x w|:
    the linear's fp16 bound carried through the fp16-edge GELU, plus the fp32
    summation bound of the K = 3 c_in products."""
    x = np.abs(_f16(frames_bits))
    w = np.abs(weight.astype(np.float64))
    streams, rows, c_in = x.shape
    stride = (rows - 2) // out_bits.shape[1]
    frames_out = out_bits.shape[1]
    mag = np.zeros(out_bits.shape, np.float64)
    for j in range(3):
        mag += x[:, j: j + stride * (frames_out - 1) + 1: stride, :] @ w[:, :, j].T
    bound = ATOL + RTOL * np.abs(_f16(out_bits)) + 1.13 * 3 * c_in * 2.0**-24 * mag
    if positions:
        bound += 2 * RTOL * np.abs(_f16(act_bits))
    else:
        bound += RTOL * np.abs(_f16(act_bits))
    return bound


def test_mel_frames_bit_exact(cuda, fp8, oracle):
    import torch

    rng = np.random.default_rng(1)
    for streams, mels, frames in ((1, 128, 3000), (3, 80, 203), (2, 8, 1)):
        mel = (rng.standard_normal((streams, mels, frames)) * 3).astype(np.float32)
        mel.ravel()[:5] = [0.0, -0.0, 70000.0, 1e-8, -65520.0]  # zero, overflow to inf, subnormal, tie
        got = fp8.mel_frames(torch.from_numpy(mel).to(cuda))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), oracle.mel_frames(mel))


def test_conv_weight_layout(cuda, fp8):
    import torch

    w = torch.randn(96, 64, 3, device=cuda).half()
    got = fp8.conv1d_weight_layout(w)
    assert torch.equal(got, w.permute(0, 2, 1).contiguous())


@pytest.mark.parametrize("streams,frames_in,c_in,c_out,stride,pos", [
    (2, 300, 128, 256, 1, False),     # conv1-like, ragged 128-row tiles
    (1, 3000, 128, 1280, 1, False),   # conv1 at full size
    (2, 256, 1280, 256, 2, True),     # conv2-like on CTA pairs (K = 3840), positional add
    (3, 100, 1280, 1280, 2, True),    # single-CTA tiles, 50 rows per stream
    (1, 3000, 1280, 1280, 2, True),   # conv2 at full size
    (2, 64, 64, 32, 2, False),        # smallest shapes: one K block per tap, one store box wide
])
def test_conv1d_gelu_matches_oracle(cuda, fp8, oracle, native, streams, frames_in, c_in, c_out, stride, pos):
    import torch

    rng = np.random.default_rng(frames_in + c_in + stride)
    frames_out = frames_in // stride
    x = np.zeros((streams, frames_in + 2, c_in), np.float16)
    x[:, 1:-1] = halves(rng, (streams, frames_in, c_in), 1.0)
    w = halves(rng, (c_out, c_in, 3), 0.02)
    b = halves(rng, (c_out,), 0.02)
    positions = halves(rng, (frames_out, c_out), 0.5) if pos else None
    wd = fp8.conv1d_weight_layout(torch.from_numpy(w).to(cuda))
    y = fp8.conv1d_gelu(torch.from_numpy(x).to(cuda), wd, torch.from_numpy(b).to(cuda), stride,
                        positions=None if positions is None else torch.from_numpy(positions).to(cuda))
    torch.cuda.synchronize()
    assert native.device_error() == 0
    pre, act, out = oracle.conv1d_gelu(x, w, b, stride, positions)
    got = y.cpu().numpy().view(np.uint16)
    bound = conv_bound(x.view(np.uint16), w, act, out, pos)
    err = np.abs(_f16(got) - _f16(out))
    excess = float((err - bound).max())
    mism = int((got != out).sum())
    print(f"conv {streams}x{frames_in}x{c_in}->{c_out}/s{stride}: max_abs={err.max():.3g} mismatch={mism}/{got.size}")
    assert excess <= 0
    assert mism <= max(got.size // 200, 8)


def test_conv1d_padded_output_rows(cuda, fp8, oracle):
    """y_rows = frames_out + 2, y_row0 = 1: the padding rows are left as they were."""
    import torch

    rng = np.random.default_rng(7)
    streams, frames, c_in, c_out = 2, 200, 128, 256
    x = np.zeros((streams, frames + 2, c_in), np.float16)
    x[:, 1:-1] = halves(rng, (streams, frames, c_in))
    w = halves(rng, (c_out, c_in, 3), 0.02)
    b = halves(rng, (c_out,), 0.02)
    out = torch.full((streams, frames + 2, c_out), 0x1234, dtype=torch.int16, device=cuda).view(torch.float16)
    fp8.conv1d_gelu(torch.from_numpy(x).to(cuda), fp8.conv1d_weight_layout(torch.from_numpy(w).to(cuda)),
                    torch.from_numpy(b).to(cuda), 1, out=out, out_row0=1)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    assert (got[:, 0] == 0x1234).all() and (got[:, -1] == 0x1234).all()
    dense = fp8.conv1d_gelu(torch.from_numpy(x).to(cuda), fp8.conv1d_weight_layout(torch.from_numpy(w).to(cuda)),
                            torch.from_numpy(b).to(cuda), 1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got[:, 1:-1], dense.cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("streams,tokens,groups", [(2, 1500, 4), (3, 100, 2), (1, 129, 2), (5, 7, 2)])
def test_linear_heads_equals_flat_linear(cuda, fp8, oracle, native, streams, tokens, groups):
    """Same arithmetic as lffw_fp8_linear, stored [group][stream][head][token][64]; the
    key rows' -0 bias leaves their values (and -0) as a bias-free linear gives them."""
    import torch

    heads, d = 20, 1280
    n = groups * heads * 64
    rng = np.random.default_rng(tokens + groups)
    x = torch.from_numpy(halves(rng, (streams * tokens, d))).to(cuda)
    w = torch.from_numpy(halves(rng, (n, d), 0.02)).to(cuda)
    bias = torch.from_numpy(halves(rng, (n,), 0.02)).to(cuda)
    bias.view(torch.int16).view(groups, heads * 64)[0::2] = -32768  # -0.0 on the "key" groups
    q = fp8.QuantizedWeight.from_half(w, bias)
    codes = fp8.quantize(x, 0.01)
    y = fp8.linear_heads(codes, q.codes, q.scales, 0.01, streams=streams, heads=heads, bias=bias)
    flat, _ = fp8.linear(codes, q.codes, q.scales, 0.01, bias=bias)
    nobias, _ = fp8.linear(codes, q.codes, q.scales, 0.01)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    want = flat.view(streams, tokens, groups, heads, 64).permute(2, 0, 3, 1, 4)
    assert torch.equal(y.view(torch.int16), want.contiguous().view(torch.int16))
    keys = nobias.view(streams, tokens, groups, heads, 64).permute(2, 0, 3, 1, 4)[0::2]
    assert torch.equal(y[0::2].view(torch.int16), keys.contiguous().view(torch.int16))
    # and against the oracle on a few rows
    rows = np.unique(np.array([0, tokens - 1, streams * tokens - 1]))
    xq = codes.cpu().numpy()[rows]
    y_ref, _ = oracle.fp8_linear(xq, q.codes.cpu().numpy(), 0.01, q.scales.cpu().numpy(), bias.cpu().numpy())
    got = flat.cpu().numpy().view(np.uint16)[rows]
    assert compare_halves(got, y_ref, extra=1280 * 2.0**-24 * 4)[2] <= 0


# ---- the composed encoder ---------------------------------------------------

SMALL = dict(layers=2, decoder_layers=2, frames=300)


@pytest.fixture(scope="module")
def small_encoder(cuda, enc, fp8):
    import torch

    from importlib import import_module

    audio = import_module(PACKAGE + ".audio")
    config = enc.EncoderConfig(**SMALL)
    ck = enc.synthetic_checkpoint(config, seed=3, device=cuda)
    weights = enc.EncoderWeights.from_checkpoint(ck, config)
    mel_full = audio.synthetic_mel_batch(2, seed=40)
    mel = np.ascontiguousarray(mel_full[:, :, : config.frames])
    mel_d = torch.from_numpy(mel).to(cuda)
    scales = enc.calibrate(weights, mel_d)
    return config, ck, weights, scales, mel, mel_d


def test_calibrated_scales_cover_every_key(small_encoder, enc):
    config, _, _, scales, _, _ = small_encoder
    keys = enc.scale_keys(config)
    for names in keys.values():
        for key in names:
            assert np.isfinite(scales[key]) and scales[key] > 0
    with pytest.raises(ValueError, match="model.encoder.layers.1.fc2"):
        bad = dict(scales)
        del bad["model.encoder.layers.1.fc2"]
        enc._scales_for(config, bad)


def _codes_close(got, want, what, min_equal=0.98, far=0):
    """E4M3 codes of values that agree to about an fp16 ulp: mostly identical, and
    otherwise adjacent codes (same sign, magnitude one step apart), except for at
    most `far` codes further apart."""
    got, want = got.astype(np.int32), want.astype(np.int32)
    diff = got != want
    frac = 1 - diff.mean()
    step = np.abs((got & 0x7F) - (want & 0x7F))
    sign_ok = ((got ^ want) & 0x80) == 0
    zero = ((got & 0x7F) == 0) | ((want & 0x7F) == 0)
    adjacent = (step <= 1) & (sign_ok | zero)
    print(f"{what}: {frac:.5f} identical codes, {int((diff & ~adjacent).sum())} further apart")
    assert frac >= min_equal, what
    assert int((diff & ~adjacent).sum()) <= far, what


def test_encoder_stage_by_stage(small_encoder, enc, fp8, oracle, native, cuda):
    import torch

    config, ck, weights, scales, mel, mel_d = small_encoder
    streams, t, d = 2, config.positions, config.d_model
    e = enc.Encoder(weights, scales, streams)
    e.mel.copy_(mel_d)
    host = lambda tensor: tensor.cpu().numpy()
    bits = lambda tensor: tensor.cpu().numpy().view(np.uint16)
    sc = e.scales
    calls = iter(e._calls)
    stream = torch.cuda.current_stream().cuda_stream

    def step(expect):
        name, call = next(calls)
        assert name == expect
        native.check(call(stream), name)
        torch.cuda.synchronize()
        assert native.device_error() == 0

    step("lffw_mel_frames")
    frames = bits(e.frames)
    np.testing.assert_array_equal(frames, oracle.mel_frames(mel))

    w1 = host(ck["model.encoder.conv1.weight"])
    b1 = host(ck["model.encoder.conv1.bias"])
    step("lffw_conv1d_gelu")
    h1 = bits(e.h1)
    assert (h1[:, 0] == 0).all() and (h1[:, -1] == 0).all()
    _, act, out = oracle.conv1d_gelu(frames, w1, b1, 1)
    err = np.abs(_f16(h1[:, 1:-1]) - _f16(out))
    assert (err <= conv_bound(frames, w1, act, out, False)).all()

    w2 = host(ck["model.encoder.conv2.weight"])
    b2 = host(ck["model.encoder.conv2.bias"])
    pos = host(ck["model.encoder.embed_positions.weight"])[:t]
    step("lffw_conv1d_gelu")
    x = bits(e.x0).reshape(streams * t, d)
    _, act, out = oracle.conv1d_gelu(h1, w2, b2, 2, pos)
    err = np.abs(_f16(x.reshape(streams, t, d)) - _f16(out))
    assert (err <= conv_bound(h1, w2, act, out, True)).all()

    def linear_check(codes, weight, act_scale, got, what, gelu=False, next_scale=None, far=0):
        wq, ws = host(weight.codes), host(weight.scales)
        b = host(weight.bias) if weight.bias is not None else None
        y_ref, c_ref = oracle.fp8_linear(codes, wq, act_scale, ws, b, gelu=gelu, next_scale=next_scale,
                                         want_y=next_scale is None)
        if next_scale is not None:
            # A one-ulp move of the pre-GELU value can move the GELU output by two
            # ulps, so a few codes may be two steps apart.
            _codes_close(got, c_ref, what, far=far)
            return
        xa = np.abs(oracle.e4m3_to_float(codes).astype(np.float64))
        wa = np.abs(oracle.e4m3_to_float(wq).astype(np.float64))
        extra = codes.shape[1] * 2.0**-24 * (xa @ wa.T) * (np.float64(act_scale) * ws.astype(np.float64))
        max_abs, _, excess, mism = compare_halves(got, y_ref, extra=extra)
        print(f"{what}: max_abs={max_abs:.3g} mismatch={mism}/{got.size}")
        assert excess <= 0, what

    def fused_residual_check(codes, weight, act_scale, got, residual, what):
        """The plan's linear adds the residual in its epilogue: the same linear
        alone (its y checked against the oracle) plus the fp16 residual add must
        give the plan's output bit for bit."""
        alone, _ = fp8.linear(torch.from_numpy(codes).to(cuda), weight.codes, weight.scales, act_scale,
                              bias=weight.bias)
        torch.cuda.synchronize()
        y = bits(alone).reshape(got.shape)
        linear_check(codes, weight, act_scale, y, what)
        want = (_f16(y).astype(np.float32) + _f16(residual).astype(np.float32)).astype(np.float16)
        np.testing.assert_array_equal(got, want.view(np.uint16))  # one fp16 rounding of the exact sum

    for i, L in enumerate(weights.layers):
        g1, be1 = host(L.ln1[0]), host(L.ln1[1])
        step("lffw_layer_norm")
        _, _, c_ref = oracle.layer_norm(x, g1, be1, code_scale=sc["qkv"][i])
        ln_codes = host(e.ln_codes)
        _codes_close(ln_codes, c_ref, f"layer {i} LN1 codes", min_equal=0.99)

        step("lffw_fp8_linear")
        qkv = bits(e.qkv)
        linear_check(ln_codes, L.qkv, sc["qkv"][i], qkv, f"layer {i} qkv")
        # k columns carry the -0 bias: identical to a bias-free product
        step("lffw_self_attention")
        attn_codes = host(e.attn_codes)
        # The plan's launch writes codes only: the same launch with the fp16 output too
        # gives those codes bit for bit, and its fp16 output is held to the
        # self-attention bound (fixed bound + score-flip and one-pass slack).
        out, codes = fp8.self_attention(e.qkv, streams, config.heads, code_scale=sc["out"][i])
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host(codes), attn_codes)
        want, _ = oracle.self_attention(qkv, streams, config.heads)
        ref = _f16(want)
        slack = _score_flip_slack(_f16(qkv).astype(np.float16), streams, config.heads, ref, one_pass=True)
        err = np.abs(_f16(bits(out)) - ref)
        print(f"layer {i} attention: max_abs={err.max():.3g} mismatch={int((bits(out) != want).sum())}/{want.size}")
        assert np.all(err <= ATOL + RTOL * np.abs(ref) + slack), f"layer {i} attention"

        step("lffw_fp8_linear")
        mid = bits(e.stream_buf[1])
        fused_residual_check(attn_codes, L.out, sc["out"][i], mid, x, f"layer {i} out_proj + residual")
        x = mid

        g2, be2 = host(L.ln2[0]), host(L.ln2[1])
        step("lffw_layer_norm")
        _, _, c_ref = oracle.layer_norm(x, g2, be2, code_scale=sc["fc1"][i])
        ln2_codes = host(e.ln_codes)
        _codes_close(ln2_codes, c_ref, f"layer {i} LN2 codes", min_equal=0.99)

        step("lffw_fp8_linear")
        fc2_codes = host(e.fc2_codes)
        linear_check(ln2_codes, L.fc1, sc["fc1"][i], fc2_codes, f"layer {i} fc1+GELU codes", gelu=True,
                     next_scale=sc["fc2"][i], far=max(4, fc2_codes.size // 50000))
        step("lffw_fp8_linear")
        nxt = bits(e.stream_buf[0])
        fused_residual_check(fc2_codes, L.fc2, sc["fc2"][i], nxt, x, f"layer {i} fc2 + residual")
        x = nxt

    gp, bp = host(weights.ln_post[0]), host(weights.ln_post[1])
    step("lffw_layer_norm")
    _, y_ref, c_ref = oracle.layer_norm(x, gp, bp, code_scale=sc["cross"][0])
    states = bits(e.states).reshape(streams * t, d)
    diff = np.abs(_f16(states) - _f16(y_ref))
    ulp = np.spacing(np.abs(_f16(y_ref)).astype(np.float16)).astype(np.float64)
    assert (diff <= ulp + 2.0**-24).all()
    kv_codes = host(e.kv_codes)
    _codes_close(kv_codes, c_ref, "final LN codes", min_equal=0.99)

    step("lffw_fp8_linear_heads")
    with pytest.raises(StopIteration):
        next(calls)
    kv = bits(e.cross_kv)  # [2 * decoder_layers, streams, heads, t, 64]
    flat = kv.transpose(1, 3, 0, 2, 4).reshape(streams * t, -1)  # back to [rows, group * heads * 64]
    linear_check(kv_codes, weights.cross_kv, sc["cross"][0], flat, "cross k/v")


def _oracle_forward(ck, weights, scales, mel, config, oracle, perturb=None):
    """The oracle's own composition of the encoder stages (states, cross k/v as
    float64).  With `perturb` (a seed), 0.5% of the conv output values move by one
    fp16 ulp first: the size of difference the convolution kernel itself shows."""
    host = lambda tensor: tensor.cpu().numpy()
    streams = mel.shape[0]
    t, d = config.positions, config.d_model
    frames = oracle.mel_frames(mel)
    _, _, h1 = oracle.conv1d_gelu(frames, host(ck["model.encoder.conv1.weight"]),
                                  host(ck["model.encoder.conv1.bias"]), 1)
    h1p = np.zeros((streams, config.frames + 2, d), np.uint16)
    h1p[:, 1:-1] = h1
    _, _, x = oracle.conv1d_gelu(h1p, host(ck["model.encoder.conv2.weight"]), host(ck["model.encoder.conv2.bias"]),
                                 2, host(ck["model.encoder.embed_positions.weight"])[:t])
    x = x.reshape(streams * t, d).copy()
    if perturb is not None:
        rng = np.random.default_rng(perturb)
        flat = x.reshape(-1)
        ok = np.flatnonzero(((flat & 0x7FFF) != 0) & ((flat & 0x7FFF) < 0x7BFF))
        idx = rng.choice(ok, flat.size // 200, replace=False)
        flat[idx] = (flat[idx].astype(np.int32) + rng.choice([-1, 1], idx.size)).astype(np.uint16)
    residual = None
    for i, L in enumerate(weights.layers):
        lin = lambda codes, w, s, **kw: oracle.fp8_linear(codes, host(w.codes), s, host(w.scales),
                                                          None if w.bias is None else host(w.bias), **kw)
        s_x, _, codes = oracle.layer_norm(x, host(L.ln1[0]), host(L.ln1[1]), residual=residual,
                                          code_scale=scales["qkv"][i])
        x = s_x
        qkv, _ = lin(codes, L.qkv, scales["qkv"][i])
        _, ac = oracle.self_attention(qkv, streams, config.heads, code_scale=scales["out"][i])
        o, _ = lin(ac, L.out, scales["out"][i])
        x, _, codes = oracle.layer_norm(x, host(L.ln2[0]), host(L.ln2[1]), residual=o, code_scale=scales["fc1"][i])
        _, hc = lin(codes, L.fc1, scales["fc1"][i], gelu=True, next_scale=scales["fc2"][i], want_y=False)
        residual, _ = lin(hc, L.fc2, scales["fc2"][i])
    _, y, codes = oracle.layer_norm(x, host(weights.ln_post[0]), host(weights.ln_post[1]), residual=residual,
                                    code_scale=scales["cross"][0])
    kv, _ = oracle.fp8_linear(codes, host(weights.cross_kv.codes), scales["cross"][0],
                              host(weights.cross_kv.scales), host(weights.cross_kv.bias))
    kv = _f16(kv).reshape(streams, t, 2 * config.decoder_layers, config.heads, 64).transpose(2, 0, 3, 1, 4)
    return _f16(y), kv


def test_encoder_forward_end_to_end(small_encoder, enc, oracle, native, cuda):
    """The whole plan against the oracle's own composition of the same stages.

    Per-stage rounding differences compound: where a value moves by one fp16 ulp
    across an E4M3 rounding boundary its code moves a whole step (6-12%), and each
    following linear spreads that.  The bound is therefore calibrated on the oracle
    itself: the GPU's distance from the oracle must stay within a small multiple of
    the distance between two oracle runs whose conv outputs differ by one ulp in
    0.5% of the values (the conv kernel's own mismatch rate)."""
    import torch

    config, ck, weights, scales, mel, mel_d = small_encoder
    streams, t, d = 2, config.positions, config.d_model
    e = enc.Encoder(weights, scales, streams)
    states, kv = e.forward(mel_d)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    got_states = states.cpu().numpy().astype(np.float64).reshape(streams * t, d)
    got_kv = kv.cpu().numpy().astype(np.float64)
    # determinism: a second forward gives the same bits
    states2, kv2 = e.forward(mel_d)
    torch.cuda.synchronize()
    assert np.array_equal(states2.cpu().numpy().astype(np.float64).reshape(streams * t, d), got_states)
    assert torch.equal(kv2.view(torch.int16), torch.from_numpy(got_kv.astype(np.float16)).to(cuda).view(torch.int16))

    want_states, want_kv = _oracle_forward(ck, weights, e.scales, mel, config, oracle)
    floor_states, floor_kv = _oracle_forward(ck, weights, e.scales, mel, config, oracle, perturb=1)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))
    r_states, r_kv = rel(got_states, want_states), rel(got_kv, want_kv)
    f_states, f_kv = rel(floor_states, want_states), rel(floor_kv, want_kv)
    print(f"end to end: states rel-RMS {r_states:.2e} (oracle one-ulp floor {f_states:.2e}), "
          f"cross k/v {r_kv:.2e} (floor {f_kv:.2e}), states max_abs {np.abs(got_states - want_states).max():.3g}")
    assert r_states <= 4 * f_states and r_kv <= 4 * f_kv


def test_encoder_stream_slices_are_bit_identical(small_encoder, enc, native, cuda):
    """Streams computed in slices (chunk) write the same bits as one slice of all."""
    import torch

    config, ck, weights, scales, mel, mel_d = small_encoder
    mel3 = torch.cat([mel_d, mel_d[:1].flip(-1).contiguous()])
    whole = enc.Encoder(weights, scales, 3, chunk=3)
    states, kv = whole.forward(mel3)
    torch.cuda.synchronize()
    states, kv = states.clone(), kv.clone()
    sliced = enc.Encoder(weights, scales, 3, chunk=2)
    s2, kv2 = sliced.forward(mel3)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    assert torch.equal(states.view(torch.int16), s2.view(torch.int16))
    assert torch.equal(kv.view(torch.int16), kv2.view(torch.int16))


def test_encoder_forward_with_host_buffers(small_encoder, enc, native, cuda):
    """forward() with log-mel in pinned host memory and states copied back to pinned
    host memory (copies overlapped slice by slice) gives the same bits as the
    device-resident forward, on two calls in a row."""
    import torch

    config, ck, weights, scales, mel, mel_d = small_encoder
    mel3 = torch.cat([mel_d, mel_d[:1].flip(-1).contiguous()])
    e = enc.Encoder(weights, scales, 3, chunk=2)
    states, kv = e.forward(mel3)
    torch.cuda.synchronize()
    states, kv = states.clone(), kv.clone()
    mel_host = mel3.cpu().pin_memory()
    out = torch.empty(tuple(states.shape), dtype=torch.float16).pin_memory()
    stream = torch.cuda.Stream()
    for _ in range(2):
        out.zero_()
        _, kv2 = e.forward(mel_host, stream, states_out=out)
        stream.synchronize()
        assert native.device_error() == 0
        assert torch.equal(out.view(torch.int16), states.cpu().view(torch.int16))
        assert torch.equal(kv2.view(torch.int16), kv.view(torch.int16))
