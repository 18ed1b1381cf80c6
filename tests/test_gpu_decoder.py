"""The greedy decoder (decoder.py, network_graph.cpp:378-416) against the oracle:
its three new kernels -- token + position embedding, self-attention over the fp16
KV cache with the step's key and value appended, greedy token selection -- and
the composed step, stage by stage (each stage fed the GPU's own inputs), then a
short greedy decode end to end and through a replayed CUDA graph."""

from __future__ import annotations

import importlib

import numpy as np
import pytest

from conftest import PACKAGE
from helpers import ATOL, RTOL, compare_halves, halves

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dec(lffw):
    return importlib.import_module(PACKAGE + ".decoder")


def _f16(bits):
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float64)


def _attention_slack(q, k, v, ref):
    """Score-flip slack of one query row per (stream, head) (see test_gpu_attention):
    sum_j p_j ulp(s_j) (|v_j| + |out|), from the oracle's own fp16 score edges."""
    streams, heads, keys, d = k.shape
    c = float(np.float16(d ** -0.25))
    qs = (q.astype(np.float64).reshape(streams, heads, d) * c).astype(np.float16).astype(np.float64)
    ks = (k.astype(np.float64) * c).astype(np.float16).astype(np.float64)
    slack = np.zeros((streams, heads * d))
    for s in range(streams):
        for h in range(heads):
            s16 = (ks[s, h] @ qs[s, h]).astype(np.float16)
            ulp = np.abs(np.spacing(s16)).astype(np.float64)
            sc = s16.astype(np.float64)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            pu = p * ulp
            o = np.abs(ref[s, h * d:(h + 1) * d])
            slack[s, h * d:(h + 1) * d] = pu @ np.abs(v[s, h].astype(np.float64)) + o * pu.sum()
    return slack


def test_decoder_embed_bit_exact(cuda, fp8, native):
    import torch

    rng = np.random.default_rng(3)
    vocab, positions, width = 51866, 448, 1280
    table = torch.from_numpy(halves(rng, (vocab, width), 0.5)).to(cuda)
    pos = torch.from_numpy(halves(rng, (positions, width), 0.5)).to(cuda)
    tokens = torch.tensor([0, 50258, vocab - 1, 17], dtype=torch.int32, device=cuda)
    lengths = torch.tensor([0, 5, positions - 1, 200], dtype=torch.int32, device=cuda)
    x = fp8.decoder_embed(tokens, lengths, table, pos)
    torch.cuda.synchronize()
    assert fp8.decoder_error() == 0
    want = (table[tokens.long()].float().cpu().numpy().astype(np.float64) +
            pos[lengths.long()].float().cpu().numpy().astype(np.float64)).astype(np.float16)
    np.testing.assert_array_equal(x.cpu().numpy().view(np.uint16), want.view(np.uint16))
    # a token outside the table is reported, not read
    bad = torch.tensor([vocab], dtype=torch.int32, device=cuda)
    fp8.decoder_embed(bad, lengths[:1], table, pos)
    torch.cuda.synchronize()
    assert fp8.decoder_error() == 1
    assert fp8.decoder_error() == 0


@pytest.mark.parametrize("lengths", [[0, 1, 5], [127, 128, 129], [300, 447, 63], [0, 255, 383, 446]])
def test_decoder_self_attention_matches_oracle(cuda, fp8, oracle, native, lengths):
    import torch

    rng = np.random.default_rng(sum(lengths) + len(lengths))
    streams, heads, capacity = len(lengths), 20, 448
    width = heads * 64
    qkv = halves(rng, (streams, 3 * width))
    cache_k = halves(rng, (streams, heads, capacity, 64))
    cache_v = halves(rng, (streams, heads, capacity, 64))
    ck, cv = torch.from_numpy(cache_k).to(cuda), torch.from_numpy(cache_v).to(cuda)
    lens = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    out, codes = fp8.decoder_self_attention(torch.from_numpy(qkv).to(cuda), ck, cv, lens, code_scale=0.004)
    torch.cuda.synchronize()
    assert fp8.decoder_error() == 0
    got_k, got_v = ck.cpu().numpy(), cv.cpu().numpy()
    got = out.cpu().numpy()
    for s, n0 in enumerate(lengths):
        # the step's key and value landed at row n0, nothing else moved
        new_k = qkv[s, width:2 * width].reshape(heads, 64)
        new_v = qkv[s, 2 * width:].reshape(heads, 64)
        np.testing.assert_array_equal(got_k[s, :, n0], new_k)
        np.testing.assert_array_equal(got_v[s, :, n0], new_v)
        keep = np.ones(capacity, bool)
        keep[n0] = False
        np.testing.assert_array_equal(got_k[s, :, keep], cache_k[s, :, keep])
        n = n0 + 1
        want, _ = oracle.cross_attention(qkv[s:s + 1, :width], got_k[s:s + 1, :, :n].copy(),
                                         got_v[s:s + 1, :, :n].copy(), 1)
        ref = _f16(want)
        slack = _attention_slack(qkv[s:s + 1, :width], got_k[s:s + 1, :, :n], got_v[s:s + 1, :, :n], ref)
        err = np.abs(got[s:s + 1].astype(np.float64) - ref)
        assert np.all(err <= ATOL + RTOL * np.abs(ref) + slack), (s, n0, float(err.max()))
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(got.view(np.uint16), np.float32(0.004)))


def test_decoder_self_attention_full_cache_is_reported(cuda, fp8):
    import torch

    streams, heads, capacity = 2, 4, 8
    qkv = torch.zeros((streams, 3 * heads * 64), dtype=torch.float16, device=cuda)
    ck = torch.zeros((streams, heads, capacity, 64), dtype=torch.float16, device=cuda)
    cv = torch.zeros_like(ck)
    lens = torch.tensor([3, capacity], dtype=torch.int32, device=cuda)
    fp8.decoder_self_attention(qkv, ck, cv, lens, code_scale=0.01)
    torch.cuda.synchronize()
    assert fp8.decoder_error() == 2


def test_greedy_select_first_maximum_and_suppression(cuda, fp8):
    import torch

    rng = np.random.default_rng(9)
    streams, vocab = 5, 51866
    logits = halves(rng, (streams, vocab), 3.0)
    supp = np.zeros((streams, vocab), np.float32)
    supp[:, 50257:] = -np.inf
    logits[1, [7, 900, 51000]] = np.float16(60000)   # tie: the first index wins
    logits[2, 50300] = np.float16(65504)              # suppressed: ignored
    logits[3, :] = np.float16(-2.0)                   # all equal: token 0
    lengths = torch.tensor([3, 4, 5, 6, 7], dtype=torch.int32, device=cuda)
    tokens = fp8.greedy_select(torch.from_numpy(logits).to(cuda), torch.from_numpy(supp).to(cuda), lengths=lengths)
    torch.cuda.synchronize()
    want = np.argmax(logits.astype(np.float32) + supp, axis=1)
    np.testing.assert_array_equal(tokens.cpu().numpy(), want)
    assert want[1] == 7 and want[3] == 0 and want[2] != 50300
    np.testing.assert_array_equal(lengths.cpu().numpy(), [4, 5, 6, 7, 8])


# ---- the composed decoder ---------------------------------------------------

SMALL = dict(layers=2)
STREAMS = 3


@pytest.fixture(scope="module")
def small_decoder(cuda, dec, fp8):
    import torch

    config = dec.DecoderConfig(**SMALL)
    g = torch.Generator(device=cuda).manual_seed(12)
    ck = dec.add_synthetic_decoder({}, config, seed=21, device=cuda)
    weights = dec.DecoderWeights.from_checkpoint(ck, config)
    # cross K/V as an encoder would leave them: [2 * layers, streams, heads, positions, 64]
    cross_kv = (torch.randn((2 * config.layers, STREAMS, config.heads, config.audio_positions, 64), generator=g,
                            device=cuda)).half()
    scales = dec.calibrate(weights, cross_kv, STREAMS, steps=3)
    return config, ck, weights, scales, cross_kv


def test_decoder_calibration_covers_every_key(small_decoder, dec):
    config, _, _, scales, _ = small_decoder
    for names in dec.scale_keys(config).values():
        for key in names:
            assert np.isfinite(scales[key]) and scales[key] > 0
    with pytest.raises(ValueError, match="model.decoder.layers.1.fc2"):
        bad = dict(scales)
        del bad["model.decoder.layers.1.fc2"]
        dec._scales_for(config, bad)


def _codes_close(got, want, what, min_equal=0.97, far=0):
    got, want = got.astype(np.int32), want.astype(np.int32)
    diff = got != want
    step = np.abs((got & 0x7F) - (want & 0x7F))
    sign_ok = ((got ^ want) & 0x80) == 0
    zero = ((got & 0x7F) == 0) | ((want & 0x7F) == 0)
    adjacent = (step <= 1) & (sign_ok | zero)
    print(f"{what}: {1 - diff.mean():.5f} identical codes, {int((diff & ~adjacent).sum())} further apart")
    assert 1 - diff.mean() >= min_equal, what
    assert int((diff & ~adjacent).sum()) <= far, what


def test_decoder_step_stage_by_stage(small_decoder, dec, fp8, oracle, native, cuda):
    """Two greedy steps, every launch alone, each checked against the oracle on the
    GPU's own inputs of that stage."""
    import torch

    config, ck, weights, scales, cross_kv = small_decoder
    d = dec.Decoder(weights, scales, cross_kv, STREAMS)
    d.reset()
    host = lambda t: t.cpu().numpy()
    bits = lambda t: t.cpu().numpy().view(np.uint16)
    sc = d.scales
    stream = torch.cuda.current_stream().cuda_stream
    token_table = host(weights.token_table)
    pos_table = host(weights.position_table)
    for step_no in range(2):
        calls = iter(d._calls)

        def step(expect):
            name, call = next(calls)
            assert name == expect, (name, expect)
            native.check(call(stream), name)
            torch.cuda.synchronize()
            assert native.device_error() == 0 and fp8.decoder_error() == 0

        tokens, lengths = host(d.tokens).copy(), host(d.lengths).copy()
        assert (lengths == step_no).all()
        step("lffw_decoder_embed")
        x = bits(d.x0)
        want = (token_table[tokens].astype(np.float64) + pos_table[lengths].astype(np.float64)).astype(np.float16)
        np.testing.assert_array_equal(x, want.view(np.uint16))

        def lin_check(codes, lin, act_scale, got, what, gelu=False, next_scale=None):
            wq, ws = host(lin.q.codes), host(lin.q.scales)
            b = host(lin.q.bias) if lin.q.bias is not None else None
            y_ref, c_ref = oracle.fp8_linear(codes, wq, act_scale, ws, b, gelu=gelu, next_scale=next_scale,
                                             want_y=next_scale is None)
            if next_scale is not None:
                _codes_close(got, c_ref, what, far=2)
                return
            xa = np.abs(oracle.e4m3_to_float(codes).astype(np.float64))
            wa = np.abs(oracle.e4m3_to_float(wq).astype(np.float64))
            extra = codes.shape[1] * 2.0**-24 * (xa @ wa.T) * (np.float64(act_scale) * ws.astype(np.float64))
            assert compare_halves(got, y_ref, extra=extra)[2] <= 0, what

        residual = None
        for i, L in enumerate(weights.layers):
            step("lffw_layer_norm")
            if residual is None:
                _, _, c_ref = oracle.layer_norm(x, host(L.ln1[0]), host(L.ln1[1]), code_scale=sc["qkv"][i])
                x_used = x
            else:
                s_ref, _, c_ref = oracle.layer_norm(x, host(L.ln1[0]), host(L.ln1[1]), residual=residual,
                                                    code_scale=sc["qkv"][i])
                x_used = s_ref
            codes = host(d.ln_codes)
            _codes_close(codes, c_ref, f"step {step_no} layer {i} LN1")
            step("lffw_fp8_linear")
            qkv = bits(d.qkv)
            lin_check(codes, L.qkv, sc["qkv"][i], qkv, "qkv")
            step("lffw_decoder_self_attention")
            n = step_no + 1
            kc, vc = host(d.cache_k[i])[:, :, :n].copy(), host(d.cache_v[i])[:, :, :n].copy()
            np.testing.assert_array_equal(kc[:, :, step_no].reshape(STREAMS, -1).view(np.uint16), qkv[:, 1280:2560])
            np.testing.assert_array_equal(vc[:, :, step_no].reshape(STREAMS, -1).view(np.uint16), qkv[:, 2560:])
            out_ref, codes_ref = oracle.cross_attention(qkv[:, :1280].copy(), kc, vc, 1, code_scale=sc["self_out"][i])
            _codes_close(host(d.attn_codes), codes_ref, "self-attention codes", far=2)
            step("lffw_fp8_linear")
            o = bits(d.o)
            lin_check(host(d.attn_codes), L.self_out, sc["self_out"][i], o, "self out_proj")
            step("lffw_layer_norm")
            s_ref, _, c_ref = oracle.layer_norm(x_used, host(L.ln2[0]), host(L.ln2[1]), residual=o,
                                                code_scale=sc["cross_q"][i])
            x2 = [b for b in d.stream_buf if np.array_equal(bits(b), s_ref)]
            assert x2, "residual sum"
            x_used = s_ref
            codes = host(d.ln_codes)
            _codes_close(codes, c_ref, "LN2")
            step("lffw_fp8_linear")
            q = bits(d.q)
            lin_check(codes, L.cross_q, sc["cross_q"][i], q, "cross q_proj")
            step("lffw_cross_attention")
            kx, vx = host(cross_kv[2 * i]), host(cross_kv[2 * i + 1])
            _, codes_ref = oracle.cross_attention(q, kx.view(np.uint16), vx.view(np.uint16), 1,
                                                  code_scale=sc["cross_out"][i])
            _codes_close(host(d.attn_codes), codes_ref, "cross-attention codes", far=2)
            step("lffw_fp8_linear")
            o = bits(d.o)
            lin_check(host(d.attn_codes), L.cross_out, sc["cross_out"][i], o, "cross out_proj")
            step("lffw_layer_norm")
            s_ref, _, c_ref = oracle.layer_norm(x_used, host(L.ln3[0]), host(L.ln3[1]), residual=o,
                                                code_scale=sc["fc1"][i])
            x_used = s_ref
            codes = host(d.ln_codes)
            _codes_close(codes, c_ref, "LN3")
            step("lffw_fp8_linear")
            fc2_codes = host(d.fc2_codes)
            lin_check(codes, L.fc1, sc["fc1"][i], fc2_codes, "fc1 codes", gelu=True, next_scale=sc["fc2"][i])
            step("lffw_fp8_linear")
            residual = bits(d.r)
            lin_check(fc2_codes, L.fc2, sc["fc2"][i], residual, "fc2")
            x = x_used
        step("lffw_layer_norm")
        _, y_ref, _ = oracle.layer_norm(x, host(weights.ln_post[0]), host(weights.ln_post[1]), residual=residual)
        y = bits(d.states)
        ulp = np.spacing(np.abs(_f16(y_ref)).astype(np.float16)).astype(np.float64)
        assert (np.abs(_f16(y) - _f16(y_ref)) <= ulp + 2.0**-24).all()
        step("lffw_fp16_linear")
        logits = bits(d.logits)
        exact = _f16(y) @ token_table.astype(np.float64).T
        want = oracle.half_from_double(exact)
        bound = 1280 * 2.0**-24 * (np.abs(_f16(y)) @ np.abs(token_table.astype(np.float64)).T)
        assert compare_halves(logits, want, extra=bound)[2] <= 0
        step("lffw_greedy_select")
        with pytest.raises(StopIteration):
            next(calls)
        choice = np.argmax(_f16(logits).astype(np.float32) + host(d.suppression), axis=1)
        np.testing.assert_array_equal(host(d.tokens), choice)
        np.testing.assert_array_equal(host(d.lengths), lengths + 1)


def test_greedy_decode_graph_replay_matches_eager(small_decoder, dec, native, cuda):
    """One captured step replayed for every step (lengths and tokens live on the
    device) gives the eager steps' tokens, caches and logits bit for bit."""
    import torch

    config, ck, weights, scales, cross_kv = small_decoder
    steps = 6
    eager = dec.Decoder(weights, scales, cross_kv, STREAMS)
    eager.reset()
    tokens_eager = []
    for _ in range(steps):
        eager.step()
        tokens_eager.append(eager.tokens.clone())
    torch.cuda.synchronize()
    graphed = dec.Decoder(weights, scales, cross_kv, STREAMS)
    s = torch.cuda.Stream(cuda)
    graphed.reset()
    with torch.cuda.stream(s):
        graphed.step(s)  # warm-up outside capture, then start over
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        graphed.step(s)
    graphed.reset()
    graphed.cache_k.zero_()
    graphed.cache_v.zero_()
    tokens_graph = []
    with torch.cuda.stream(s):
        for _ in range(steps):
            graph.replay()
            tokens_graph.append(graphed.tokens.clone())
    torch.cuda.synchronize()
    assert native.device_error() == 0
    for a, b in zip(tokens_eager, tokens_graph):
        assert torch.equal(a, b)
    assert torch.equal(eager.cache_k.view(torch.int16), graphed.cache_k.view(torch.int16))
    assert torch.equal(eager.logits.view(torch.int16), graphed.logits.view(torch.int16))
    assert (graphed.lengths.cpu().numpy() == steps).all()
    del graph
