"""A chain of dependent small-m linears in one persistent launch (lffw_chain_*).

Each link's input is the previous link's E4M3 codes, so the chain's ordering
(link i's activations are read only after every row block of link i-1 is
written) is exercised.  Checks: every link against the CPU oracle
(cpp/src/network_graph.cpp:115-183 semantics) on the GPU's own input codes,
within the linear's bound (helpers.ATOL/RTOL plus the fp32 summation term),
codes bit-exact as Q of the GPU's own fp16 output; reruns and graph replays
bit-identical (the K slices of a split row block are summed in a fixed order);
and per-call lffw_fp8_linear results within one fp16 ulp (the two paths sum
the same products in different fp32 orders)."""

from __future__ import annotations

import numpy as np
import pytest

from helpers import RTOL, accumulation_bound, compare_halves, halves

pytestmark = pytest.mark.gpu


def _links(torch, fp8, cuda, m, shapes, seed):
    """shapes: (k, n, gelu, bias) per link; link i reads link i-1's codes."""
    rng = np.random.default_rng(seed)
    x = fp8.quantize(torch.from_numpy(halves(rng, (m, shapes[0][0]))).to(cuda), 0.01)
    links, inputs = [], x
    for k, n, gelu, has_bias in shapes:
        assert inputs.shape[-1] == k
        w = torch.from_numpy(halves(rng, (n, k), 0.02)).to(cuda)
        b = torch.from_numpy(halves(rng, (n,), 0.02)).to(cuda) if has_bias else None
        q = fp8.QuantizedWeight.from_half(w, b)
        links.append(dict(x_codes=inputs, w_codes=q.codes, w_packed=fp8.pack_skinny(q.codes), w_scales=q.scales,
                          act_scale=0.01, bias=q.bias, bias_host=None if b is None else b.cpu().numpy(),
                          gelu=gelu, out=torch.empty((m, n), dtype=torch.float16, device=cuda),
                          next_scale=0.02 if gelu else 0.01,
                          next_codes=torch.empty((m, n), dtype=torch.uint8, device=cuda)))
        inputs = links[-1]["next_codes"]
    return links


def _run_chain(torch, fp8, native, links):
    chain = fp8.LinearChain(links)
    chain.run()
    torch.cuda.synchronize()
    assert native.device_error() == 0
    got = [(link["out"].clone(), link["next_codes"].clone()) for link in links]
    # A second run of the same chain (its counters are reset per run) gives the same bits.
    chain.run()
    torch.cuda.synchronize()
    for i, link in enumerate(links):
        assert torch.equal(link["out"], got[i][0]) and torch.equal(link["next_codes"], got[i][1]), f"rerun, link {i}"
    chain.close()
    return got


def _check_oracle(oracle, links, got):
    for i, (link, (y, codes)) in enumerate(zip(links, got)):
        xq = link["x_codes"].cpu().numpy()
        wq = link["w_codes"].cpu().numpy()
        ws = link["w_scales"].cpu().numpy()
        act = np.float32(link["act_scale"])
        y_ref, _ = oracle.fp8_linear(xq, wq, act, ws, link["bias_host"], gelu=link["gelu"])
        y_bits = y.cpu().numpy().view(np.uint16)
        extra = accumulation_bound(oracle, xq, wq, act, ws, xq.shape[-1], gain=1.13 if link["gelu"] else 1.0)
        rtol = 2 * RTOL if link["gelu"] else RTOL
        max_abs, _, excess, mismatches = compare_halves(y_bits, y_ref, rtol=rtol, extra=extra)
        assert excess <= 0, f"link {i}: max_abs {max_abs}"
        assert mismatches <= max(8, y_bits.size // 500), f"link {i}: {mismatches} mismatches"
        np.testing.assert_array_equal(codes.cpu().numpy(), oracle.quantize(y_bits, np.float32(link["next_scale"])))


LAYER = [(1280, 3840, False, True), (3840, 1280, False, True), (1280, 1280, False, False),
         (1280, 5120, True, True), (5120, 1280, False, True)]


@pytest.mark.parametrize("m,shapes", [
    (20, LAYER),                                   # a decoder layer's linears, chained
    (1, LAYER),
    (32, LAYER + LAYER),
    (7, [(1280, 1280, False, True)] * 12),         # a long chain of 10-block links
    (13, [(1024, 1024, False, True), (1024, 2048, True, True), (2048, 640, False, False)]),
    # K in 1 to 32 slices (split row blocks summed by the last slice), ragged N,
    # K below one 128-byte block, more units than CTAs
    (13, [(384, 16, False, True), (16, 4096, True, False), (4096, 48, False, True)]),
    (3, [(256, 40960, False, True), (40960, 272, True, True)]),
    (32, [(640, 1008, False, True), (1008, 128, False, False), (128, 1408, False, True), (1408, 3856, True, True)]),
])
def test_chain_matches_oracle(cuda, fp8, oracle, native, m, shapes):
    import torch

    links = _links(torch, fp8, cuda, m, shapes, seed=m + len(shapes))
    got = _run_chain(torch, fp8, native, links)
    _check_oracle(oracle, links, got)
    # The per-call path sums the same products in another fp32 order: both lie
    # within the summation bound of the exact sum, so within twice it of each other.
    for i, ((y, _), link) in enumerate(zip(got, links)):
        y_ref, _ = fp8.linear(link["x_codes"], None, link["w_scales"], link["act_scale"], bias=link["bias"],
                              gelu=link["gelu"], w_packed=link["w_packed"])
        torch.cuda.synchronize()
        xq = link["x_codes"].cpu().numpy()
        extra = 2 * accumulation_bound(oracle, xq, link["w_codes"].cpu().numpy(), np.float32(link["act_scale"]),
                                       link["w_scales"].cpu().numpy(), xq.shape[-1], gain=1.13 if link["gelu"] else 1.0)
        _, _, excess, _ = compare_halves(y.cpu().numpy().view(np.uint16), y_ref.cpu().numpy().view(np.uint16),
                                         rtol=(4 if link["gelu"] else 2) * RTOL, extra=extra)
        assert excess <= 0, f"link {i}"


def test_chain_codes_only_and_device_scale(cuda, fp8, native):
    """Links without an fp16 output, and a device-resident act_scale, give the
    same codes as the full chain."""
    import torch

    links = _links(torch, fp8, cuda, 9, LAYER[:3], seed=5)
    full = _run_chain(torch, fp8, native, links)
    scale = torch.tensor([0.01], dtype=torch.float32, device=cuda)
    lean = [dict(link, out=None, act_scale=scale if i == 1 else link["act_scale"],
                 next_codes=torch.empty_like(link["next_codes"])) for i, link in enumerate(links)]
    for i in range(1, len(lean)):
        lean[i]["x_codes"] = lean[i - 1]["next_codes"]
    chain = fp8.LinearChain(lean)
    chain.run()
    torch.cuda.synchronize()
    assert native.device_error() == 0
    for i, link in enumerate(lean):
        assert torch.equal(link["next_codes"], full[i][1]), f"link {i}"
    chain.close()


def test_chain_in_a_cuda_graph(cuda, fp8, native):
    """The chain (counter reset + launch) replays from a captured graph."""
    import torch

    links = _links(torch, fp8, cuda, 20, LAYER, seed=6)
    chain = fp8.LinearChain(links)
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        chain.run(torch.cuda.current_stream())
    for link in links:
        link["next_codes"].zero_()
        link["out"].zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert native.device_error() == 0
    first = [(link["out"].clone(), link["next_codes"].clone()) for link in links]
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    for i, link in enumerate(links):
        assert torch.equal(link["out"], first[i][0]) and torch.equal(link["next_codes"], first[i][1])
    del graph
    eager = _run_chain(torch, fp8, native, links)
    for i in range(len(links)):
        assert torch.equal(eager[i][0], first[i][0]) and torch.equal(eager[i][1], first[i][1]), f"link {i}"
    chain.close()


def test_chain_rejects_mixed_m(cuda, fp8, native):
    import torch

    a = _links(torch, fp8, cuda, 4, [(256, 256, False, True)], seed=2)
    b = _links(torch, fp8, cuda, 5, [(256, 256, False, True)], seed=3)
    with pytest.raises(native.NativeError):
        fp8.LinearChain([a[0], b[0]])
