"""C ABI contracts that need no GPU: the library loads and exports every
symbol include/lffw_fp8.h declares; argument validation rejects bad calls
before touching a device; the plugin creators keep the reference's names,
versions, namespace, fields and shape/dtype/format checks
(cpp/tests/plugin_contracts.cpp:38-130)."""

from __future__ import annotations

import ctypes

import pytest

NS = b"listenflow.fastest_whisper"


@pytest.fixture(scope="module")
def lib(native):
    return native.library()


def test_every_declared_symbol_is_exported(native, lib):
    names = native.declared_symbols()
    assert "lffw_fp8_linear" in names and "tensoracle_bundle_sha256" in names
    for name in names:
        assert hasattr(lib, name), name
    digest = native.bundle_sha256()
    assert len(digest) == 64 and all(c in "0123456789abcdef" for c in digest)


def _linear_args(native, **over):
    a = native.LinearArgs()
    a.struct_size = ctypes.sizeof(native.LinearArgs)
    a.m, a.n, a.k = 128, 256, 1280
    a.x_codes, a.w_codes, a.w_scales, a.y = 0x10000, 0x20000, 0x30000, 0x40000
    a.act_scale = 0.01
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    dict(m=0), dict(n=0), dict(k=0), dict(k=1288), dict(n=250), dict(m=2**31),
    dict(x_codes=None), dict(w_codes=None), dict(w_scales=None), dict(y=None),
    dict(x_codes=0x10008), dict(y=0x40002), dict(bias=0x50004),
    dict(act_scale=0.0), dict(act_scale=-0.1), dict(act_scale=float("nan")), dict(act_scale=float("inf")),
    dict(next_codes=0x60000, next_scale=0.0), dict(epilogue=7),
    # the residual add: y only (no GELU, no next codes), n % 32 == 0, aligned, row-major weights
    dict(residual=0x70000, epilogue=1), dict(residual=0x70000, next_codes=0x60000, next_scale=0.01),
    dict(residual=0x70000, y=None, next_codes=0x60000, next_scale=0.01), dict(residual=0x70000, n=272),
    dict(residual=0x70008), dict(residual=0x70000, m=4, w_layout=1),
])
def test_linear_rejects_invalid_arguments(native, lib, change):
    a = _linear_args(native, **change)
    assert lib.lffw_fp8_linear(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_linear_abi_mismatch_and_null(native, lib):
    a = _linear_args(native, struct_size=8)
    assert lib.lffw_fp8_linear(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_fp8_linear(None, None) == native.INVALID_ARGUMENT


def test_linear_residual_field_ignored_for_older_callers(native, lib):
    """A caller built before the residual field passes a shorter struct_size: whatever
    lies past it is not read, so a misaligned value there is no argument error."""
    a = _linear_args(native, residual=0x70008)
    assert lib.lffw_fp8_linear(ctypes.byref(a), None) == native.INVALID_ARGUMENT
    a.struct_size = native.LinearArgs.residual.offset
    assert lib.lffw_fp8_linear(ctypes.byref(a), None) != native.INVALID_ARGUMENT


def _chain(native, lib, links):
    arr = (native.LinearArgs * len(links))(*links)
    handle = ctypes.c_void_p(0x1234)
    status = lib.lffw_chain_create(arr, len(links), ctypes.byref(handle))
    return status, handle.value


@pytest.mark.parametrize("links", [
    # row-major weights, m above the small-m limit, links of different m, a bad link
    lambda n: [_linear_args(n, m=4)],
    lambda n: [_linear_args(n, m=33, w_layout=n.WEIGHTS_SKINNY_TILES)],
    lambda n: [_linear_args(n, m=4, w_layout=n.WEIGHTS_SKINNY_TILES),
               _linear_args(n, m=5, w_layout=n.WEIGHTS_SKINNY_TILES)],
    lambda n: [_linear_args(n, m=4, w_layout=n.WEIGHTS_SKINNY_TILES),
               _linear_args(n, m=4, w_layout=n.WEIGHTS_SKINNY_TILES, act_scale=0.0)],
])
def test_chain_rejects_invalid_links(native, lib, links):
    status, handle = _chain(native, lib, links(native))
    assert status == native.INVALID_ARGUMENT
    assert handle is None  # the out-pointer is cleared on failure


def test_chain_null_and_count(native, lib):
    bad = native.INVALID_ARGUMENT
    one = (native.LinearArgs * 1)(_linear_args(native, m=4, w_layout=native.WEIGHTS_SKINNY_TILES))
    handle = ctypes.c_void_p()
    assert lib.lffw_chain_create(None, 1, ctypes.byref(handle)) == bad
    assert lib.lffw_chain_create(one, 0, ctypes.byref(handle)) == bad
    assert lib.lffw_chain_create(one, -1, ctypes.byref(handle)) == bad
    assert lib.lffw_chain_create(one, 1, None) == bad
    assert lib.lffw_chain_run(None, None) == bad
    lib.lffw_chain_destroy(None)  # a no-op


def test_other_entry_points_reject_invalid_arguments(native, lib):
    bad = native.INVALID_ARGUMENT
    assert lib.lffw_fp8_quantize(0x1000, 16, 0.0, None, 0x2000, None) == bad
    assert lib.lffw_fp8_quantize(0x1000, 0, 1.0, None, 0x2000, None) == bad
    assert lib.lffw_fp8_quantize(None, 16, 1.0, None, 0x2000, None) == bad
    assert lib.lffw_fp8_quantize_rows(0x1000, 0, 16, 0x2000, 0x3000, None) == bad
    assert lib.lffw_fp8_weight_scales(None, 4, 16, 0x2000, None) == bad
    assert lib.lffw_fp8_dynamic_scale(0x1000, 16, 0x2002, None, None) == bad
    assert lib.lffw_fp16_fc1(0x1000, 0x2000, 0x3000, 0x4000, 5120, 1284, None) == bad
    assert lib.lffw_fp16_qkv(0x1000, 0x2000, None, 0x3000, 0x4000, 1280, None) == bad
    assert lib.lffw_fp16_bias(0x1000, 0, 0x2000, 0, None) == bad
    assert lib.lffw_fp16_bias(0x1000, 0, 0x2000, 2**31, None) == bad
    assert lib.lffw_fp16_gelu(None, 0x2000, 4, None) == bad


def _norm_args(native, **over):
    a = native.LayerNormArgs()
    a.struct_size = ctypes.sizeof(native.LayerNormArgs)
    a.rows, a.cols = 16, 1280
    a.x, a.gamma, a.beta, a.codes = 0x10000, 0x20000, 0x30000, 0x40000
    a.epsilon = 1e-5
    a.code_scale = 0.01
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    {"rows": 0}, {"cols": 4}, {"cols": 1284}, {"cols": 4104}, {"x": None}, {"gamma": None},
    {"beta": None}, {"x": 0x10008}, {"residual": 0x50004}, {"codes": None},
    {"epsilon": -1.0}, {"epsilon": float("nan")}, {"epsilon": float("inf")},
    {"code_scale": 0.0}, {"code_scale": float("nan")}, {"code_scale": 2.0**126},
])
def test_layer_norm_rejects_invalid_arguments(native, lib, change):
    """No output at all, ragged or oversized rows, misaligned pointers, a bad
    epsilon or code scale: rejected before any device call."""
    a = _norm_args(native, **change)
    assert lib.lffw_layer_norm(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_layer_norm_abi_mismatch_and_null(native, lib):
    a = _norm_args(native)
    a.struct_size = 8
    assert lib.lffw_layer_norm(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_layer_norm(None, None) == native.INVALID_ARGUMENT


def _attn_args(native, **over):
    a = native.CrossAttentionArgs()
    a.struct_size = ctypes.sizeof(native.CrossAttentionArgs)
    a.streams, a.queries, a.heads, a.head_dim, a.keys = 4, 5, 20, 64, 1500
    a.q, a.k, a.v, a.out = 0x10000, 0x20000, 0x30000, 0x40000
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    {"head_dim": 128}, {"queries": 0}, {"queries": 17}, {"keys": 0}, {"keys": 4097}, {"streams": 0},
    {"heads": 0}, {"streams": 2**20, "heads": 2**10}, {"q": None}, {"k": None}, {"v": None}, {"out": None},
    {"q": 0x10002}, {"v": 0x30008}, {"out_codes": 0x50000, "code_scale": 0.0},
])
def test_cross_attention_rejects_invalid_arguments(native, lib, change):
    a = _attn_args(native, **change)
    assert lib.lffw_cross_attention(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_cross_attention_abi_mismatch_and_null(native, lib):
    a = _attn_args(native)
    a.struct_size = 16
    assert lib.lffw_cross_attention(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_cross_attention(None, None) == native.INVALID_ARGUMENT


def _self_args(native, **over):
    a = native.SelfAttentionArgs()
    a.struct_size = ctypes.sizeof(native.SelfAttentionArgs)
    a.streams, a.tokens, a.heads, a.head_dim = 8, 1500, 20, 64
    a.q, a.k, a.v, a.out = 0x10000, 0x10000 + 2560, 0x10000 + 5120, 0x40000
    a.q_ld = a.k_ld = a.v_ld = 3840
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    {"head_dim": 32}, {"tokens": 0}, {"streams": 0}, {"heads": 0}, {"streams": 2**16, "tokens": 2**15},
    {"q_ld": 1000}, {"k_ld": 3844}, {"v_ld": 0}, {"q": None}, {"out": None}, {"k": 0x10004},
    {"out_codes": 0x50000, "code_scale": float("inf")},
    # 2^30 rows of one token: 2^30 x 20 (stream, head, query block) items, past 32 bits
    {"streams": 2**30, "tokens": 1},
    # items + 65536 reaches 2^31: the persistent loop's last step would overflow
    {"streams": 2**31 - 65536, "tokens": 1, "heads": 1},
])
def test_self_attention_rejects_invalid_arguments(native, lib, change):
    a = _self_args(native, **change)
    assert lib.lffw_self_attention(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_self_attention_abi_mismatch_and_null(native, lib):
    a = _self_args(native)
    a.struct_size = 16
    assert lib.lffw_self_attention(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_self_attention(None, None) == native.INVALID_ARGUMENT


def test_device_gate_without_sm100(native, lib):
    import torch

    if torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0):
        assert lib.lffw_device_supported(0) == native.SUCCESS
    else:
        assert lib.lffw_device_supported(0) != native.SUCCESS
    assert lib.lffw_device_supported(-1) == native.INVALID_ARGUMENT


# ---- plugin creators ---------------------------------------------------------

def creators(native, lib):
    out = {}
    for i in range(lib.lffw_plugin_creator_count()):
        name, version, ns = ctypes.c_char_p(), ctypes.c_char_p(), ctypes.c_char_p()
        fields = ctypes.POINTER(native.PluginField)()
        count = ctypes.c_int32()
        assert lib.lffw_plugin_creator(i, ctypes.byref(name), ctypes.byref(version), ctypes.byref(ns),
                                       ctypes.byref(fields), ctypes.byref(count)) == 0
        out[name.value.decode()] = (version.value, ns.value,
                                    [(fields[j].name.decode(), fields[j].type, fields[j].length)
                                     for j in range(count.value)])
    assert lib.lffw_plugin_creator(lib.lffw_plugin_creator_count(), None, None, None, None, None) == -1
    return out


def test_creator_names_versions_namespace_and_fields(native, lib):
    c = creators(native, lib)
    assert c["LffwFp16Fc1"] == (b"1", NS, [("bundle_sha256", native.FIELD_CHAR, 64)])
    assert c["LffwFp16Qkv"] == (b"2", NS, [("bundle_sha256", native.FIELD_CHAR, 64)])
    assert c["LffwFp16Bias"] == (b"1", NS, [("bundle_sha256", native.FIELD_CHAR, 64),
                                            ("bias", native.FIELD_FLOAT16, 1)])
    assert c["LffwFp8Linear"][0:2] == (b"1", NS)
    assert [f[0] for f in c["LffwFp8Linear"][2]] == ["bundle_sha256", "act_scale", "epilogue", "output_scale",
                                                    "has_bias"]


class Fields:
    """Keeps the ctypes buffers of a field collection alive."""

    def __init__(self, native, spec):
        self.keep = []
        arr = (native.PluginField * max(1, len(spec)))()
        for i, (name, ctype, ftype, values) in enumerate(spec):
            buf = (ctype * len(values))(*values)
            self.keep.append(buf)
            arr[i].name = name.encode()
            arr[i].data = ctypes.cast(buf, ctypes.c_void_p)
            arr[i].type = ftype
            arr[i].length = len(values)
        self.array, self.count = arr, len(spec)


def digest_field(native, text=None):
    d = (text or native.bundle_sha256()).encode()
    return ("bundle_sha256", ctypes.c_char, native.FIELD_CHAR, list(d))


def create(native, lib, name, version, spec, phase=0, ns=NS):
    f = Fields(native, spec)
    return lib.lffw_plugin_create(name.encode(), version, ns, f.array, f.count, phase)


def fp8_spec(native, act=0.01, epi=0, out=0.0, has_bias=1):
    return [digest_field(native), ("act_scale", ctypes.c_float, native.FIELD_FLOAT32, [act]),
            ("epilogue", ctypes.c_int32, native.FIELD_INT32, [epi]),
            ("output_scale", ctypes.c_float, native.FIELD_FLOAT32, [out]),
            ("has_bias", ctypes.c_int32, native.FIELD_INT32, [has_bias])]


def test_create_accepts_exact_fields_and_rejects_everything_else(native, lib):
    good = [digest_field(native)]
    for name, version in (("LffwFp16Fc1", b"1"), ("LffwFp16Qkv", b"2")):
        for phase in (native.PHASE_BUILD, native.PHASE_RUNTIME):
            p = create(native, lib, name, version, good, phase)
            assert p
            clone = lib.lffw_plugin_clone(p)
            assert clone
            lib.lffw_plugin_destroy(clone)
            lib.lffw_plugin_destroy(p)
        assert not create(native, lib, name, version, good, phase=2)
        assert not create(native, lib, name, b"9", good)
        assert not create(native, lib, name, version, good, ns=b"other")
        assert not create(native, lib, name, version, [digest_field(native, "0" * 64)])
        assert not create(native, lib, name, version, [])
        assert not create(native, lib, name, version,
                          good + [("bias", ctypes.c_uint16, native.FIELD_FLOAT16, [0xB600])])
        assert not create(native, lib, name, version,
                          [("bundle_sha256", ctypes.c_char, native.FIELD_INT8, list(native.bundle_sha256().encode()))])
    bias = good + [("bias", ctypes.c_uint16, native.FIELD_FLOAT16, [0xB600])]  # -0.375
    p = create(native, lib, "LffwFp16Bias", b"1", bias)
    assert p
    lib.lffw_plugin_destroy(p)
    assert not create(native, lib, "LffwFp16Bias", b"1", good)
    assert not create(native, lib, "LffwFp16Bias", b"1",
                      good + [("bias", ctypes.c_float, native.FIELD_FLOAT32, [0.5])])
    p = create(native, lib, "LffwFp8Linear", b"1", fp8_spec(native))
    assert p
    lib.lffw_plugin_destroy(p)
    for bad in (dict(act=0.0), dict(act=float("nan")), dict(epi=3), dict(out=-1.0), dict(has_bias=2)):
        assert not create(native, lib, "LffwFp8Linear", b"1", fp8_spec(native, **bad))


def _valid(native, lib, plugin, inputs, output):
    ins = (native.TensorDesc * len(inputs))(*inputs)
    return lib.lffw_plugin_validate(plugin, ins, len(inputs), ctypes.byref(output)) == 0


@pytest.mark.parametrize("name,version", [("LffwFp16Fc1", b"1"), ("LffwFp16Qkv", b"2")])
def test_projection_shape_checks(native, lib, name, version):
    T = native.TensorDesc.of
    qkv = name == "LffwFp16Qkv"
    rows = 3840 if qkv else 5120
    plugin = create(native, lib, name, version, [digest_field(native)])
    try:
        inputs = [T((1, 1, 1280)), T((rows, 1280)), T((1280,) if qkv else (5120,))]
        if qkv:
            inputs.append(T((1280,)))
        output = T((1, 1, rows))
        assert _valid(native, lib, plugin, inputs, output)
        assert lib.lffw_plugin_workspace_size(plugin, None, 0) == 0  # plugin_contracts.cpp:58
        for i in range(len(inputs)):
            bad = list(inputs)
            bad[i] = T(inputs[i].shape, native.DT_FLOAT)
            assert not _valid(native, lib, plugin, bad, output), "fp32 input"
            bad[i] = T(inputs[i].shape, native.DT_HALF, native.FORMAT_CHW2)
            assert not _valid(native, lib, plugin, bad, output), "non-LINEAR input"
            shape = list(inputs[i].shape)
            shape[-1] -= 1
            bad[i] = T(shape)
            assert not _valid(native, lib, plugin, bad, output), "width"
        assert not _valid(native, lib, plugin, inputs, T((1, 1, rows), native.DT_FLOAT))
        assert not _valid(native, lib, plugin, inputs, T((1, 1, rows + 1)))
        for x in ((1280,), (1, 2, 1280), (2, 1, 1280)):
            assert not _valid(native, lib, plugin, [T(x)] + inputs[1:], output)
        for w in ((1280, rows), (1, rows, 1280)):
            assert not _valid(native, lib, plugin, [inputs[0], T(w)] + inputs[2:], output)
        assert not _valid(native, lib, plugin, inputs[:2] + [T((1, inputs[2].shape[0]))] + inputs[3:], output)
        assert not _valid(native, lib, plugin, inputs[:-1], output)
    finally:
        lib.lffw_plugin_destroy(plugin)


def test_bias_plugin_count_boundaries(native, lib):
    T = native.TensorDesc.of
    spec = [digest_field(native), ("bias", ctypes.c_uint16, native.FIELD_FLOAT16, [0xB600])]
    plugin = create(native, lib, "LffwFp16Bias", b"1", spec)
    try:
        for n in (1, 127, 128, 129, 4097, 2**31 - 1, -1):
            assert _valid(native, lib, plugin, [T((n,))], T((n,))), n
        for n in (0, -2, 2**31):
            assert not _valid(native, lib, plugin, [T((n,))], T((n,))), n
        assert not _valid(native, lib, plugin, [T((5,))], T((6,)))
        assert not _valid(native, lib, plugin, [T((5,), native.DT_FLOAT)], T((5,)))
        assert not _valid(native, lib, plugin, [T((1, 5))], T((1, 5)))
    finally:
        lib.lffw_plugin_destroy(plugin)


def test_fp8_linear_plugin_shape_checks_and_workspace(native, lib):
    T = native.TensorDesc.of
    plugin = create(native, lib, "LffwFp8Linear", b"1", fp8_spec(native))
    codes_out = create(native, lib, "LffwFp8Linear", b"1", fp8_spec(native, out=0.05, has_bias=0))
    try:
        x16 = T((8, 1500, 1280))
        w = T((5120, 1280), native.DT_FP8)
        s = T((5120,), native.DT_FLOAT)
        b = T((5120,))
        out = T((8, 1500, 5120))
        assert _valid(native, lib, plugin, [x16, w, s, b], out)
        assert _valid(native, lib, plugin, [T((12000, 1280), native.DT_FP8), w, s, b], T((12000, 5120)))
        ins = (native.TensorDesc * 4)(x16, w, s, b)
        assert lib.lffw_plugin_workspace_size(plugin, ins, 4) == 12000 * 1280
        fp8_in = (native.TensorDesc * 4)(T((12000, 1280), native.DT_FP8), w, s, b)
        assert lib.lffw_plugin_workspace_size(plugin, fp8_in, 4) == 0
        assert not _valid(native, lib, plugin, [x16, w, s], out)  # has_bias=1 needs 4 inputs
        assert not _valid(native, lib, plugin, [x16, T((5120, 1280)), s, b], out)
        assert not _valid(native, lib, plugin, [x16, w, T((5120,)), b], out)
        assert not _valid(native, lib, plugin, [x16, T((5120, 1288), native.DT_FP8), s, b], out)
        assert not _valid(native, lib, plugin, [x16, w, s, b], T((8, 1500, 5120), native.DT_FP8))
        assert not _valid(native, lib, plugin, [x16, w, s, b], T((8, 1501, 5120)))
        assert _valid(native, lib, codes_out, [x16, w, s], T((8, 1500, 5120), native.DT_FP8))
        assert not _valid(native, lib, codes_out, [x16, w, s], T((8, 1500, 5120)))
    finally:
        lib.lffw_plugin_destroy(plugin)
        lib.lffw_plugin_destroy(codes_out)


def test_enqueue_rejects_null_and_bad_shapes_without_a_launch(native, lib):
    T = native.TensorDesc.of
    plugin = create(native, lib, "LffwFp16Fc1", b"1", [digest_field(native)])
    try:
        ins = (native.TensorDesc * 3)(T((1, 1, 1280)), T((5120, 1280)), T((5120,)))
        out = T((1, 1, 5120))
        ptrs = (ctypes.c_void_p * 3)(0x1000, 0x2000, None)
        outs = (ctypes.c_void_p * 1)(0x4000)
        assert lib.lffw_plugin_enqueue(plugin, ins, ctypes.byref(out), ptrs, outs, None, None) == -1
        ptrs[2] = 0x3000
        bad_out = T((1, 1, 5121))
        assert lib.lffw_plugin_enqueue(plugin, ins, ctypes.byref(bad_out), ptrs, outs, None, None) == -1
        assert lib.lffw_plugin_enqueue(None, ins, ctypes.byref(out), ptrs, outs, None, None) == -1
    finally:
        lib.lffw_plugin_destroy(plugin)


def _conv_args(native, **over):
    a = native.Conv1dArgs()
    a.struct_size = ctypes.sizeof(native.Conv1dArgs)
    a.streams, a.frames_in, a.c_in, a.c_out, a.stride = 2, 3000, 1280, 1280, 2
    a.x, a.weight, a.bias, a.y = 0x10000, 0x20000, 0x30000, 0x40000
    a.y_rows, a.y_row0 = 1500, 0
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    {"stride": 3}, {"stride": 0}, {"streams": 0}, {"frames_in": 1}, {"frames_in": 2999}, {"c_in": 96},
    {"c_in": 0}, {"c_out": 48}, {"y_rows": 1499}, {"y_row0": 1}, {"y_row0": -1}, {"x": None}, {"weight": None},
    {"bias": None}, {"y": None}, {"x": 0x10008}, {"positions": 0x50004}, {"streams": 2**20, "y_rows": 2**12},
])
def test_conv1d_rejects_invalid_arguments(native, lib, change):
    a = _conv_args(native, **change)
    assert lib.lffw_conv1d_gelu(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_conv1d_abi_mismatch_and_null(native, lib):
    a = _conv_args(native, struct_size=8)
    assert lib.lffw_conv1d_gelu(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_conv1d_gelu(None, None) == native.INVALID_ARGUMENT


def _heads_args(native, **over):
    a = native.HeadsLinearArgs()
    a.struct_size = ctypes.sizeof(native.HeadsLinearArgs)
    a.streams, a.tokens, a.heads, a.n, a.k = 8, 1500, 20, 81920, 1280
    a.x_codes, a.w_codes, a.w_scales, a.y = 0x10000, 0x20000, 0x30000, 0x40000
    a.act_scale = 0.01
    for key, value in over.items():
        setattr(a, key, value)
    return a


@pytest.mark.parametrize("change", [
    {"streams": 0}, {"tokens": 0}, {"heads": 0}, {"k": 1288}, {"k": 0}, {"n": 1000}, {"n": 81920 + 64},
    {"x_codes": None}, {"w_codes": None}, {"w_scales": None}, {"y": None}, {"y": 0x40002},
    {"act_scale": 0.0}, {"act_scale": float("nan")}, {"streams": 2**20, "tokens": 2**11}, {"y_streams": 7},
])
def test_linear_heads_rejects_invalid_arguments(native, lib, change):
    a = _heads_args(native, **change)
    assert lib.lffw_fp8_linear_heads(ctypes.byref(a), None) == native.INVALID_ARGUMENT


def test_linear_heads_abi_mismatch_and_null(native, lib):
    a = _heads_args(native, struct_size=8)
    assert lib.lffw_fp8_linear_heads(ctypes.byref(a), None) == native.ABI_MISMATCH
    assert lib.lffw_fp8_linear_heads(None, None) == native.INVALID_ARGUMENT


@pytest.mark.parametrize("args", [
    (None, 1, 128, 3000, 0x20000), (0x10000, 0, 128, 3000, 0x20000), (0x10000, 1, 12, 3000, 0x20000),
    (0x10000, 1, 128, 0, 0x20000), (0x10000, 1, 128, 3000, None), (0x10004, 1, 128, 3000, 0x20000),
])
def test_mel_frames_rejects_invalid_arguments(native, lib, args):
    assert lib.lffw_mel_frames(*args, None) == native.INVALID_ARGUMENT


def test_conv_weight_layout_rejects_invalid_arguments(native, lib):
    assert lib.lffw_conv1d_weight_layout(None, 4, 4, 0x10000, None) == native.INVALID_ARGUMENT
    assert lib.lffw_conv1d_weight_layout(0x10000, 0, 4, 0x20000, None) == native.INVALID_ARGUMENT
    assert lib.lffw_conv1d_weight_layout(0x10000, 4, 4, 0x10000, None) == native.INVALID_ARGUMENT
