"""sana_op_linear_attention_noalloc (fixed device scratch, no allocation) against
sana_op_linear_attention_device (caller-provided workspace), through the C ABI.

The file name sorts last, so in a full run it goes after every other test of the process;
it sets up everything it uses itself, so it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-6  # relative L2; both entry points run the same kernels on the same inputs

_vp, _i = ctypes.c_void_p, ctypes.c_int


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def env():
    import torch
    from sana_b200 import SANA_MODE_BF16, SanaCuda
    g = SanaCuda(0, SANA_MODE_BF16)
    g.lib.sana_op_linear_attention_workspace.restype = ctypes.c_size_t
    st = torch.cuda.Stream()
    g.set_stream(st.cuda_stream)
    yield torch, g, st
    g.close()


def _case(torch, S, T, heads, D, seed):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(S * T, 3 * heads * D, generator=gen).to(device="cuda", dtype=torch.bfloat16)
    return qkv


def _with_workspace(torch, g, qkv, S, T, heads, D):
    ws = g.lib.sana_op_linear_attention_workspace(_i(S), _i(T), _i(heads), _i(D))
    part = torch.empty(ws // 4, device="cuda", dtype=torch.float32)
    out = torch.empty(S * T, heads * D, device="cuda", dtype=torch.bfloat16)
    g._call("sana_op_linear_attention_device", _vp(qkv.data_ptr()), _i(S), _i(T), _i(heads), _i(D),
            _vp(part.data_ptr()), _vp(out.data_ptr()))
    return out


def _noalloc(torch, g, qkv, S, T, heads, D):
    out = torch.empty(S * T, heads * D, device="cuda", dtype=torch.bfloat16)
    g._call("sana_op_linear_attention_noalloc", _vp(qkv.data_ptr()), _i(S), _i(T), _i(heads), _i(D),
            _vp(out.data_ptr()))
    return out


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row(env):
    torch, g, st = env
    cases = [(2, 1024, 36, 32, 11), (2, 1024, 16, 72, 12)]
    with torch.cuda.stream(st):
        inputs = [_case(torch, *c) for c in cases]
        refs = [_with_workspace(torch, g, x, *c[:4]) for x, c in zip(inputs, cases)]
        st.synchronize()
        # two calls back to back on one stream, different shapes, no sync in between
        got = [_noalloc(torch, g, x, *c[:4]) for x, c in zip(inputs, cases)]
        st.synchronize()
    for c, a, b in zip(cases, got, refs):
        e = rel_err(a.float().cpu().numpy(), b.float().cpu().numpy())
        assert e <= TOL, (c, e)
        assert torch.isfinite(a.float()).all()


def test_noalloc_allocates_no_device_memory(env):
    torch, g, st = env
    c = (2, 1024, 36, 32)
    with torch.cuda.stream(st):
        x = _case(torch, *c, 21)
        ref = _with_workspace(torch, g, x, *c)
        outs = [torch.empty(c[0] * c[1], c[2] * c[3], device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        # first call: the one-time set-up on this device
        g._call("sana_op_linear_attention_noalloc", _vp(x.data_ptr()), *map(_i, c), _vp(outs[0].data_ptr()))
        st.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for o in outs:
            g._call("sana_op_linear_attention_noalloc", _vp(x.data_ptr()), *map(_i, c), _vp(o.data_ptr()))
        st.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0
    for o in outs:
        assert rel_err(o.float().cpu().numpy(), ref.float().cpu().numpy()) <= TOL


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch(env):
    torch, g, st = env
    S, T, heads, D = 16, 1024, 36, 32
    need = g.lib.sana_op_linear_attention_workspace(_i(S), _i(T), _i(heads), _i(D))
    assert need > 8 << 20
    out = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="exceeds the fixed"):
        # rejected before anything is launched, so the tiny buffers are never touched
        g._call("sana_op_linear_attention_noalloc", _vp(out.data_ptr()), _i(S), _i(T), _i(heads), _i(D),
                _vp(out.data_ptr()))
    assert torch.count_nonzero(out).item() == 0
