"""q35b_attn_decode_noalloc against q35_launch_attn_decode, through the C ABI.

The no-alloc entry point keeps its split partials in a fixed device array;
it must give the same attention output as the single-split entry point
within the attention tolerance used elsewhere (1e-5 of the output's
magnitude: the split merge re-associates the softmax sums), on calls made
back to back on one stream.  Named to be collected last, so it runs both in
a fresh process and after every other GPU test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def L():
    from qwen35_b200 import lib
    return lib.load()


def _case(rng, heads, kv_heads, slot):
    hd = 256
    kv_dim = kv_heads * hd
    q = torch.from_numpy(rng.standard_normal(heads * hd).astype(np.float32)).cuda()
    g = torch.from_numpy(rng.standard_normal(heads * hd).astype(np.float32)).cuda()
    K = torch.from_numpy(rng.standard_normal((slot + 1, kv_dim)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((slot + 1, kv_dim)).astype(np.float32)).cuda()
    return dict(q=q, g=g, K=K, V=V, heads=heads, gqa=heads // kv_heads, hd=hd, kv_dim=kv_dim, slot=slot)


def _ref(L, c, stream):
    out = torch.zeros(c["heads"] * c["hd"], device="cuda")
    att = torch.zeros(c["slot"] + 1, device="cuda")
    rc = L.q35_launch_attn_decode(c["q"].data_ptr(), c["g"].data_ptr(), c["K"].data_ptr(), c["V"].data_ptr(),
                                  att.data_ptr(), out.data_ptr(), c["slot"], c["heads"], c["gqa"], c["hd"],
                                  c["kv_dim"], 1.0 / 16, stream)
    assert rc == 0
    return out, att


def _noalloc(L, c, out, stream):
    return L.q35b_attn_decode_noalloc(c["q"].data_ptr(), c["g"].data_ptr(), c["K"].data_ptr(), c["V"].data_ptr(),
                                      out.data_ptr(), c["slot"], c["heads"], c["gqa"], c["hd"], c["kv_dim"],
                                      1.0 / 16, stream)


def test_noalloc_matches_attn_decode_twice(L):
    rng = np.random.default_rng(77)
    stream = torch.cuda.current_stream().cuda_stream
    # long context over many splits (8 heads / 2 kv heads), then a short one
    # with gqa 8, then a context long enough to hit the 64-split cap
    cases = [_case(rng, 8, 2, 5000), _case(rng, 16, 2, 700), _case(rng, 4, 1, 9000)]
    outs = [torch.full((c["heads"] * c["hd"],), float("nan"), device="cuda") for c in cases]
    for c, o in zip(cases, outs):        # back to back, one stream, no sync between
        assert _noalloc(L, c, o, stream) == 0
    refs = [_ref(L, c, stream) for c in cases]
    torch.cuda.synchronize()
    for (ref, _), o in zip(refs, outs):
        assert torch.isfinite(o).all()
        err = (o - ref).abs().max().item()
        assert err <= TOL * max(1.0, ref.abs().max().item()), err
    # again, after the array holds the last call's partials
    again = torch.zeros_like(outs[0])
    assert _noalloc(L, cases[0], again, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(again, outs[0])
    code = __import__("ctypes").c_int(0)
    L.q35b_get_error(__import__("ctypes").byref(code))
    assert code.value == 0


def test_noalloc_rejects_too_many_heads(L):
    """72 query heads exceed the array's 64: error 1, nothing launched.
    The buffers are sized for the request anyway."""
    rng = np.random.default_rng(5)
    c = _case(rng, 72, 9, 3)
    out = torch.zeros(72 * 256, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert _noalloc(L, c, out, stream) == 1
    torch.cuda.synchronize()
    assert not out.any()
