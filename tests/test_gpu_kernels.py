"""Kernel parity on the GPU, through the C ABI (include/q35.h), against the
CPU oracle on the same seeded inputs.

Bars: integer / byte work (activation quantizers, weight encoders,
dequantizers), the block-ordered GEMV fold, the norms (serial sum order) and
the GDN recurrence are bit-exact; attention's softmax / P.V reductions and
the double-evaluated transcendentals are within 1e-5 relative.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle_lib import (TT, GEOM, ROOT, act_row_bytes, bp, dequant, fp, load_oracle, matvec_q, quantize_act,
                        quantize_weight, row_bytes)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from qwen35_b200 import lib
    return lib.load()


@pytest.fixture(scope="module")
def O():
    return load_oracle()


_KEEP = []


@pytest.fixture(autouse=True)
def _keepalive():
    """device copies made inline (dev(x).data_ptr() as a call argument) must
    outlive the asynchronous kernel that reads them; free them after the test"""
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


S = None  # legacy default stream


def ok(rc):
    assert rc == 0, f"cuda error {rc}"


def assert_no_kernel_error(L):
    code = ctypes.c_int(-1)
    ok(L.q35b_get_error(ctypes.byref(code)))
    assert code.value == 0


TYPES = ["Q8_0", "IQ4_NL", "Q4_K", "Q5_K", "Q6_K"]


def test_quantize_q8_0_bit_exact(L, O):
    rng = np.random.default_rng(0)
    for scale in (1e-6, 1e-3, 1.0, 300.0):
        x = (rng.standard_normal(32 * 257) * scale).astype(np.float32)
        x[:32] = 0.0
        x[32:64] = 7.0
        ref = quantize_act(O, TT["Q8_0"], x)[0]
        xd = dev(x)
        out = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
        ok(L.q35_launch_quantize_q8_0(xd.data_ptr(), out.data_ptr(), x.size // 32, S))
        assert np.array_equal(host(out), ref)


def test_quantize_q8_K_bit_exact(L, O):
    rng = np.random.default_rng(1)
    for scale in (1e-5, 1.0, 1e4):
        x = (rng.standard_normal(256 * 37) * scale).astype(np.float32)
        x[:256] = 0.0
        ref = quantize_act(O, TT["Q4_K"], x)[0]
        xd = dev(x)
        out = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
        ok(L.q35_launch_quantize_q8_K(xd.data_ptr(), out.data_ptr(), x.size // 256, S))
        assert np.array_equal(host(out), ref)


@pytest.mark.parametrize("name", TYPES)
def test_weight_encoder_bit_exact(L, O, name):
    tt = TT[name]
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((64, 1024)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0
    ref = quantize_weight(O, tt, w)
    e, b = GEOM[tt]
    out = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
    ok(L.q35b_quantize_weight(tt, dev(w).data_ptr(), out.data_ptr(), w.size // e, S))
    assert np.array_equal(host(out).reshape(ref.shape), ref)


@pytest.mark.parametrize("name", TYPES)
def test_dequant_row_bit_exact(L, O, name):
    tt = TT[name]
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((4, 1024)) * 0.05).astype(np.float32)
    wq = quantize_weight(O, tt, w)
    ref = dequant(O, tt, wq, 1024)
    wd = dev(wq)
    for r in range(4):
        out = torch.zeros(1024, dtype=torch.float32, device="cuda")
        ok(L.q35_launch_dequantize_row(tt, wd[r].data_ptr(), out.data_ptr(), 1024, S))
        assert np.array_equal(host(out).view(np.uint32), ref[r].view(np.uint32))


def _gemv_case(L, O, name, rows, cols, tokens, seed):
    tt = TT[name]
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    wq = quantize_weight(O, tt, w)
    xq = quantize_act(O, tt, x)
    ref = matvec_q(O, tt, wq, xq, rows, cols, tokens)
    out = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    ok(L.q35_launch_mul_mat_vec(dev(wq).data_ptr(), dev(xq).data_ptr(), out.data_ptr(), rows, cols, tokens, tt, S))
    got = host(out)
    return got, ref


@pytest.mark.parametrize("name", TYPES)
@pytest.mark.parametrize("tokens", [1, 3, 8, 13])
def test_gemv_bit_exact(L, O, name, tokens):
    """out[t*rows+r] == the reference scalar tier's strict block-order fold"""
    # lane-per-row kernel: columns split over 8, 4, 2 and 1 warps, and tall
    # matrices (4 row groups per CTA);
    # cols % 256 != 0 takes the block-splitting kernel
    shapes = [(300, 1024), (64, 3584), (129, 2048), (10000, 512), (19000, 256), (40000, 256)]
    if GEOM[TT[name]][0] == 32:
        shapes.append((77, 2080))
    for rows, cols in shapes:
        got, ref = _gemv_case(L, O, name, rows, cols, tokens, seed=rows + tokens)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (name, rows, cols, tokens)
    assert_no_kernel_error(L)


@pytest.mark.parametrize("name", ["Q8_0", "IQ4_NL", "Q4_K", "Q5_K"])
@pytest.mark.parametrize("tokens", [16, 37, 64, 100])
def test_mmq_tensor_core_bit_exact(L, O, name, tokens):
    """>= 16 tokens of Q8_0 / IQ4_NL / Q4_K / Q5_K go to the tcgen05 MMQ: the
    int8 (sub-)block dots on the tensor core, scales, mins and the f32 fold in
    block order on the CUDA cores -- bit-exact with the reference scalar tier
    like the decode GEMV"""
    # token tiles of 64 / 32 / 16 by how many row tiles there are (Q8_0 /
    # IQ4_NL: 16 for the short matrices, 32 for 100 row tiles at 37 / 64
    # tokens, 64 for 149 row tiles; K-quants: 32 or 64)
    for rows, cols in [(300, 1024), (129, 2048), (1000, 768), (128, 256), (12800, 256), (19000, 256)]:
        got, ref = _gemv_case(L, O, name, rows, cols, tokens, seed=rows + 7 * tokens)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (name, rows, cols, tokens)
    assert_no_kernel_error(L)


Q6_K_PADDED = 0x1000 + 14  # Q6_K in 224-byte blocks (210 bytes + 14 of padding): 16-byte rows


def _pad_q6k(wq, rows, cols):
    nb = cols // 256
    out = np.zeros((rows, nb, 224), dtype=np.uint8)
    out[:, :, :210] = wq.reshape(rows, nb, 210)
    return out.reshape(rows, nb * 224)


@pytest.mark.parametrize("tokens", [16, 37, 64, 100])
def test_mmq_q6_k_bit_exact(L, O, tokens):
    """>= 16 tokens of Q6_K (224-byte blocks, the engine's load-time layout)
    go to the tcgen05 MMQ: scales folded into the weights, split into two
    int8 digits, isum = 64*H + L from two TMEM accumulators per block, the f32
    step (d*dy)*isum in block order -- bit-exact with the scalar tier"""
    tt = TT["Q6_K"]
    for rows, cols in [(300, 1024), (129, 2560), (128, 256), (12800, 256), (19000, 512)]:
        rng = np.random.default_rng(rows + 7 * tokens)
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        x = rng.standard_normal((tokens, cols)).astype(np.float32)
        wq = quantize_weight(O, tt, w)
        xq = quantize_act(O, tt, x)
        ref = matvec_q(O, tt, wq, xq, rows, cols, tokens)
        out = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
        wp = dev(_pad_q6k(wq, rows, cols))
        ok(L.q35b_mul_mat_vec_multi(1, (ctypes.c_void_p * 1)(wp.data_ptr()), (ctypes.c_int * 1)(Q6_K_PADDED),
                                    (ctypes.c_longlong * 1)(rows), (ctypes.c_void_p * 1)(out.data_ptr()),
                                    (ctypes.c_longlong * 1)(rows), (ctypes.c_int * 1)(0), dev(xq).data_ptr(),
                                    cols, tokens, S))
        got = host(out)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (rows, cols, tokens)
    assert_no_kernel_error(L)


@pytest.mark.parametrize("name", ["Q4_K", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("tokens", [16, 25, 32, 64])
def test_mmq_split_k_bit_exact(L, O, name, tokens):
    """q35b_mul_mat_vec_multi_ws: a matrix with few row tiles splits K over
    CTAs (up to 32 tokens), each block's f32 term goes to the workspace and a
    second kernel adds them in block order -- bit-exact with the scalar tier,
    write and residual mode, and a workspace reused across calls; at 64
    tokens the workspace is left unused and the result is the same"""
    tt = TT[name]
    code = Q6_K_PADDED if name == "Q6_K" else tt
    for rows, cols, mode in [(300, 4096, 0), (128, 2048, 1), (640, 9216, 1)]:
        rng = np.random.default_rng(rows + cols + tokens)
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        x = rng.standard_normal((tokens, cols)).astype(np.float32)
        wq = quantize_weight(O, tt, w)
        xq = quantize_act(O, tt, x)
        ref = matvec_q(O, tt, wq, xq, rows, cols, tokens)
        base = rng.standard_normal((tokens, rows)).astype(np.float32)
        if mode:
            ref = (base + ref).astype(np.float32)
        wd = dev(_pad_q6k(wq, rows, cols) if name == "Q6_K" else wq)
        work = torch.full(((cols // 256) * tokens * rows,), float("nan"), dtype=torch.float32, device="cuda")
        for _ in range(2):
            out = dev(base) if mode else torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
            ok(L.q35b_mul_mat_vec_multi_ws(1, (ctypes.c_void_p * 1)(wd.data_ptr()), (ctypes.c_int * 1)(code),
                                           (ctypes.c_longlong * 1)(rows), (ctypes.c_void_p * 1)(out.data_ptr()),
                                           (ctypes.c_longlong * 1)(rows), (ctypes.c_int * 1)(mode),
                                           dev(xq).data_ptr(), cols, tokens, work.data_ptr(), work.numel() * 4, S))
            got = host(out)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (name, rows, cols, tokens, mode)
        # the split ran and wrote its terms (32 tokens or fewer), or was skipped
        assert torch.isnan(work).all().item() == (tokens > 32)
    assert_no_kernel_error(L)


def test_mmq_q6_k_mixed_segments_residual(L, O):
    """Q4_K and padded Q6_K matrices in one MMQ launch, the Q6_K one in
    residual mode"""
    rng = np.random.default_rng(21)
    cols, tokens = 512, 40
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    xq = quantize_act(O, TT["Q4_K"], x)
    wk = quantize_weight(O, TT["Q4_K"], (rng.standard_normal((200, cols)) * 0.02).astype(np.float32))
    w6 = quantize_weight(O, TT["Q6_K"], (rng.standard_normal((150, cols)) * 0.02).astype(np.float32))
    base = rng.standard_normal((tokens, 150)).astype(np.float32)
    ref_k = matvec_q(O, TT["Q4_K"], wk, xq, 200, cols, tokens)
    ref_6 = (base + matvec_q(O, TT["Q6_K"], w6, xq, 150, cols, tokens)).astype(np.float32)
    ok_, o6 = torch.zeros((tokens, 200), dtype=torch.float32, device="cuda"), dev(base)
    ws = [dev(wk), dev(_pad_q6k(w6, 150, cols))]
    ok(L.q35b_mul_mat_vec_multi(2, (ctypes.c_void_p * 2)(*[w.data_ptr() for w in ws]),
                                (ctypes.c_int * 2)(TT["Q4_K"], Q6_K_PADDED), (ctypes.c_longlong * 2)(200, 150),
                                (ctypes.c_void_p * 2)(ok_.data_ptr(), o6.data_ptr()), (ctypes.c_longlong * 2)(200, 150),
                                (ctypes.c_int * 2)(0, 1), dev(xq).data_ptr(), cols, tokens, S))
    assert np.array_equal(host(ok_).view(np.uint32), ref_k.view(np.uint32))
    assert np.array_equal(host(o6).view(np.uint32), ref_6.view(np.uint32))
    assert_no_kernel_error(L)


def test_mmq_multi_and_residual(L, O):
    """the MMQ over mixed IQ4_NL / Q8_0 matrices in one launch, residual mode"""
    rng = np.random.default_rng(14)
    cols, tokens = 512, 40
    shapes = [(TT["IQ4_NL"], 300), (TT["Q8_0"], 16), (TT["Q8_0"], 130)]
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    xq = quantize_act(O, TT["Q8_0"], x)
    ws, refs, outs = [], [], []
    base = rng.standard_normal((tokens, 130)).astype(np.float32)
    for i, (tt, rows) in enumerate(shapes):
        wq = quantize_weight(O, tt, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
        ws.append(dev(wq))
        r = matvec_q(O, tt, wq, xq, rows, cols, tokens)
        if i == 2:
            r = (base + r).astype(np.float32)
            outs.append(dev(base))
        else:
            outs.append(torch.zeros((tokens, rows), dtype=torch.float32, device="cuda"))
        refs.append(r)
    n = 3
    W = (ctypes.c_void_p * n)(*[w.data_ptr() for w in ws])
    T = (ctypes.c_int * n)(*[s[0] for s in shapes])
    R = (ctypes.c_longlong * n)(*[s[1] for s in shapes])
    Op = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    LD = (ctypes.c_longlong * n)(*[s[1] for s in shapes])
    M = (ctypes.c_int * n)(0, 0, 1)
    ok(L.q35b_mul_mat_vec_multi(n, W, T, R, Op, LD, M, dev(xq).data_ptr(), cols, tokens, S))
    for o, r in zip(outs, refs):
        assert np.array_equal(host(o).view(np.uint32), r.view(np.uint32))
    assert_no_kernel_error(L)


def test_gemv_golden_rows(L, O):
    """the reference's udtest rows (96 x 256) through the device GEMV"""
    gold = os.path.join(ROOT, "tests", "golden", "udtest")
    ax = np.fromfile(os.path.join(gold, "A_x.f32"), dtype=np.float32)
    for name, rb in [("Q4_K", 144), ("Q5_K", 176), ("Q6_K", 210), ("IQ4_NL", 144), ("Q4_0", 144)]:
        tt = TT[name]
        rows = np.fromfile(os.path.join(gold, f"{name}.bin"), dtype=np.uint8).reshape(-1, rb)
        exp = np.fromfile(os.path.join(gold, f"{name}_expected.f32"), dtype=np.float32)
        xq = quantize_act(O, tt, ax)
        ref = matvec_q(O, tt, rows, xq, 96, 256, 1)[0]
        out = torch.zeros(96, dtype=torch.float32, device="cuda")
        ok(L.q35_launch_mul_mat_vec(dev(rows).data_ptr(), dev(xq).data_ptr(), out.data_ptr(), 96, 256, 1, tt, S))
        got = host(out)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name
        # and close to the f32 known answers (activation quantization error only)
        rel = np.abs(got - exp) / np.maximum(np.abs(exp), 1)
        assert rel.max() < 5e-2, (name, rel.max())


@pytest.mark.parametrize("name", TYPES)
def test_gemv_unaligned_weight_base(L, O, name):
    """a matrix starting 2 bytes past a 16-byte boundary (GGUF blocks are only
    2-byte aligned) is streamed correctly, head/tail bytes included"""
    tt = TT[name]
    rng = np.random.default_rng(9)
    rows, cols = 37, 768
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    wq = quantize_weight(O, tt, w)
    xq = quantize_act(O, tt, rng.standard_normal(cols).astype(np.float32))
    ref = matvec_q(O, tt, wq, xq, rows, cols, 1)[0]
    buf = torch.zeros(wq.size + 64, dtype=torch.uint8, device="cuda")
    buf[2:2 + wq.size] = dev(wq.reshape(-1))
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    ok(L.q35_launch_mul_mat_vec(buf.data_ptr() + 2, dev(xq).data_ptr(), out.data_ptr(), rows, cols, 1, tt, S))
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))


def test_gemv_multi_and_residual(L, O):
    """one launch over 3 matrices; mode 1 adds into the output (x += W y),
    bit-exact with the separate matvec then addResid"""
    rng = np.random.default_rng(4)
    cols, tokens = 1024, 2
    shapes = [(TT["IQ4_NL"], 512), (TT["Q8_0"], 16), (TT["Q8_0"], 48)]
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    xq = quantize_act(O, TT["Q8_0"], x)
    ws, refs, outs = [], [], []
    base = rng.standard_normal((tokens, 48)).astype(np.float32)
    for i, (tt, rows) in enumerate(shapes):
        wq = quantize_weight(O, tt, (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
        ws.append(dev(wq))
        r = matvec_q(O, tt, wq, xq, rows, cols, tokens)
        if i == 2:
            r = (base + r).astype(np.float32)
            outs.append(dev(base))
        else:
            outs.append(torch.zeros((tokens, rows), dtype=torch.float32, device="cuda"))
        refs.append(r)
    n = 3
    W = (ctypes.c_void_p * n)(*[w.data_ptr() for w in ws])
    T = (ctypes.c_int * n)(*[s[0] for s in shapes])
    R = (ctypes.c_longlong * n)(*[s[1] for s in shapes])
    Op = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    LD = (ctypes.c_longlong * n)(*[s[1] for s in shapes])
    M = (ctypes.c_int * n)(0, 0, 1)
    ok(L.q35b_mul_mat_vec_multi(n, W, T, R, Op, LD, M, dev(xq).data_ptr(), cols, tokens, S))
    for o, r in zip(outs, refs):
        assert np.array_equal(host(o).view(np.uint32), r.view(np.uint32))


def test_gemv_rejects_mixed_families(L):
    n = 2
    W = (ctypes.c_void_p * n)(16, 16)
    T = (ctypes.c_int * n)(TT["Q8_0"], TT["Q4_K"])
    R = (ctypes.c_longlong * n)(4, 4)
    Op = (ctypes.c_void_p * n)(16, 16)
    LD = (ctypes.c_longlong * n)(4, 4)
    assert L.q35b_mul_mat_vec_multi(n, W, T, R, Op, LD, None, 16, 256, 1, S) == 1


def test_gdn_step_rows_bit_exact(L, O):
    """q35_launch_gdn_step_rows == CPU gdnFused per head (h % nk k-head map)"""
    rng = np.random.default_rng(5)
    heads, nk, kd = 6, 3, 128
    state = (rng.standard_normal((heads, kd, kd)) * 0.1).astype(np.float32)
    k = rng.standard_normal(nk * kd).astype(np.float32)
    q = rng.standard_normal(nk * kd).astype(np.float32)
    v = rng.standard_normal(heads * kd).astype(np.float32)
    gamma = rng.uniform(0.5, 1.0, heads).astype(np.float32)
    beta = rng.uniform(0.0, 1.0, heads).astype(np.float32)
    rs, rkm, rdl, rout = state.copy(), np.zeros(heads * kd, np.float32), np.zeros(heads * kd, np.float32), \
        np.zeros(heads * kd, np.float32)
    O.q35o_gdn_step_rows(fp(rs), fp(k), fp(v), fp(q), fp(rkm), fp(rdl), fp(rout), fp(gamma), fp(beta), heads, nk,
                         kd, kd)
    ds, dkm, ddl, dout = dev(state), *[torch.zeros(heads * kd, device="cuda") for _ in range(3)]
    ok(L.q35_launch_gdn_step_rows(ds.data_ptr(), kd * kd, dev(k).data_ptr(), kd, dev(v).data_ptr(), kd,
                                  dev(q).data_ptr(), kd, dkm.data_ptr(), ddl.data_ptr(), dout.data_ptr(),
                                  dev(gamma).data_ptr(), dev(beta).data_ptr(), heads, nk, kd, kd, S))
    for a, b in [(ds, rs), (dkm, rkm), (ddl, rdl), (dout, rout)]:
        assert np.array_equal(host(a).reshape(-1).view(np.uint32), b.reshape(-1).view(np.uint32))


def test_gdn_chunk_equals_rows(L, O):
    """gdnStepRowsChunk == rows x gdnStepRows, bit-identical
    (src/chunk_slot_tests.zig:247), incl. recurrence dependence"""
    rng = np.random.default_rng(6)
    heads, nk, kd, rows = 4, 2, 128, 5
    conv_dim = 2 * nk * kd + heads * kd
    state = (rng.standard_normal((heads, kd, kd)) * 0.1).astype(np.float32)
    qkv = rng.standard_normal((rows, conv_dim)).astype(np.float32)
    gam = rng.uniform(0.5, 1.0, (rows, heads)).astype(np.float32)
    bet = rng.uniform(0.0, 1.0, (rows, heads)).astype(np.float32)
    rs = state.copy()
    rout = np.zeros((rows, heads * kd), np.float32)
    km = np.zeros(heads * kd, np.float32)
    dl = np.zeros(heads * kd, np.float32)
    for t in range(rows):
        row = qkv[t]
        O.q35o_gdn_step_rows(fp(rs), fp(row[nk * kd:]), fp(row[2 * nk * kd:]), fp(row), fp(km), fp(dl),
                             fp(rout[t]), fp(gam[t]), fp(bet[t]), heads, nk, kd, kd)
    ds, dq = dev(state), dev(qkv)
    dkm = torch.zeros((rows, heads * kd), device="cuda")
    ddl = torch.zeros_like(dkm)
    dout = torch.zeros_like(dkm)
    base = dq.data_ptr()
    ok(L.q35_launch_gdn_step_rows_chunk(ds.data_ptr(), kd * kd, base + 4 * nk * kd, conv_dim,
                                        base + 4 * 2 * nk * kd, conv_dim, base, conv_dim, dkm.data_ptr(),
                                        heads * kd, ddl.data_ptr(), heads * kd, dout.data_ptr(), heads * kd,
                                        dev(gam).data_ptr(), heads, dev(bet).data_ptr(), heads, heads, nk, kd, kd,
                                        rows, S))
    assert np.array_equal(host(ds).view(np.uint32), rs.view(np.uint32))
    assert np.array_equal(host(dout).view(np.uint32), rout.view(np.uint32))


def _wy_inputs(rng, heads, nk, kd, rows, decay_scale=1.0):
    """config-3 statistics: q / k l2-normalised (q also x 1/sqrt(kd)),
    v ~ N(0,1), beta = sigmoid(N(0,1)), gamma = exp(-softplus(N(0,1)))"""
    def l2n(x):
        return x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
    k = l2n(rng.standard_normal((rows, nk, kd))).astype(np.float32)
    q = (l2n(rng.standard_normal((rows, nk, kd))) / np.sqrt(kd)).astype(np.float32)
    v = rng.standard_normal((rows, heads, kd)).astype(np.float32)
    bet = (1 / (1 + np.exp(-rng.standard_normal((rows, heads))))).astype(np.float32)
    gam = np.exp(-decay_scale * np.log1p(np.exp(rng.standard_normal((rows, heads))))).astype(np.float32)
    state = (rng.standard_normal((heads, kd, kd)) * 0.1).astype(np.float32)
    return k, q, v, bet, gam, state


@pytest.mark.parametrize("rows,decay_scale", [(525, 1.0), (33, 1.0), (7, 1.0), (96, 0.02), (64, 60.0)])
def test_gdn_wy_matches_per_token(L, rows, decay_scale):
    """q35_launch_gdn_step_wy (WY form, 32-token blocks) against the per-token
    chunk kernel on the same inputs: out, km, delta and the final state
    within 1e-4 relative L2 (the reference records 1.6e-7..1.8e-6 for its WY
    kernel at rows = 525, api.h:290-296).  Covers a ragged last block, fewer
    rows than one block, slow decay (gamma ~ 0.99) and decay strong enough
    that gamma underflows toward 0."""
    rng = np.random.default_rng(rows)
    heads, nk, kd = 4, 2, 128
    k, q, v, bet, gam, state = _wy_inputs(rng, heads, nk, kd, rows, decay_scale)
    dk, dq, dv, db, dg = dev(k), dev(q), dev(v), dev(bet), dev(gam)
    outs = []
    for fn in (L.q35_launch_gdn_step_rows_chunk, L.q35_launch_gdn_step_wy):
        ds = dev(state)
        dkm, ddl, dout = (torch.zeros((rows, heads * kd), device="cuda") for _ in range(3))
        ok(fn(ds.data_ptr(), kd * kd, dk.data_ptr(), nk * kd, dv.data_ptr(), heads * kd, dq.data_ptr(), nk * kd,
              dkm.data_ptr(), heads * kd, ddl.data_ptr(), heads * kd, dout.data_ptr(), heads * kd,
              dg.data_ptr(), heads, db.data_ptr(), heads, heads, nk, kd, kd, rows, S))
        outs.append([host(t).astype(np.float64) for t in (dout, dkm, ddl, ds)])
    for name, a, b in zip(("out", "km", "delta", "state"), outs[1], outs[0]):
        assert np.isfinite(a).all(), name
        rel = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert rel < 1e-4, (name, rel)


def test_conv_gamma_exact_paths(L, O):
    rng = np.random.default_rng(7)
    n, tokens = 768, 3
    conv = rng.standard_normal(n * 3).astype(np.float32)
    y = rng.standard_normal((tokens, n)).astype(np.float32)
    w = rng.standard_normal(n * 4).astype(np.float32)
    rc, ry = conv.copy(), y.copy()
    for t in range(tokens):
        O.q35o_conv_step(fp(rc), fp(ry[t]), fp(w), n)
    dc, dy = dev(conv), dev(y)
    ok(L.q35_launch_conv_step_rows(dc.data_ptr(), dy.data_ptr(), dev(w).data_ptr(), n, tokens, n, S))
    assert np.array_equal(host(dc), rc)
    assert np.abs(host(dy) - ry).max() <= 1e-6 * np.abs(ry).max()
    nv = 16
    a = rng.standard_normal(nv).astype(np.float32) * 3
    b = rng.standard_normal(nv).astype(np.float32)
    sa = -np.exp(rng.uniform(-1, 1, nv)).astype(np.float32)
    dt = rng.standard_normal(nv).astype(np.float32)
    rb, rg = b.copy(), np.zeros(nv, np.float32)
    O.q35o_gdn_gamma(fp(a), fp(rb), fp(sa), fp(dt), fp(rg), nv)
    db, dg = dev(b), torch.zeros(nv, device="cuda")
    ok(L.q35_launch_gdn_gamma(dev(a).data_ptr(), db.data_ptr(), dev(sa).data_ptr(), dev(dt).data_ptr(),
                              dg.data_ptr(), nv, S))
    assert np.abs(host(db) - rb).max() <= 1e-6
    assert np.abs(host(dg) - rg).max() <= 1e-6


def test_norms_and_activations(L, O):
    rng = np.random.default_rng(8)
    rows, n = 5, 1024
    x = rng.standard_normal((rows, n)).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    ref = np.zeros_like(x)
    O.q35o_rmsnorm_rows(fp(ref), fp(x), fp(w), rows, n, 1e-6)
    out = torch.zeros_like(dev(x))
    ok(L.q35_launch_rmsnorm(out.data_ptr(), dev(x).data_ptr(), dev(w).data_ptr(), rows, n, 1e-6, S))
    # sums of squares are taken in the CPU's serial order: bit-exact
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))
    nk, kd = 4, 128
    v = rng.standard_normal(3 * nk * kd).astype(np.float32)
    rv = v.copy()
    O.q35o_l2norm_qk_scale(fp(rv), nk, kd, nk * kd, np.float32(1 / np.sqrt(128)))
    dv = dev(v)
    ok(L.q35_launch_l2norm_qk_scale(dv.data_ptr(), nk, kd, nk * kd, 1e-6, float(np.float32(1 / np.sqrt(128))), S))
    assert np.array_equal(host(dv).view(np.uint32), rv.view(np.uint32))
    g = rng.standard_normal(4096).astype(np.float32) * 4
    u = rng.standard_normal(4096).astype(np.float32)
    rg = g.copy()
    O.q35o_swiglu(fp(rg), fp(u), 4096)
    dg = dev(g)
    ok(L.q35_launch_swiglu(dg.data_ptr(), dev(u).data_ptr(), 4096, S))
    assert np.abs(host(dg) - rg).max() <= 1e-6 * np.abs(rg).max()
    sm = rng.standard_normal(3000).astype(np.float32) * 5
    rsm = sm.copy()
    O.q35o_softmax(fp(rsm), 3000)
    dsm = dev(sm)
    ok(L.q35_launch_softmax(dsm.data_ptr(), 3000, S))
    assert np.abs(host(dsm) - rsm).max() <= 1e-6


def test_rmsnorm_segmented_sum_edge_rows(L, O):
    """The CTA-wide sum of squares runs one chain segment per warp from
    candidate start values around a double-precision estimate and stitches
    them; rows whose f32 chain drifts far from the exact prefix (small
    squares absorbed by a huge first one), all-zero rows, growing and tiny
    magnitudes must still give the serial order's bits (the stitch falls
    back to a serial pass over a segment whose window misses)."""
    rng = np.random.default_rng(21)
    n = 1024
    rows = []
    r = np.full(n, 1e14, np.float32)
    r[0] = 1e18
    rows.append(r)                                                   # absorbed: window misses
    rows.append(np.zeros(n, np.float32))                             # stays at +0
    rows.append((np.geomspace(1e-3, 1e3, n) * rng.choice([-1, 1], n)).astype(np.float32))
    rows.append((rng.standard_normal(n) * 1e-20).astype(np.float32))  # subnormal squares
    r = rng.standard_normal(n).astype(np.float32)
    r[::7] *= 3e4
    rows.append(r)
    for cols in (1024, 1000, 2560, 37):
        x = np.stack([np.resize(rr, cols) for rr in rows]).astype(np.float32)
        w = rng.standard_normal(cols).astype(np.float32)
        ref = np.zeros_like(x)
        O.q35o_rmsnorm_rows(fp(ref), fp(x), fp(w), x.shape[0], cols, 1e-6)
        out = torch.zeros_like(dev(x))
        ok(L.q35_launch_rmsnorm(out.data_ptr(), dev(x).data_ptr(), dev(w).data_ptr(), x.shape[0], cols, 1e-6, S))
        assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32)), cols


def test_rope_and_argmax(L, O):
    rng = np.random.default_rng(10)
    heads, hd = 8, 256
    for pos in (0, 1, 37, 4095):
        x = rng.standard_normal(heads * hd).astype(np.float32)
        rx = x.copy()
        O.q35o_rope64_rows(fp(rx), 1, heads, hd, pos, 1e7)
        dx = dev(x)
        ok(L.q35_launch_rope64(dx.data_ptr(), heads, hd, pos, 1e7, S))
        assert np.abs(host(dx) - rx).max() <= 1e-5, pos
    x = rng.standard_normal(248320).astype(np.float32)
    x[1000] = x[200000] = 9.0  # tie: first index wins
    o = torch.zeros(1, dtype=torch.int32, device="cuda")
    ok(L.q35_launch_argmax(dev(x).data_ptr(), x.size, o.data_ptr(), S))
    assert int(host(o)[0]) == 1000 == O.q35o_argmax(fp(x), x.size)


@pytest.mark.parametrize("slot", [0, 5, 300, 1100, 4095, 9000])
def test_attn_decode(L, O, slot):
    rng = np.random.default_rng(slot)
    heads, kvh, hd = 8, 2, 256
    kv_dim = kvh * hd
    q = rng.standard_normal(heads * hd).astype(np.float32)
    g = rng.standard_normal(heads * hd).astype(np.float32)
    K = rng.standard_normal((slot + 1, kv_dim)).astype(np.float32)
    V = rng.standard_normal((slot + 1, kv_dim)).astype(np.float32)
    att = np.zeros(slot + 1, np.float32)
    ref = np.zeros(heads * hd, np.float32)
    scale = np.float32(1 / 16)
    O.q35o_attn_decode(fp(q), fp(g), fp(K), fp(V), fp(att), fp(ref), slot, heads, heads // kvh, hd, kv_dim, scale)
    out = torch.zeros(heads * hd, device="cuda")
    datt = torch.zeros(slot + 1, device="cuda")
    ok(L.q35_launch_attn_decode(dev(q).data_ptr(), dev(g).data_ptr(), dev(K).data_ptr(), dev(V).data_ptr(),
                                datt.data_ptr(), out.data_ptr(), slot, heads, heads // kvh, hd, kv_dim,
                                float(scale), S))
    assert np.abs(host(out) - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
    # device-slot twin
    ds = torch.tensor([slot], dtype=torch.int32, device="cuda")
    out2 = torch.zeros_like(out)
    ok(L.q35_launch_attn_decode_dyn(dev(q).data_ptr(), dev(g).data_ptr(), dev(K).data_ptr(), dev(V).data_ptr(),
                                    datt.data_ptr(), out2.data_ptr(), ds.data_ptr(), heads, heads // kvh, hd,
                                    kv_dim, float(scale), S))
    assert torch.equal(out, out2)


def test_attn_chunk_equals_decode_rows(L):
    """attnChunk == k x attnDecode (src/chunk_slot_tests.zig:40)"""
    rng = np.random.default_rng(11)
    heads, kvh, hd, slot0, rows = 4, 1, 256, 20, 6
    kv_dim = kvh * hd
    q = dev(rng.standard_normal((rows, heads * hd)).astype(np.float32))
    g = dev(rng.standard_normal((rows, heads * hd)).astype(np.float32))
    K = dev(rng.standard_normal((slot0 + rows, kv_dim)).astype(np.float32))
    V = dev(rng.standard_normal((slot0 + rows, kv_dim)).astype(np.float32))
    out = torch.zeros((rows, heads * hd), device="cuda")
    ok(L.q35_launch_attn_chunk(q.data_ptr(), g.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), slot0, rows,
                               heads, heads // kvh, hd, kv_dim, 1 / 16, S))
    for r in range(rows):
        o = torch.zeros(heads * hd, device="cuda")
        att = torch.zeros(slot0 + rows, device="cuda")
        ok(L.q35_launch_attn_decode(q[r].data_ptr(), g[r].data_ptr(), K.data_ptr(), V.data_ptr(), att.data_ptr(),
                                    o.data_ptr(), slot0 + r, heads, heads // kvh, hd, kv_dim, 1 / 16, S))
        assert torch.equal(o, out[r])
    assert_no_kernel_error(L)


def test_bounded_wait_ends_with_an_error_not_a_hang(L):
    """failure detection without a GPU fault: a kernel whose wait is never
    satisfied gives up after its limit, records a site code, and the context
    keeps working"""
    import time
    assert_no_kernel_error(L)
    t0 = time.time()
    ok(L.q35b_selftest_wait(100, S))
    assert time.time() - t0 < 5.0
    code = ctypes.c_int(0)
    ok(L.q35b_get_error(ctypes.byref(code)))
    assert code.value == 150
    # the context is still usable: a GEMV runs and is exact
    got, ref = _gemv_case(L, load_oracle(), "Q8_0", 64, 512, 1, seed=3)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert_no_kernel_error(L)


LEGACY = ["Q4_0", "Q4_1", "Q5_0", "Q5_1"]


@pytest.mark.parametrize("name", LEGACY)
def test_legacy_encoder_and_dequant_bit_exact(L, O, name):
    """Q4_0 / Q4_1 / Q5_0 / Q5_1: the device weight encoder gives the oracle's
    bytes, and the device dequantizer its values (GGUF nibble layout)"""
    tt = TT[name]
    rng = np.random.default_rng(31)
    w = (rng.standard_normal((16, 1024)) * 0.05).astype(np.float32)
    w[0, :64] = 0.0
    w[1, :32] = 3.0
    ref = quantize_weight(O, tt, w)
    e, b = GEOM[tt]
    out = torch.zeros(ref.size, dtype=torch.uint8, device="cuda")
    ok(L.q35b_quantize_weight(tt, dev(w).data_ptr(), out.data_ptr(), w.size // e, S))
    assert np.array_equal(host(out).reshape(ref.shape), ref)
    deq = dequant(O, tt, ref, 1024)
    wd = dev(ref)
    for r in range(16):
        o = torch.zeros(1024, dtype=torch.float32, device="cuda")
        ok(L.q35_launch_dequantize_row(tt, wd[r].data_ptr(), o.data_ptr(), 1024, S))
        assert np.array_equal(host(o).view(np.uint32), deq[r].view(np.uint32))
    # the encoding is close to the input (a round trip of the format)
    assert np.abs(deq - w).max() <= np.abs(w).max() * (0.15 if name.startswith("Q4") else 0.08)


@pytest.mark.parametrize("name", LEGACY)
@pytest.mark.parametrize("tokens", [1, 3, 8, 16, 37])
def test_legacy_gemv_bit_exact(L, O, name, tokens):
    """Q4_0 / Q4_1 / Q5_0 / Q5_1 through q35_launch_mul_mat_vec: the
    lane-per-row kernel (cols % 256 == 0, passes of up to 8 tokens; the MMQ
    declines these types) and the block-splitting kernel (cols % 256 != 0,
    unaligned base) against the reference scalar tier's fold, bit for bit"""
    for rows, cols in [(300, 1024), (64, 3584), (129, 2048), (10000, 512), (77, 2080)]:
        got, ref = _gemv_case(L, O, name, rows, cols, tokens, seed=rows + 3 * tokens)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (name, rows, cols, tokens)
    assert_no_kernel_error(L)
