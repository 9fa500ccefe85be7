"""Parity at the benchmark's own sizes, on the GPU, against the CPU oracle.

* the quantized matvec over BASELINE config 2 -- every hot type on the
  1024 x 6144 and 1024 x 248320 matrices at 1, 8, 64 and 512 tokens, through
  the drop-in launcher (and the engine's padded Q6_K layout): the GPU computes
  every row, the oracle a sample of rows (both ends, every 128-row tile edge
  it lands on, random rows), compared bit for bit;
* the chunked GDN prefill at config 3's lengths (2048 and 8192 tokens, and a
  ragged 4099) against the oracle's per-token recurrence: the exact chunk
  kernel bit for bit, the WY form within 1e-4 relative L2;
* q / gate deinterleave, and the seeded synthetic generator that lets a CPU
  process rebuild the benchmark's weights.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle_lib import GEOM, TT, bp, fp, load_oracle, matvec_q, quantize_act

pytestmark = pytest.mark.gpu

S = None


@pytest.fixture(scope="module")
def L():
    from qwen35_b200 import lib
    return lib.load()


@pytest.fixture(scope="module")
def O():
    return load_oracle()


def ok(rc):
    assert rc == 0, f"cuda error {rc}"


def no_kernel_error(L):
    code = ctypes.c_int(-1)
    ok(L.q35b_get_error(ctypes.byref(code)))
    assert code.value == 0


def test_synth_fill_matches_host(L, O):
    """q35b_synth_fill == the oracle's C restatement == the numpy statement,
    bit for bit (the benchmark's CPU arm rebuilds the GPU arm's weights)"""
    from qwen35_b200 import configs
    for key, sigma, n in ((0, 0.02, 1 << 20), (2**64 - 7, 0.5, 100003), (123456789, 1.0, 4097)):
        k = configs.synth_k(sigma)
        d = torch.empty(n, dtype=torch.float32, device="cuda")
        ok(L.q35b_synth_fill(key, n, k, d.data_ptr(), S))
        got = d.cpu().numpy()
        ref = np.empty(n, np.float32)
        O.q35o_synth_fill(key, n, k, fp(ref))
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(configs.synth_normal_np(key, n, sigma).view(np.uint32), ref.view(np.uint32))
    assert abs(float(got.std()) - 1.0) < 0.05


CONFIG2_TYPES = ["Q8_0", "IQ4_NL", "Q4_K", "Q5_K", "Q6_K"]
CONFIG2_SHAPES = [(1024, 6144), (1024, 248320)]  # [in, out]
Q6_K_PADDED = 0x1000 + 14


def _device_weights(L, tt, rows, cols, key):
    """config-2 weights: N(0, 1) f32 from q35b_synth_fill, packed by the
    device encoder (bit-identical with the oracle's, test_weight_encoder_bit_exact)"""
    from qwen35_b200 import configs
    e, b = GEOM[tt]
    n = rows * cols
    f = torch.empty(n, dtype=torch.float32, device="cuda")
    ok(L.q35b_synth_fill(key, n, configs.synth_k(1.0), f.data_ptr(), S))
    wq = torch.empty(n // e * b, dtype=torch.uint8, device="cuda")
    ok(L.q35b_quantize_weight(tt, f.data_ptr(), wq.data_ptr(), n // e, S))
    del f
    return wq.view(rows, cols // e * b)


def _sample_rows(rows, rng):
    idx = set(range(min(rows, 96))) | set(range(max(0, rows - 96), rows))
    for t in range(128, rows, 128 * max(1, rows // (128 * 24))):  # tile edges
        idx |= {t - 1, t}
    idx |= set(int(i) for i in rng.choice(rows, min(rows, 600), replace=False))
    return np.array(sorted(idx), dtype=np.int64)


@pytest.mark.parametrize("tokens", [1, 8, 64, 512])
@pytest.mark.parametrize("shape", CONFIG2_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
@pytest.mark.parametrize("name", CONFIG2_TYPES)
def test_matvec_config2_grid(L, O, name, shape, tokens):
    """q35_launch_mul_mat_vec on BASELINE config 2 (lane-per-row GEMV below 16
    tokens, the tcgen05 MMQ from 16; raw 210-byte Q6_K rows on the generic
    kernel, and the engine's 224-byte Q6_K layout on the MMQ), bit-exact with
    the scalar tier on sampled rows"""
    cols, rows = shape
    tt = TT[name]
    wq = _device_weights(L, tt, rows, cols, key=tt * 1000003 + rows + 7 * cols)
    rng = np.random.default_rng(rows + tokens)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    xq = quantize_act(O, tt, x)
    dxq = torch.from_numpy(xq).cuda()
    idx = _sample_rows(rows, rng)
    ref = matvec_q(O, tt, np.ascontiguousarray(wq[torch.from_numpy(idx).cuda()].cpu().numpy()), xq, len(idx), cols,
                   tokens)
    out = torch.full((tokens, rows), float("nan"), dtype=torch.float32, device="cuda")
    ok(L.q35_launch_mul_mat_vec(wq.data_ptr(), dxq.data_ptr(), out.data_ptr(), rows, cols, tokens, tt, S))
    got = out.cpu().numpy()[:, idx]
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (name, rows, cols, tokens)
    assert not torch.isnan(out).any().item()
    if name == "Q6_K" and tokens >= 16:
        nb = cols // 256
        wp = torch.zeros((rows, nb, 224), dtype=torch.uint8, device="cuda")
        wp[:, :, :210] = wq.view(rows, nb, 210)
        out.fill_(float("nan"))
        ok(L.q35b_mul_mat_vec_multi(1, (ctypes.c_void_p * 1)(wp.data_ptr()), (ctypes.c_int * 1)(Q6_K_PADDED),
                                    (ctypes.c_longlong * 1)(rows), (ctypes.c_void_p * 1)(out.data_ptr()),
                                    (ctypes.c_longlong * 1)(rows), (ctypes.c_int * 1)(0), dxq.data_ptr(), cols,
                                    tokens, S))
        got = out.cpu().numpy()[:, idx]
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), ("Q6_K padded", rows, cols, tokens)
    no_kernel_error(L)


def _gdn_inputs(rng, heads, nk, kd, rows):
    """config-3 statistics: q / k l2-normalised (q also x 1/sqrt(kd)),
    v ~ N(0,1), beta = sigmoid(N(0,1)), gamma = exp(-softplus(N(0,1)))"""
    def l2n(x):
        return x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
    k = l2n(rng.standard_normal((rows, nk, kd))).astype(np.float32)
    q = (l2n(rng.standard_normal((rows, nk, kd))) / np.sqrt(kd)).astype(np.float32)
    v = rng.standard_normal((rows, heads, kd)).astype(np.float32)
    bet = (1 / (1 + np.exp(-rng.standard_normal((rows, heads))))).astype(np.float32)
    gam = np.exp(-np.log1p(np.exp(rng.standard_normal((rows, heads))))).astype(np.float32)
    state = (rng.standard_normal((heads, kd, kd)) * 0.1).astype(np.float32)
    return k, q, v, bet, gam, state


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("rows,heads,nk", [(2048, 16, 16), (4099, 4, 2), (8192, 2, 1)])
def test_gdn_prefill_vs_oracle_per_token(L, O, rows, heads, nk):
    """BASELINE config 3 prefill lengths: the oracle steps the recurrence one
    token at a time (src/backend_cpu.zig:1036-1056); the exact chunk kernel
    (q35_launch_gdn_step_rows_chunk) matches it bit for bit, the WY form
    (q35_launch_gdn_step_wy) within 1e-4 relative L2 in out, km, delta and
    the final state"""
    kd = 128
    rng = np.random.default_rng(rows + heads)
    k, q, v, bet, gam, state = _gdn_inputs(rng, heads, nk, kd, rows)
    rs = state.copy()
    rout, rkm, rdl = (np.zeros((rows, heads * kd), np.float32) for _ in range(3))
    for t in range(rows):
        O.q35o_gdn_step_rows(fp(rs), fp(k[t]), fp(v[t]), fp(q[t]), fp(rkm[t]), fp(rdl[t]), fp(rout[t]),
                             fp(gam[t]), fp(bet[t]), heads, nk, kd, kd)
    dk, dq, dv, db, dg = (torch.from_numpy(a).cuda() for a in (k, q, v, bet, gam))
    for fn, exact in ((L.q35_launch_gdn_step_rows_chunk, True), (L.q35_launch_gdn_step_wy, False)):
        ds = torch.from_numpy(state).cuda()
        dkm, ddl, dout = (torch.zeros((rows, heads * kd), device="cuda") for _ in range(3))
        ok(fn(ds.data_ptr(), kd * kd, dk.data_ptr(), nk * kd, dv.data_ptr(), heads * kd, dq.data_ptr(), nk * kd,
              dkm.data_ptr(), heads * kd, ddl.data_ptr(), heads * kd, dout.data_ptr(), heads * kd,
              dg.data_ptr(), heads, db.data_ptr(), heads, heads, nk, kd, kd, rows, S))
        got = [t.cpu().numpy() for t in (dout, dkm, ddl, ds)]
        for nm, a, b in zip(("out", "km", "delta", "state"), got, (rout, rkm, rdl, rs)):
            if exact:
                assert np.array_equal(a.reshape(-1).view(np.uint32), b.reshape(-1).view(np.uint32)), nm
            else:
                assert np.isfinite(a).all(), nm
                assert _rel(a, b) < 1e-4, (nm, _rel(a, b))
    no_kernel_error(L)


@pytest.mark.parametrize("tokens", [1, 5])
def test_deinterleave_qg(L, O, tokens):
    """attn_q rows [h][q_h | gate_h] -> q and gate (elementwise.zig:428-433),
    single and strided over tokens"""
    heads, hd = 8, 256
    rng = np.random.default_rng(tokens)
    src = rng.standard_normal((tokens, 2 * heads * hd)).astype(np.float32)
    rq = np.zeros((tokens, heads * hd), np.float32)
    rg = np.zeros_like(rq)
    for t in range(tokens):
        O.q35o_deinterleave_qg(fp(rq[t]), fp(rg[t]), fp(src[t]), heads, hd)
    ds = torch.from_numpy(src).cuda()
    dq = torch.full((tokens, heads * hd), float("nan"), device="cuda")
    dg = torch.full_like(dq, float("nan"))
    if tokens == 1:
        ok(L.q35_launch_deinterleave_qg(dq.data_ptr(), dg.data_ptr(), ds.data_ptr(), heads, hd, S))
    else:
        ok(L.q35_launch_deinterleave_qg_strided(dq.data_ptr(), dg.data_ptr(), ds.data_ptr(), heads, hd, tokens, S))
    assert np.array_equal(dq.cpu().numpy(), rq)
    assert np.array_equal(dg.cpu().numpy(), rg)


@pytest.mark.parametrize("heads,kvh,slot0,rows", [(8, 2, 0, 300), (8, 2, 1000, 9), (4, 4, 37, 17), (16, 4, 0, 64),
                                                  (24, 4, 5, 33), (8, 1, 2, 8), (16, 2, 4090, 12)])
def test_attn_prefill_vs_oracle_rows(L, heads, kvh, slot0, rows):
    """q35b_attn_prefill (token-tiled causal attention) against the oracle's
    per-row decode attention (src/elementwise.zig:349-372) at every row of
    the chunk: bit for bit against the oracle built with correctly rounded
    exp (the device's softmax exp), within 1e-5 of the default build; group
    sizes 1 / 2 / 4 / 6 / 8, ragged tiles, contexts past 4096"""
    Ocr = load_oracle(cr_exp=True)
    O = load_oracle()
    hd, kv_dim = 256, kvh * 256
    n = slot0 + rows
    rng = np.random.default_rng(heads * 1000 + slot0 + rows)
    q = rng.standard_normal((rows, heads * hd)).astype(np.float32)
    g = rng.standard_normal((rows, heads * hd)).astype(np.float32)
    K = rng.standard_normal((n, kv_dim)).astype(np.float32)
    V = rng.standard_normal((n, kv_dim)).astype(np.float32)
    scale = np.float32(1 / 16)
    ref_cr = np.zeros((rows, heads * hd), np.float32)
    ref = np.zeros_like(ref_cr)
    att = np.zeros(n, np.float32)
    for r in range(rows):
        Ocr.q35o_attn_decode(fp(q[r]), fp(g[r]), fp(K), fp(V), fp(att), fp(ref_cr[r]), slot0 + r, heads, heads // kvh,
                             hd, kv_dim, scale)
        O.q35o_attn_decode(fp(q[r]), fp(g[r]), fp(K), fp(V), fp(att), fp(ref[r]), slot0 + r, heads, heads // kvh, hd,
                           kv_dim, scale)
    dq, dg, dK, dV = (torch.from_numpy(a).cuda() for a in (q, g, K, V))
    out = torch.full((rows, heads * hd), float("nan"), device="cuda")
    ld = n + 3
    scores = torch.full((rows * heads * ld,), float("nan"), device="cuda")
    ok(L.q35b_attn_prefill(dq.data_ptr(), dg.data_ptr(), dK.data_ptr(), dV.data_ptr(), out.data_ptr(),
                           scores.data_ptr(), ld, slot0, rows, heads, heads // kvh, hd, kv_dim, float(scale), S))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref_cr.view(np.uint32))
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))
    no_kernel_error(L)


@pytest.mark.parametrize("rows,heads,nk", [(525, 4, 2), (100, 16, 16)])
def test_wy_tensor_core_path_vs_per_head(L, rows, heads, nk):
    """q35_launch_gdn_step_wy runs the tensor-core path (Gram matrices of
    32-token chunks, two chunks per 128-row tcgen05 kind::tf32 tile with a
    3xTF32 split, feeding the column-split recurrence) when the q / k rows
    are 16-byte aligned, and the per-head CUDA-core kernel otherwise (row
    strides of 129 floats here): two re-associations of one recurrence,
    within 1e-5 of each other"""
    kd = 128
    rng = np.random.default_rng(rows + 3 * heads)
    k, q, v, bet, gam, state = _gdn_inputs(rng, heads, nk, kd, rows)
    res = []
    for pad in (0, 1):
        ld = nk * kd + pad
        kp = np.zeros((rows, ld), np.float32)
        qp = np.zeros((rows, ld), np.float32)
        kp[:, :nk * kd] = k.reshape(rows, -1)
        qp[:, :nk * kd] = q.reshape(rows, -1)
        dk, dq, dv, db, dg = (torch.from_numpy(a).cuda() for a in (kp, qp, v, bet, gam))
        ds = torch.from_numpy(state).cuda()
        dkm, ddl, dout = (torch.zeros((rows, heads * kd), device="cuda") for _ in range(3))
        ok(L.q35_launch_gdn_step_wy(ds.data_ptr(), kd * kd, dk.data_ptr(), ld, dv.data_ptr(), heads * kd,
                                    dq.data_ptr(), ld, dkm.data_ptr(), heads * kd, ddl.data_ptr(), heads * kd,
                                    dout.data_ptr(), heads * kd, dg.data_ptr(), heads, db.data_ptr(), heads, heads,
                                    nk, kd, kd, rows, S))
        res.append([t.cpu().numpy() for t in (dout, dkm, ddl, ds)])
    for nm, a, b in zip(("out", "km", "delta", "state"), res[0], res[1]):
        assert np.isfinite(a).all(), nm
        assert _rel(a, b) < 1e-5, (nm, _rel(a, b))


def test_wy_captured_column_split_equals_per_head(L):
    """inside a stream capture the Gram buffer of the tensor-core pass cannot
    grow, so a sequence needing more than any earlier call runs the
    column-split kernel with its own A / M dots (no G), which follows the
    per-head kernel (the unaligned path) bit for bit; the graph's replay is
    compared with the per-head result and with the tensor-core path's"""
    kd, heads, nk, rows = 128, 16, 16, 4099
    rng = np.random.default_rng(4099)
    k, q, v, bet, gam, state = _gdn_inputs(rng, heads, nk, kd, rows)
    dv, db, dg = (torch.from_numpy(a).cuda() for a in (v, bet, gam))

    def call(ld, stream, rows_):
        kp = np.zeros((rows_, ld), np.float32)
        qp = np.zeros((rows_, ld), np.float32)
        kp[:, :nk * kd] = k[:rows_].reshape(rows_, -1)
        qp[:, :nk * kd] = q[:rows_].reshape(rows_, -1)
        dk, dq = torch.from_numpy(kp).cuda(), torch.from_numpy(qp).cuda()
        ds = torch.from_numpy(state).cuda()
        dkm, ddl, dout = (torch.zeros((rows_, heads * kd), device="cuda") for _ in range(3))
        torch.cuda.synchronize()

        def run():
            ok(L.q35_launch_gdn_step_wy(ds.data_ptr(), kd * kd, dk.data_ptr(), ld, dv.data_ptr(), heads * kd,
                                        dq.data_ptr(), ld, dkm.data_ptr(), heads * kd, ddl.data_ptr(), heads * kd,
                                        dout.data_ptr(), heads * kd, dg.data_ptr(), heads, db.data_ptr(), heads,
                                        heads, nk, kd, kd, rows_, stream))
        return run, (dout, dkm, ddl, ds), (dk, dq)

    run, _, _ = call(nk * kd, S, 64)  # a small aligned call: every launch attribute set
    run()
    torch.cuda.synchronize()
    run, per_head, _keep1 = call(nk * kd + 1, S, rows)
    run()
    gs = torch.cuda.Stream()
    with torch.cuda.stream(gs):
        run, captured, _keep2 = call(nk * kd, ctypes.c_void_p(gs.cuda_stream), rows)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gs):
            run()
    graph.replay()
    torch.cuda.synchronize()
    run, tensor_core, _keep3 = call(nk * kd, S, rows)
    run()
    torch.cuda.synchronize()
    for nm, a, b, c in zip(("out", "km", "delta", "state"), captured, per_head, tensor_core):
        a, b, c = (t.cpu().numpy() for t in (a, b, c))
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), nm
        assert _rel(c, b) < 1e-5, (nm, _rel(c, b))
    del graph
    no_kernel_error(L)
