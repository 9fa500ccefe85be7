"""Pin the CPU oracle before trusting it.

1. Known-answer vectors from the reference (testdata/udtest, checked by
   src/quant_dequant.zig:1126-1205 at 1e-3): dequant(row) . A_x == expected.
2. The reference's hand-computed unit tests (src/backend_cpu.zig:1311-1380,
   src/engine.zig:2201-2386), restated.
3. The reference's own x86 C kernels, compiled from its sources into
   oracle/_ref/libq35ref.so: with QWEN35_FORCE_SCALAR=all they take their
   scalar tier and the oracle must match them bit for bit.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle_lib import (TT, GEOM, ROOT, REF_SO, act_row_bytes, bp, dequant, fp, ip, load_oracle,
                        matvec_q, quantize_act, quantize_weight, row_bytes)

GOLD = os.path.join(ROOT, "tests", "golden", "udtest")


@pytest.fixture(scope="module")
def L():
    return load_oracle()


@pytest.mark.parametrize("name,rb", [("Q4_K", 144), ("Q5_K", 176), ("Q6_K", 210),
                                     ("IQ4_NL", 144), ("Q4_0", 144), ("Q4_1", 160), ("IQ4_XS", 136)])
def test_golden_dequant(L, name, rb):
    ax = np.fromfile(os.path.join(GOLD, "A_x.f32"), dtype=np.float32)
    rows = np.fromfile(os.path.join(GOLD, f"{name}.bin"), dtype=np.uint8).reshape(-1, rb)
    exp = np.fromfile(os.path.join(GOLD, f"{name}_expected.f32"), dtype=np.float32)
    assert rows.shape[0] == 96 and exp.shape[0] == 96
    deq = dequant(L, TT[name], rows, 256)
    # the reference's check: serial f32 sum of dequant*ax (quant_dequant.zig:1113-1114)
    got = np.array([np.float32(0) + np.cumsum((deq[r] * ax).astype(np.float32), dtype=np.float32)[-1]
                    for r in range(96)], dtype=np.float32)
    err = np.abs(got - exp).max()
    assert err < 1e-3, err
    # measured margin is far tighter than the reference's 1e-3 bar
    assert err < 1e-4, err


def _deq_act(L, tt, xq, cols):
    """f32 values the quantized activation stands for"""
    if GEOM[tt][0] == 32:
        return dequant(L, TT["Q8_0"], xq, cols)[0]
    out = np.zeros(cols, dtype=np.float32)
    for b in range(cols // 256):
        blk = xq[0, b * 292:(b + 1) * 292]
        out[b * 256:(b + 1) * 256] = blk[:4].view(np.float32)[0] * blk[4:260].view(np.int8)
    return out


def test_golden_rowdot_matches_dequant(L):
    """rowDot kernels match dot(dequant(row)) (quant_dequant.zig:1126-1173),
    here on the quantized activation the matvec path consumes: the only
    difference left is the f32 block fold, so the bar is 1e-5 relative."""
    ax = np.fromfile(os.path.join(GOLD, "A_x.f32"), dtype=np.float32)
    for name, rb in [("Q4_K", 144), ("Q5_K", 176), ("Q6_K", 210), ("IQ4_NL", 144), ("Q4_0", 144), ("Q4_1", 160),
                     ("IQ4_XS", 136)]:
        tt = TT[name]
        rows = np.fromfile(os.path.join(GOLD, f"{name}.bin"), dtype=np.uint8).reshape(-1, rb)
        xq = quantize_act(L, tt, ax)
        out = matvec_q(L, tt, rows, xq, 96, 256, 1)[0]
        ref = dequant(L, tt, rows, 256).astype(np.float64) @ _deq_act(L, tt, xq, 256).astype(np.float64)
        rel = np.abs(out - ref) / np.maximum(np.abs(ref), 1)
        assert rel.max() < 1e-5, (name, rel.max())


def test_q8_0_hand_block(L):
    """backend_cpu.zig:1366-1380"""
    d = np.zeros(34, dtype=np.uint8)
    h = L.q35o_f32_to_f16(1.5)
    d[0], d[1] = h & 0xFF, h >> 8
    qs = np.array([0, 1, -1, 32, -128] + [0] * 27, dtype=np.int8)
    d[2:] = qs.view(np.uint8)
    out = dequant(L, TT["Q8_0"], d[None], 32)[0]
    assert list(out[:5]) == [0.0, 1.5, -1.5, 48.0, -192.0]


def test_q8_0_matvec_vs_f32(L):
    """backend_cpu.zig:1311-1350: Q8_0 matvec == f32 matvec over dequantized
    weights and dequantized activation, within 1e-5 rel + 1e-4 abs."""
    rng = np.random.default_rng(42)
    rows, cols = 5, 96
    w = (rng.random((rows, cols), dtype=np.float32) * 2 - 1)
    x = (rng.random(cols, dtype=np.float32) * 2 - 1)
    wq = np.zeros((rows, cols // 32 * 34), dtype=np.uint8)
    L.q35o_quantize_weight(TT["Q8_0"], rows * cols, fp(w), bp(wq))
    wf = dequant(L, TT["Q8_0"], wq, cols)
    xq = quantize_act(L, TT["Q8_0"], x)
    xf = dequant(L, TT["Q8_0"], xq, cols)[0]
    out = matvec_q(L, TT["Q8_0"], wq, xq, rows, cols, 1)[0]
    ref = wf @ xf
    assert np.all(np.abs(out - ref) <= np.abs(ref) * 1e-5 + 1e-4)


def test_q8_0_zero_x(L):
    wq = np.zeros((2, 34), dtype=np.uint8)
    vals = np.array([1, 2, 3] + [0] * 29, dtype=np.float32)
    L.q35o_quantize_weight(TT["Q8_0"], 32, fp(vals), bp(wq[0]))
    L.q35o_quantize_weight(TT["Q8_0"], 32, fp(vals), bp(wq[1]))
    xq = quantize_act(L, TT["Q8_0"], np.zeros(32, dtype=np.float32))
    out = matvec_q(L, TT["Q8_0"], wq, xq, 2, 32, 1)[0]
    assert out[0] == 0 and out[1] == 0


def test_f16_exhaustive(L):
    """quant_dequant.zig:1246-1292: every f16 code decodes exactly."""
    codes = np.arange(65536, dtype=np.uint16)
    ref = codes.view(np.float16).astype(np.float32)
    got = np.array([L.q35o_f16_to_f32(int(c)) for c in codes], dtype=np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(ref)]))


def test_f32_to_f16_rne(L):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-8, 5, 20000),
                        np.array([65504, 65519, 65520, 1e-8, 6e-8, 3e-5], dtype=np.float32)]).astype(np.float32)
    got = np.array([L.q35o_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, ref)


def test_weight_quantizers_roundtrip(L):
    rng = np.random.default_rng(7)
    w = rng.standard_normal((8, 1024)).astype(np.float32) * 0.02
    for name, tol in [("Q8_0", 0.01), ("IQ4_NL", 0.12), ("Q4_K", 0.12), ("Q5_K", 0.06), ("Q6_K", 0.03)]:
        tt = TT[name]
        wq = quantize_weight(L, tt, w)
        assert wq.shape[1] == row_bytes(tt, 1024)
        back = dequant(L, tt, wq, 1024)
        rel = np.linalg.norm(back - w) / np.linalg.norm(w)
        assert rel < tol, (name, rel)


def test_activation_quantizers(L):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(1024).astype(np.float32)
    q0 = quantize_act(L, TT["Q8_0"], x)[0]
    assert q0.size == 1024 // 32 * 34
    qk = quantize_act(L, TT["Q4_K"], x)[0]
    assert qk.size == 4 * 292
    blk = qk[:292]
    qs = blk[4:260].view(np.int8).astype(np.int32)
    bs = blk[260:292].view(np.int16)
    assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
    assert qs.min() >= -127
    z = quantize_act(L, TT["Q8_0"], np.zeros(32, dtype=np.float32))[0]
    assert z[0] == 0x00 and z[1] == 0x3C  # scale 1.0 stored when amax == 0


def test_elementwise_hand_values(L):
    """src/engine.zig:2201-2247"""
    out = np.zeros(2, dtype=np.float32)
    L.q35o_rmsnorm(fp(out), fp(np.array([3, 4], dtype=np.float32)), fp(np.ones(2, dtype=np.float32)), 2, 0.0)
    inv = 1 / np.sqrt(12.5)
    assert abs(out[0] - 3 * inv) < 1e-6 and abs(out[1] - 4 * inv) < 1e-6
    assert abs(L.q35o_silu(0.0)) < 1e-6
    assert abs(L.q35o_silu(1.0) - 0.7310586) < 1e-5
    assert abs(L.q35o_silu(-1.0) + 0.26894143) < 1e-5
    assert abs(L.q35o_sigmoid(0.0) - 0.5) < 1e-6
    assert abs(L.q35o_softplus(0.0) - np.log(2)) < 1e-6
    assert abs(L.q35o_softplus(25.0) - 25) < 1e-5
    x = np.array([1, 2, 1000, -5], dtype=np.float32)
    L.q35o_softmax(fp(x), 4)
    assert abs(x.sum() - 1) < 1e-5 and x[2] > 0.99
    y = np.array([3, 4], dtype=np.float32)
    L.q35o_l2norm(fp(y), 2)
    assert abs(y[0] - 0.6) < 1e-6 and abs(y[1] - 0.8) < 1e-6


def test_rope_hand_values(L):
    """src/engine.zig:2249-2291"""
    x = np.arange(256, dtype=np.float32)
    L.q35o_rope64(fp(x), 0, 1e7)
    assert np.allclose(x, np.arange(256), atol=1e-4)
    y = np.arange(256, dtype=np.float32)
    L.q35o_rope64(fp(y), 1, 1e7)
    assert abs(y[0] - (-32 * 0.84147096)) < 1e-3
    assert abs(y[32] - 32 * 0.54030234) < 1e-3
    c1, s1 = 0.82290208, 0.56818324
    assert abs(y[1] - (1 * c1 - 33 * s1)) < 1e-3 and abs(y[33] - (1 * s1 + 33 * c1)) < 1e-3
    assert np.array_equal(y[64:], np.arange(64, 256, dtype=np.float32))
    z = np.zeros(64, dtype=np.float32)
    z[31] = 1
    L.q35o_rope64(fp(z), 1000000, 1e7)
    assert abs(z[31] - np.cos(np.float32(1e6) * np.float32(1.6548171e-07))) < 1e-4
    # every head of a row is rotated
    r = np.tile(np.arange(256, dtype=np.float32), 3)
    L.q35o_rope64_rows(fp(r), 1, 3, 256, 1, 1e7)
    assert np.array_equal(r[:256], r[256:512]) and np.array_equal(r[:256], r[512:])
    assert abs(r[0] - (-32 * 0.84147096)) < 1e-3


def test_conv_step_hand_values(L):
    """src/engine.zig:2301-2347"""
    conv = np.zeros(3, dtype=np.float32)
    wc = np.array([1, 0.5, 0.25, 2], dtype=np.float32)
    silu = lambda v: v / (1 + np.exp(-v))
    q = np.array([1], dtype=np.float32)
    L.q35o_conv_step(fp(conv), fp(q), fp(wc), 1)
    assert abs(q[0] - silu(2.0)) < 1e-5
    q[0] = 10
    L.q35o_conv_step(fp(conv), fp(q), fp(wc), 1)
    assert abs(q[0] - silu(20.25)) < 1e-4
    q[0] = 100
    L.q35o_conv_step(fp(conv), fp(q), fp(wc), 1)
    assert abs(q[0] - silu(203.0)) < 1e-3


def test_gdn_step_hand_values(L):
    """src/engine.zig:2349-2386 (kd = vd = 2)"""
    S = np.zeros(4, dtype=np.float32)
    k = np.array([0, 1], dtype=np.float32)
    v = np.array([3, 4], dtype=np.float32)
    q = np.array([1, 0], dtype=np.float32)
    km = np.zeros(2, dtype=np.float32)
    dl = np.zeros(2, dtype=np.float32)
    o = np.zeros(2, dtype=np.float32)
    L.q35o_gdn_fused(fp(S), fp(k), fp(v), fp(q), fp(km), fp(dl), fp(o), 0.9, 0.5, 2, 2)
    assert list(o) == [0, 0] and list(S) == [0, 0, 1.5, 2]
    L.q35o_gdn_fused(fp(S), fp(k), fp(v), fp(k), fp(km), fp(dl), fp(o), 1.0, 0.0, 2, 2)
    assert list(o) == [1.5, 2]


def test_attn_decode_matches_numpy(L):
    rng = np.random.default_rng(5)
    heads, kvh, hd, n = 8, 2, 256, 37
    q = rng.standard_normal(heads * hd).astype(np.float32)
    g = rng.standard_normal(heads * hd).astype(np.float32)
    K = rng.standard_normal((n, kvh * hd)).astype(np.float32)
    V = rng.standard_normal((n, kvh * hd)).astype(np.float32)
    att = np.zeros(n, dtype=np.float32)
    out = np.zeros(heads * hd, dtype=np.float32)
    L.q35o_attn_decode(fp(q), fp(g), fp(K), fp(V), fp(att), fp(out), n - 1, heads, heads // kvh, hd,
                       kvh * hd, np.float32(1 / 16))
    ref = np.zeros_like(out, dtype=np.float64)
    for h in range(heads):
        kh = h // (heads // kvh)
        s = K[:, kh * hd:(kh + 1) * hd].astype(np.float64) @ q[h * hd:(h + 1) * hd] / 16
        p = np.exp(s - s.max())
        p /= p.sum()
        ref[h * hd:(h + 1) * hd] = p @ V[:, kh * hd:(kh + 1) * hd]
    ref *= 1 / (1 + np.exp(-g.astype(np.float64)))
    assert np.abs(out - ref).max() < 1e-5


REF_PROBE = r"""
import ctypes, sys, numpy as np
sys.path.insert(0, sys.argv[1])
from oracle_lib import load_oracle, load_ref, quantize_weight, TT, fp, bp, row_bytes, act_row_bytes
O = load_oracle(); R = ctypes.CDLL(sys.argv[2])
rng = np.random.default_rng(11)
def interleave_q5(w, tt):
    # GGUF Q5_0 / Q5_1 blocks -> the nibble order the reference's scalar
    # kernels read (element j in nibble j & 1 of qs[j / 2])
    b = 22 if tt == "Q5_0" else 24
    off = 6 if tt == "Q5_0" else 8
    w = w.reshape(-1, b).copy()
    qs = w[:, off:off + 16]
    q = np.concatenate([qs & 0x0F, qs >> 4], axis=1)  # element order 0..31
    w[:, off:off + 16] = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return w.reshape(-1)
def iq4xs_row(cols):
    # any nibbles / scale bits are valid IQ4_XS; d a finite f16
    w = rng.integers(0, 256, size=(cols // 256, 136), dtype=np.uint8)
    w[:, 0:2] = (rng.uniform(0.5, 2.0, cols // 256) * 1e-3).astype(np.float16).view(np.uint8).reshape(-1, 2)
    return w.reshape(-1)
for nm in ("q8_0_q8_0","iq4_nl_q8_0","q4_k_q8_k","q5_k_q8_k","q6_k_q8_k","q4_0_q8_0","q4_1_q8_0","q5_0_q8_0",
           "q5_1_q8_0","iq4_xs_q8_k"):
    getattr(R, nm).restype = ctypes.c_float
    getattr(R, nm).argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
R.quantize_q8_0.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
R.quantize_q8_K.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
cols = 1024
bad = 0
for trial in range(40):
    x = (rng.standard_normal(cols) * 10.0 ** rng.integers(-3, 3)).astype(np.float32)
    if trial == 0: x[:64] = 0
    a0 = np.zeros(cols // 32 * 34, np.uint8); b0 = np.zeros_like(a0)
    R.quantize_q8_0(cols, x.ctypes.data, a0.ctypes.data); O.q35o_quantize_q8_0(cols, fp(x), bp(b0))
    ak = np.zeros(cols // 256 * 292, np.uint8); bk = np.zeros_like(ak)
    R.quantize_q8_K(cols, x.ctypes.data, ak.ctypes.data); O.q35o_quantize_q8_K(cols, fp(x), bp(bk))
    bad += (not np.array_equal(a0, b0)) + (not np.array_equal(ak, bk))
    for nm, tt in (("q8_0_q8_0","Q8_0"),("iq4_nl_q8_0","IQ4_NL"),("q4_k_q8_k","Q4_K"),("q5_k_q8_k","Q5_K"),
                   ("q6_k_q8_k","Q6_K"),("q4_0_q8_0","Q4_0"),("q4_1_q8_0","Q4_1"),("q5_0_q8_0","Q5_0"),
                   ("q5_1_q8_0","Q5_1"),("iq4_xs_q8_k","IQ4_XS")):
        w = (iq4xs_row(cols) if tt == "IQ4_XS" else
             quantize_weight(O, TT[tt], rng.standard_normal((1, cols)).astype(np.float32) * 0.02)[0])
        xq = a0 if tt in ("Q8_0","IQ4_NL","Q4_0","Q4_1","Q5_0","Q5_1") else ak
        wr = interleave_q5(w, tt) if (tt in ("Q5_0","Q5_1") and sys.argv[3] == "exact") else w
        r = np.float32(getattr(R, nm)(cols, wr.ctypes.data, xq.ctypes.data))
        o = np.float32(O.q35o_vec_dot(TT[tt], cols, bp(w), bp(xq)))
        if sys.argv[3] == "exact":
            bad += int(r.view(np.uint32) != o.view(np.uint32))
        else:
            bad += int(abs(r - o) > 1e-5 * max(1.0, abs(o)))
print("BAD", bad)
"""


def _run_ref(mode):
    env = dict(os.environ)
    if mode == "exact":
        env["QWEN35_FORCE_SCALAR"] = "all"
        env["QWEN35_IQ_FORCE_SCALAR"] = "1"  # the IQ kernels' own scalar switch (iq_kernels.c:1008)
    else:
        env.pop("QWEN35_FORCE_SCALAR", None)
        env.pop("QWEN35_IQ_FORCE_SCALAR", None)
    r = subprocess.run([sys.executable, "-c", REF_PROBE, os.path.join(ROOT, "tests"), REF_SO, mode],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return int(r.stdout.split("BAD")[-1])


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference kernels not built (no reference tree)")
def test_against_reference_kernels_scalar_tier():
    """Oracle == reference x86 kernels' scalar tier, bit for bit, for the
    five hot types, Q4_0 / Q4_1 / Q5_0 / Q5_1 and IQ4_XS.  The reference's scalar
    Q5_0 / Q5_1 kernels read element j from nibble j & 1 of qs[j / 2]
    (kernels32.c:557, 640), unlike its AVX2 kernels and the GGUF format (low
    nibbles are elements 0..15): they are fed the same weights in that order,
    so the arithmetic is pinned bit for bit and the layout by the default
    tier below."""
    assert _run_ref("exact") == 0


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference kernels not built (no reference tree)")
def test_against_reference_kernels_default_tier():
    """The default (AVX2/VNNI) tier reorders the f32 folds (FMA lanes); within
    1e-5.  Q5_0 / Q5_1 here run the reference's AVX2 unpack, the GGUF nibble
    layout, on the oracle's weights as they are."""
    assert _run_ref("default") == 0


def test_synth_generator_c_equals_numpy(L):
    """the oracle's q35o_synth_fill (the CPU side of q35b_synth_fill) and the
    numpy statement in qwen35_b200.configs give the same bits, and the values
    have the intended spread"""
    from qwen35_b200 import configs
    for key, sigma, n in ((0, 0.02, 65536), (2**64 - 1, 1.0, 4099), (977, 0.5, 31)):
        a = np.empty(n, np.float32)
        L.q35o_synth_fill(key, n, configs.synth_k(sigma), fp(a))
        b = configs.synth_normal_np(key, n, sigma)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    a = configs.synth_normal_np(5, 1 << 18, 1.0)
    assert abs(float(a.mean())) < 0.01 and abs(float(a.std()) - 1.0) < 0.01
    v = configs.synth_vector(3, 1000, "ssm_a")
    assert (v < 0).all() and v.min() >= -np.e and v.max() <= -1 / np.e


def test_golden_f16_rows_w16_order(L):
    """the reference's F16 known-answer rows (testdata/udtest/F16, 96 x 256)
    through the oracle's restatement of the reference CUDA w16 kernel
    (mmvq.cu:339-351: one fmaf chain per row).  The reference's own golden
    check leaves F16 out (quant_dequant.zig:1185-1200) and its expected values
    differ from an exact f64 dot by up to 1.7e-3 relative, so they serve as a
    sanity band here (2e-3 relative); the order itself is pinned bit for bit
    against the f32 chain below and against the GPU (tests/test_gpu_formats.py)"""
    ax = np.fromfile(os.path.join(GOLD, "A_x.f32"), dtype=np.float32)
    w = np.fromfile(os.path.join(GOLD, "F16.bin"), dtype=np.uint16).reshape(96, 256)
    exp = np.fromfile(os.path.join(GOLD, "F16_expected.f32"), dtype=np.float32)
    out = np.zeros(96, np.float32)
    L.q35o_matvec_w16(1, w.ctypes.data, fp(ax), fp(out), 96, 256, 1)
    assert (np.abs(out - exp) / np.maximum(1.0, np.abs(exp))).max() < 2e-3
    # bf16 / f32: the same chain over exactly widened values
    wf = w.astype(np.uint16).view(np.float16).astype(np.float32)
    out32 = np.zeros(96, np.float32)
    L.q35o_matvec_f32(fp(np.ascontiguousarray(wf)), fp(ax), fp(out32), 96, 256, 1)
    assert np.array_equal(out32.view(np.uint32), out.view(np.uint32))
