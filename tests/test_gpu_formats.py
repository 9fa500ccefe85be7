"""Weight formats beyond the five hot types, on the GPU through the C ABI,
against the CPU oracle on the same bytes.

- IQ4_XS (GGUF type 23; 256-element blocks of 136 bytes, IQ4_NL codebook,
  6-bit scale per 32-element sub-block, Q8_K activation): q35_launch_mul_mat_vec
  bit-exact with the oracle's restatement of the reference's scalar tier
  (iq_kernels.c:967-1000) on the lane-per-row path (columns a multiple of
  512, 16-byte rows), the block-splitting path (other widths) and many-token
  passes; q35_launch_dequantize_row bit-exact (quant_dequant.zig:323-345);
  the reference's own known-answer rows (testdata/udtest/IQ4_XS).
- F32 / F16 / BF16 weights x f32 activation (q35_launch_mul_mat_vec_f32 /
  _w16): bit-exact with the reference's CUDA order (one fmaf chain per row,
  mmvq.cu:339-367), ragged widths and row counts, and on the reference's F16
  known-answer rows.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle_lib import ROOT, TT, bp, dequant, fp, load_oracle, matvec_q, quantize_act

pytestmark = pytest.mark.gpu

GOLD = os.path.join(ROOT, "tests", "golden", "udtest")
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


def iq4xs_rows(rng, rows, cols):
    """random IQ4_XS rows: any nibbles and scale bits are valid; d is a
    finite f16 of a plausible magnitude"""
    nb = cols // 256
    w = rng.integers(0, 256, size=(rows, nb, 136), dtype=np.uint8)
    d = (rng.uniform(0.5, 2.0, size=(rows, nb)) * 10.0 ** rng.integers(-4, -1, size=(rows, nb))).astype(np.float16)
    w[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    return w.reshape(rows, nb * 136)


@pytest.mark.parametrize("rows,cols,tokens", [(6144, 1024, 1), (3584, 1024, 2), (2048, 2560, 5), (1000, 1024, 8),
                                              (512, 768, 3), (300, 256, 1), (1024, 1024, 16), (640, 2048, 64)])
def test_iq4_xs_matvec_bit_exact(L, O, rows, cols, tokens):
    rng = np.random.default_rng(rows + cols + tokens)
    w = iq4xs_rows(rng, rows, cols)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    xq = np.concatenate([quantize_act(O, TT["IQ4_XS"], x[t]) for t in range(tokens)])
    ref = matvec_q(O, TT["IQ4_XS"], w, xq, rows, cols, tokens)
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(xq).cuda()
    out = torch.full((tokens, rows), float("nan"), device="cuda")
    ok(L.q35_launch_mul_mat_vec(dw.data_ptr(), dx.data_ptr(), out.data_ptr(), rows, cols, tokens, 23, S))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    no_kernel_error(L)


def test_iq4_xs_golden_rows(L, O):
    """the reference's known-answer rows: GPU == oracle bit for bit; the
    expected values (dots of the dequantized rows with the f32 A_x, pinned at
    1e-4 by the oracle's golden test) within a 5 % band of the quantized-
    activation dot"""
    ax = np.fromfile(os.path.join(GOLD, "A_x.f32"), dtype=np.float32)
    rows = np.fromfile(os.path.join(GOLD, "IQ4_XS.bin"), dtype=np.uint8).reshape(-1, 136)
    exp = np.fromfile(os.path.join(GOLD, "IQ4_XS_expected.f32"), dtype=np.float32)
    xq = quantize_act(O, TT["IQ4_XS"], ax)
    ref = matvec_q(O, TT["IQ4_XS"], rows, xq, 96, 256, 1)
    out = torch.zeros((1, 96), device="cuda")
    dw, dx = torch.from_numpy(rows).cuda(), torch.from_numpy(xq).cuda()
    ok(L.q35_launch_mul_mat_vec(dw.data_ptr(), dx.data_ptr(), out.data_ptr(), 96, 256, 1, 23, S))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # quantizing A_x to Q8_K costs ~1e-2 relative per element; the bar is on
    # the dequantized rows (the oracle's golden test) -- here only a sanity band
    assert np.abs(got[0] - exp).max() < 0.05 * max(1.0, float(np.abs(exp).max()))
    no_kernel_error(L)


def test_iq4_xs_dequant_row_bit_exact(L, O):
    rng = np.random.default_rng(5)
    cols = 2048
    w = iq4xs_rows(rng, 3, cols)
    ref = dequant(O, TT["IQ4_XS"], w, cols)
    for r in range(3):
        dw = torch.from_numpy(w[r].copy()).cuda()
        out = torch.full((cols,), float("nan"), device="cuda")
        ok(L.q35_launch_dequantize_row(23, dw.data_ptr(), out.data_ptr(), cols, S))
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref[r].view(np.uint32))


def _f16_bits(rng, shape):
    return rng.standard_normal(shape).astype(np.float16).view(np.uint16)


def _bf16_bits(rng, shape):
    return (rng.standard_normal(shape).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("kind", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("rows,cols,tokens", [(300, 1000, 3), (6144, 1024, 1), (33, 40, 2), (1, 7, 1)])
def test_unquantized_matvec_reference_cuda_order(L, O, kind, rows, cols, tokens):
    rng = np.random.default_rng(rows * 7 + cols + tokens)
    x = rng.standard_normal((tokens, cols)).astype(np.float32)
    out = torch.full((tokens, rows), float("nan"), device="cuda")
    ref = np.zeros((tokens, rows), np.float32)
    dx = torch.from_numpy(x).cuda()
    if kind == "F32":
        w = rng.standard_normal((rows, cols)).astype(np.float32)
        O.q35o_matvec_f32(fp(w), fp(x), fp(ref), rows, cols, tokens)
        dw = torch.from_numpy(w).cuda()
        ok(L.q35_launch_mul_mat_vec_f32(dw.data_ptr(), dx.data_ptr(), out.data_ptr(), rows, cols, tokens, S))
    else:
        tt = 1 if kind == "F16" else 30
        w = _f16_bits(rng, (rows, cols)) if kind == "F16" else _bf16_bits(rng, (rows, cols))
        O.q35o_matvec_w16(tt, w.ctypes.data, fp(x), fp(ref), rows, cols, tokens)
        dw = torch.from_numpy(w.view(np.int16)).cuda()
        ok(L.q35_launch_mul_mat_vec_w16(dw.data_ptr(), dx.data_ptr(), out.data_ptr(), rows, cols, tokens, tt, S))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_f16_golden_rows(L, O):
    """the reference's F16 known-answer rows (96 x 256) against A_x: the GPU
    equals the oracle bit for bit; the expected values (which the reference's
    own golden check leaves out) within a 2e-3 relative sanity band"""
    ax = np.fromfile(os.path.join(GOLD, "A_x.f32"), dtype=np.float32)
    w = np.fromfile(os.path.join(GOLD, "F16.bin"), dtype=np.uint16).reshape(96, 256)
    exp = np.fromfile(os.path.join(GOLD, "F16_expected.f32"), dtype=np.float32)
    ref = np.zeros((1, 96), np.float32)
    O.q35o_matvec_w16(1, w.ctypes.data, fp(ax), fp(ref), 96, 256, 1)
    out = torch.zeros((1, 96), device="cuda")
    dw, dx = torch.from_numpy(w.view(np.int16)).cuda(), torch.from_numpy(ax).cuda()
    ok(L.q35_launch_mul_mat_vec_w16(dw.data_ptr(), dx.data_ptr(), out.data_ptr(), 96, 256, 1, 1, S))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert (np.abs(got[0] - exp) / np.maximum(1.0, np.abs(exp))).max() < 2e-3
