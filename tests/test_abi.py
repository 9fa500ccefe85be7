"""CPU checks of the drop-in boundary: the shared library builds for
sm_100a, loads without a GPU, and exports exactly what include/q35.h
declares (no compute calls here)."""
import ctypes
import os
import subprocess

import pytest

from qwen35_b200 import lib as q35lib
from qwen35_b200.build import LIB, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# every launcher the reference's CUDA host binds: api.h plus the extern block
# of src/backend_cuda.zig:80-218 (sampler, w16 matvec, rope rows, func getters)
REFERENCE_API = """
q35_gpu_cc q35_gpu_sm_count q35_gpu_name q35_launch_quantize_q8_0 q35_launch_quantize_q8_K
q35_launch_quantize_q8_1_mmq q35_launch_dequantize q35_launch_dequantize_row q35_launch_mul_mat_vec
q35_launch_mul_mat_vec_q8_0 q35_launch_mul_mat_vec_f32 q35_launch_l2norm_qk_scale q35_launch_scale_vec
q35_launch_scale_vec_strided q35_launch_add_resid q35_launch_copy_range q35_launch_deinterleave_qg
q35_launch_deinterleave_qg_strided q35_launch_zero_buf q35_launch_set_int1 q35_launch_rmsnorm
q35_launch_l2norm q35_launch_l2norm_strided q35_launch_silu q35_launch_mul_silu q35_launch_mul_sigmoid
q35_launch_swiglu q35_launch_softmax q35_launch_conv_step q35_launch_conv_step_rows q35_launch_argmax
q35_launch_rope64 q35_launch_rope64_dpos q35_func_rope64_dpos q35_launch_rope64_rows_dpos
q35_func_rope64_rows_dpos q35_launch_rope64_setenv q35_launch_gdn_step_rows q35_launch_gdn_step_rows_chunk
q35_launch_gdn_step_wy q35_launch_gdn_step q35_launch_gdn_gamma q35_launch_gdn_gamma_rows
q35_launch_attn_decode q35_launch_attn_chunk q35_attn_chunk_max_rows q35_func_attn_decode_dyn
q35_func_attn_decode_coal q35_func_attn_score_split q35_launch_attn_decode_dyn q35_launch_attn_decode_coal
q35_func_attn_score_split_dyn q35_func_attn_pv_split_dyn q35_func_attn_softmax_dyn q35_func_attn_reduce
q35_launch_attn_decode_split_dyn q35_launch_attn_decode_split2 q35_launch_init_tables q35_iq_tables_bytes
q35_iq_tables_ready q35_launch_deinit_tables q35_quant_act_block_elems q35_quant_geom q35_mmq_dp4a_wants
q35_mmq_act_block_bytes q35_launch_mul_mat_vec_tile q35_launch_quantize_q8_K_mmq
 q35_launch_mul_mat_vec_w16 q35_launch_rope64_rows q35_func_rope64 q35_func_attn_decode q35_func_copy_range q35_launch_sample q35_launch_sample_init q35_launch_sample_deinit q35_sample_ctl_ints q35_sample_scratch_ints
""".split()


@pytest.fixture(scope="module")
def built():
    build()
    return LIB


def test_builds_for_sm100a(built):
    assert os.path.exists(built)
    r = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", built], capture_output=True, text=True)
    assert r.returncode == 0 and "sm_100a" in r.stdout


def test_exports_every_declared_symbol(built):
    decl = [n for n, _, _ in q35lib.parse_header()]
    assert len(decl) == len(set(decl)) and len(decl) >= 80
    nm = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in nm.splitlines() if " T " in ln}
    missing = [d for d in decl if d not in exported]
    assert not missing, missing


def test_reference_api_covered():
    decl = {n for n, _, _ in q35lib.parse_header()}
    missing = [n for n in REFERENCE_API if n not in decl]
    assert not missing, missing


def test_loads_and_binds_without_gpu(built):
    L = q35lib.load()
    for name, _, _ in q35lib.parse_header():
        assert getattr(L, name) is not None
    # pure host queries: no device needed
    e, b = ctypes.c_int(), ctypes.c_int()
    assert L.q35_quant_geom(8, ctypes.byref(e), ctypes.byref(b)) == 1 and (e.value, b.value) == (32, 34)
    assert L.q35_quant_geom(14, ctypes.byref(e), ctypes.byref(b)) == 1 and (e.value, b.value) == (256, 210)
    assert L.q35_quant_geom(3, ctypes.byref(e), ctypes.byref(b)) == 1 and (e.value, b.value) == (32, 20)  # Q4_1
    assert L.q35_quant_geom(7, ctypes.byref(e), ctypes.byref(b)) == 1 and (e.value, b.value) == (32, 24)  # Q5_1
    assert L.q35_quant_geom(23, ctypes.byref(e), ctypes.byref(b)) == 1 and (e.value, b.value) == (256, 136)  # IQ4_XS
    assert L.q35_quant_geom(16, ctypes.byref(e), ctypes.byref(b)) == 0  # IQ2_XXS: not served
    assert L.q35_quant_act_block_elems(20) == 32 and L.q35_quant_act_block_elems(13) == 256
    assert L.q35_quant_act_block_elems(99) == 0
    assert L.q35_mmq_dp4a_wants(12) == 0
    assert L.q35_launch_mul_mat_vec_tile(None, None, None, 1, 256, 8, 12, None) == -1


def test_zero_size_work_is_success(built):
    L = q35lib.load()
    # n <= 0 returns cudaSuccess without a launch (api.h:126-130)
    assert L.q35_launch_quantize_q8_0(None, None, 0, None) == 0
    assert L.q35_launch_mul_mat_vec(None, None, None, 0, 256, 1, 8, None) == 0
    assert L.q35_launch_add_resid(None, None, 0, None) == 0
    assert L.q35_launch_gdn_step_rows(None, 0, None, 0, None, 0, None, 0, None, None, None, None, None,
                                      0, 1, 128, 128, None) == 0


def test_bad_shapes_rejected(built):
    L = q35lib.load()
    inv = 1  # cudaErrorInvalidValue
    assert L.q35_launch_mul_mat_vec(None, None, None, 4, 100, 1, 8, None) == inv   # cols % 32
    assert L.q35_launch_mul_mat_vec(None, None, None, 4, 256, 1, 16, None) == inv  # unknown type (IQ2_XXS)
    assert L.q35_launch_gdn_step_rows(None, 0, None, 0, None, 0, None, 0, None, None, None, None, None,
                                      4, 2, 64, 64, None) == inv                     # kd != 128
    assert L.q35_launch_dequantize_row(8, None, None, 33, None) == inv
