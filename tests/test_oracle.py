"""Pin the CPU oracle against the reference's own outputs (golden vectors).

The golden vectors were produced by running the unmodified reference code
(``tests/golden/make_golden.py``); every comparison here is bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import w4a4_oracle as orc


@pytest.mark.parametrize("name", ["q2048", "q1024", "q16384", "q192", "q4096"])
def test_quant_fp32_matches_reference(golden, name):
    x = golden[f"{name}_x"]
    codes, scale = orc.quant_activation(x, staging="fp32")
    np.testing.assert_array_equal(codes, golden[f"{name}_codes"])
    np.testing.assert_array_equal(scale.view(np.int32), golden[f"{name}_scale"].view(np.int32))


def test_quant_rotate_override_matches_reference(golden):
    codes, scale = orc.quant_activation(golden["q2048norot_x"], rotate=False)
    np.testing.assert_array_equal(codes, golden["q2048norot_codes"])
    np.testing.assert_array_equal(scale.view(np.int32), golden["q2048norot_scale"].view(np.int32))


@pytest.mark.parametrize("name", ["w2048", "w1024", "w16384", "w128", "wzero"])
def test_pack_linear_weight_matches_reference(golden, name):
    packed = orc.pack_linear_weight(golden[f"{name}_w"])
    np.testing.assert_array_equal(packed, golden[f"{name}_packed"])


@pytest.mark.parametrize("name,k", [("pre64", 64), ("pre2048", 2048)])
def test_preshuffle_matches_reference(golden, name, k):
    tiled = orc.preshuffle_wmma_weight(golden[f"{name}_packed"], k)
    np.testing.assert_array_equal(tiled, golden[f"{name}_tiled"])
    # and the fragment-major reader recovers the row-major codes and scales
    q_row, s_row = orc.weight_codes_scales(golden[f"{name}_packed"], k, "row")
    q_frag, s_frag = orc.weight_codes_scales(tiled, k, "fragment")
    np.testing.assert_array_equal(q_row, q_frag)
    np.testing.assert_array_equal(s_row.view(np.int32), s_frag.view(np.int32))


@pytest.mark.parametrize("name", ["g2048", "g16384", "g1024", "g128"])
def test_int4_gemm_ref_matches_reference(golden, name):
    y = orc.int4_gemm_ref(golden[f"{name}_x"], golden[f"{name}_packed"])
    np.testing.assert_array_equal(y.view(np.uint16), golden[f"{name}_y"].view(np.uint16))


@pytest.mark.parametrize("name", ["g2048", "g16384"])
def test_row_padding_and_fragment_layouts_agree(golden, name):
    """Padding the row stride (apply.py:68-69) or preshuffling (pack.py:45-68)
    must not change the product (test_w4a4.py:55-78 asserts the same on GPU)."""
    x, p = golden[f"{name}_x"], golden[f"{name}_packed"]
    k = x.shape[-1]
    y = orc.int4_gemm_ref(x, p)
    y_pad = orc.int4_gemm_ref(x, orc.pad_rows(p, k // 8 + 8))
    y_frag = orc.int4_gemm_ref(x, orc.preshuffle_wmma_weight(p, k), layout="fragment")
    np.testing.assert_array_equal(y.view(np.uint16), y_pad.view(np.uint16))
    np.testing.assert_array_equal(y.view(np.uint16), y_frag.view(np.uint16))


def test_random_fixture_contains_minus_eight(golden):
    q, _ = orc.weight_codes_scales(golden["g16384_packed"], 16384, "row")
    assert (q == -8).any() and (q == 7).any()


@pytest.mark.parametrize("k", [1024, 2048])
def test_fp16_staging_two_restatements_agree(k):
    """fp16 staging (the HIP kernel's arithmetic) has no runnable reference
    here; cross-check the vectorised restatement against a literal
    loop-level restatement of int4_gemm.cu:396-449."""
    x = orc.make_activations(2, k, seed=5)
    codes, scale = orc.quant_activation(x, staging="fp16")
    for r in range(x.shape[0]):
        c_loop, sdiv = orc.quant_rot_rb_loops(x[r])
        np.testing.assert_array_equal(codes[r], c_loop)
        assert scale[r] == np.float32(sdiv * orc.inv_sqrt_k(k))


def test_fp16_staging_differs_from_fp32_by_at_most_one_code():
    x = orc.make_activations(64, 2048, seed=9)
    c16, _ = orc.quant_activation(x, staging="fp16")
    c32, _ = orc.quant_activation(x, staging="fp32")
    diff = np.abs(c16.astype(np.int32) - c32.astype(np.int32))
    assert diff.max() <= 1
    assert diff.sum() > 0  # the two modes really are different arithmetic


def test_codes_are_clamped_symmetric():
    x = orc.make_activations(16, 16384, seed=3)
    for staging in ("fp16", "fp32"):
        codes, _ = orc.quant_activation(x, staging=staging)
        assert codes.min() >= -7 and codes.max() <= 7
        assert (np.abs(codes) == 7).any(axis=1).all()  # the amax element maps to +-7


def test_nibble_roundtrip():
    rng = np.random.default_rng(0)
    q = rng.integers(-8, 8, size=(5, 64)).astype(np.int8)
    np.testing.assert_array_equal(orc.unpack_nibbles(orc.pack_nibbles(q), 64), q)


def test_zero_rows_quantise_to_zero():
    x = np.zeros((3, 2048), dtype=np.float16)
    for staging in ("fp16", "fp32"):
        codes, scale = orc.quant_activation(x, staging=staging)
        assert not codes.any()
        assert np.all(scale == np.float32(np.float32(1e-12) * orc.inv_sqrt_k(2048)))
