"""GPU parity of the sm_100a kernels against the CPU oracle (via the C ABI).

Bar: activation codes, row scales and int32 accumulators bit-exact; fp16
outputs bit-exact as well (the epilogue is two IEEE fp32 multiplies and one
round-to-nearest fp16 conversion, exactly the reference's order).  The
tolerance the reference project states for fp16 outputs (max-abs error
<= 1e-3 x RMS(y)) is asserted too, as the documented contract.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w4a4_oracle as orc
from pi05_pytorch_fast_b200 import _native as nat
from pi05_pytorch_fast_b200.w4a4 import extension as ext

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
RMS_TOL = 1e-3
STAGINGS = {"fp16": nat.STAGING_FP16, "fp32": nat.STAGING_FP32}


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def assert_fp16_equal_and_within_tol(y: np.ndarray, y_ref: np.ndarray) -> None:
    rms = float(np.sqrt(np.mean(y_ref.astype(np.float64) ** 2))) if y_ref.size else 0.0
    err = float(np.max(np.abs(y.astype(np.float64) - y_ref.astype(np.float64)))) if y.size else 0.0
    assert err <= RMS_TOL * max(rms, 1e-30) or err == 0.0, (err, rms)
    np.testing.assert_array_equal(y.view(np.uint16), y_ref.view(np.uint16))


def gemm_order(codes: np.ndarray) -> np.ndarray:
    """Natural-order int8 codes -> the GEMM's byte order (0,2,4,6,1,3,5,7 per 8)."""
    m, k = codes.shape
    return np.ascontiguousarray(codes.reshape(m, k // 8, 8)[:, :, list(ext.GEMM_GROUP_ORDER)].reshape(m, k))


def gemm_accumulators(codes: torch.Tensor, weights, fragment_major=False):
    m, k = codes.shape
    layout = nat.LAYOUT_FRAGMENT_MAJOR if fragment_major else nat.LAYOUT_ROW_MAJOR
    accs = [torch.empty((m, int(w.size(0))), dtype=torch.int32, device=codes.device) for w in weights]
    descs = nat.weights_array([(w.data_ptr(), int(w.size(0)), int(w.size(1)), layout) for w in weights])
    outs = nat.pointer_array([a.data_ptr() for a in accs])
    nat.check(nat.lib().w4a4_gemm_accumulators(codes.data_ptr(), m, k, len(weights), descs, outs,
                                              torch.cuda.current_stream().cuda_stream))
    return accs


VARIANTS = {"single_cta": nat.GEMM_SINGLE_CTA, "cta_pair": nat.GEMM_CTA_PAIR,
            "no_split": nat.GEMM_NO_SPLIT, "split_k": nat.GEMM_SPLIT_K}


@pytest.fixture(params=list(VARIANTS))
def variant(request):
    """Runs a GEMM test through each kernel variant; all must be bit-exact."""
    nat.set_gemm_variant(VARIANTS[request.param])
    yield request.param
    nat.set_gemm_variant(nat.GEMM_SINGLE_CTA)


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    nat.device_error(clear=True)
    yield
    assert nat.device_error(clear=True) == 0, "a kernel's bounded wait ran out"


# ----------------------------------------------------------------------------- quant
@pytest.mark.parametrize("staging", ["fp16", "fp32"])
@pytest.mark.parametrize("k,m", [(1024, 9), (2048, 1), (2048, 17), (2048, 776), (16384, 3),
                                 (16384, 776)])
def test_quant_codes_and_scales_bit_exact(k, m, staging):
    x = orc.make_activations(m, k, seed=k + m)
    ref_codes, ref_scale = orc.quant_activation(x, staging=staging)
    xd = to_dev(x)
    codes, scale = ext.quantize(xd, staging=STAGINGS[staging])
    np.testing.assert_array_equal(to_np(codes), ref_codes)
    np.testing.assert_array_equal(to_np(scale).view(np.int32), ref_scale.view(np.int32))
    packed, scale_p = ext.quantize(xd, staging=STAGINGS[staging], fmt="packed")
    np.testing.assert_array_equal(to_np(packed), orc.pack_nibbles(ref_codes))
    np.testing.assert_array_equal(to_np(scale_p).view(np.int32), ref_scale.view(np.int32))
    gemm_codes, _ = ext.quantize(xd, staging=STAGINGS[staging], fmt="gemm")
    np.testing.assert_array_equal(to_np(gemm_codes), gemm_order(ref_codes))


@pytest.mark.parametrize("staging", ["fp16", "fp32"])
@pytest.mark.parametrize("k,m,pad", [(2048, 5, 8), (16384, 450, 64), (16384, 2, 8)])
def test_quant_strided_rows_bit_exact(k, m, pad, staging):
    """Rows of x at a stride of k + pad elements (w4a4_quant's ldx): only the
    first k of each row are read (through the 3-D TMA map at K = 16384)."""
    x = orc.make_activations(m, k, seed=7 * k + m)
    ref_codes, ref_scale = orc.quant_activation(x, staging=staging)
    wide = np.full((m, k + pad), np.float16(1000.0))  # the pad would change amax if it were read
    wide[:, :k] = x
    xd = to_dev(wide)
    codes = torch.empty((m, k), dtype=torch.int8, device=DEV)
    scale = torch.empty((m,), dtype=torch.float32, device=DEV)
    nat.check(nat.lib().w4a4_quant(xd.data_ptr(), m, k, k + pad, nat.ROTATE_BY_K, STAGINGS[staging],
                                   nat.CODES_INT8, codes.data_ptr(), scale.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream))
    np.testing.assert_array_equal(to_np(codes), ref_codes)
    np.testing.assert_array_equal(to_np(scale).view(np.int32), ref_scale.view(np.int32))


@pytest.mark.parametrize("k", [64, 192, 4096, 2048])
def test_quant_without_rotation_bit_exact(k):
    x = orc.make_activations(13, k, seed=k)
    ref_codes, ref_scale = orc.quant_activation(x, rotate=False)
    codes, scale = ext.quantize(to_dev(x), rotate=0)
    np.testing.assert_array_equal(to_np(codes), ref_codes)
    np.testing.assert_array_equal(to_np(scale).view(np.int32), ref_scale.view(np.int32))


@pytest.mark.parametrize("name", ["q2048", "q1024", "q16384", "q192", "q4096"])
def test_quant_matches_reference_golden(golden, name):
    codes, scale = ext.quantize(to_dev(golden[f"{name}_x"]), staging=nat.STAGING_FP32)
    np.testing.assert_array_equal(to_np(codes), golden[f"{name}_codes"])
    np.testing.assert_array_equal(to_np(scale).view(np.int32), golden[f"{name}_scale"].view(np.int32))


def test_quant_ties_round_half_even():
    """Codes next to and exactly at half-integers: the kernels compute
    rint(v / sdiv) through a reciprocal with an IEEE-division fallback near
    ties, which must match the plain IEEE quotient bit for bit.  With an
    unrotated row whose amax is 7, sdiv = fl(fl(7/7) + 1e-12) = 1 exactly."""
    ties = np.array([0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5], np.float16)
    rows = []
    for sign in (1, -1):
        r = np.zeros(64, np.float16)
        r[:7] = sign * ties
        r[8:15] = sign * np.nextafter(ties, np.float16(8))    # one fp16 ulp above
        r[16:23] = sign * np.nextafter(ties, np.float16(0))   # one fp16 ulp below
        r[24] = np.float16(7.0)                               # amax = 7
        rows.append(r)
    x = np.stack(rows)
    ref_codes, ref_scale = orc.quant_activation(x, rotate=False)
    codes, scale = ext.quantize(to_dev(x), rotate=0)
    np.testing.assert_array_equal(to_np(codes), ref_codes)
    np.testing.assert_array_equal(to_np(scale).view(np.int32), ref_scale.view(np.int32))
    assert ref_scale[0] == 1.0 and ref_codes[0, 2] == 2 and ref_codes[0, 3] == 4
    assert ref_codes[1, 2] == -2


def test_quant_zero_and_constant_rows():
    x = np.zeros((4, 2048), np.float16)
    x[1] = 1.0
    x[2, 5] = -3.0
    x[3] = np.float16(65504.0) * ((np.arange(2048) % 2) * 2 - 1).astype(np.float16) / np.float16(2048)
    for staging in ("fp16", "fp32"):
        ref_codes, ref_scale = orc.quant_activation(x, staging=staging)
        codes, scale = ext.quantize(to_dev(x), staging=STAGINGS[staging])
        np.testing.assert_array_equal(to_np(codes), ref_codes)
        np.testing.assert_array_equal(to_np(scale).view(np.int32), ref_scale.view(np.int32))


# ----------------------------------------------------------------------------- GEMM
def _row_major(packed: np.ndarray, pad_to: int | None = None) -> torch.Tensor:
    k = (packed.shape[1] - 1) * 8
    p = orc.pad_rows(packed, pad_to if pad_to else k // 8 + 8)
    return to_dev(p)


GEMM_CASES = [
    # (m, k, [n per weight], layout)
    (1, 64, [24], "row"),
    (17, 2048, [200], "row"),
    (776, 2048, [2048, 256, 256], "row"),      # config 0: fused QKV
    (776, 2048, [2048], "row"),                # o_proj
    (272, 2048, [16384, 16384], "fragment"),   # gate/up, body + tail of the reference test
    (776, 16384, [2048], "row"),               # config 1: down_proj
    (3, 16384, [128], "row"),
    (257, 1024, [384, 128], "row"),
    (200, 4096, [256], "fragment"),            # split-K candidate, fragment-major
    (776, 2048, [2048, 2048, 2048], "row"),    # split-K: more tiles than clusters
    (776, 2048, [200, 328], "fragment"),       # CTA pair with a ragged last 256-row weight tile
]


@pytest.mark.parametrize("m,k,ns,layout", GEMM_CASES)
def test_gemm_accumulators_bit_exact(m, k, ns, layout, variant):
    rng = np.random.default_rng(m * 31 + k)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    packs = [orc.random_packed_weight(n, k, seed=i + m) for i, n in enumerate(ns)]
    frag = layout == "fragment"
    ws = [to_dev(orc.preshuffle_wmma_weight(p, k)) if frag else _row_major(p) for p in packs]
    accs = gemm_accumulators(to_dev(gemm_order(qa)), ws, fragment_major=frag)
    for p, acc in zip(packs, accs):
        qw, _ = orc.weight_codes_scales(p, k, "row")
        np.testing.assert_array_equal(to_np(acc), orc.int_accumulate(qa, qw))


@pytest.mark.parametrize("m,k,ns", [(4000, 16384, [384]), (25000, 2048, [640])])
def test_gemm_grouped_rasterisation_bit_exact(m, k, ns, variant):
    """Activation codes larger than ~48 MB are tiled in groups of token tiles
    (each group's codes stay in L2): 4000 x 16384 gives two groups of 208-row
    tiles (a split-K candidate), 25000 x 2048 two groups of 118 and 3 tiles."""
    rng = np.random.default_rng(m + k)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    packs = [orc.random_packed_weight(n, k, seed=i + 5) for i, n in enumerate(ns)]
    ws = [_row_major(p) for p in packs]
    accs = gemm_accumulators(to_dev(gemm_order(qa)), ws, fragment_major=False)
    for p, acc in zip(packs, accs):
        qw, _ = orc.weight_codes_scales(p, k, "row")
        np.testing.assert_array_equal(to_np(acc), orc.int_accumulate(qa, qw))


@pytest.mark.parametrize("m,k,ns,layout", GEMM_CASES)
def test_gemm_fp16_epilogue_bit_exact(m, k, ns, layout, variant):
    rng = np.random.default_rng(m * 17 + k)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    sa = (rng.random(m, dtype=np.float32) * np.float32(0.5) + np.float32(1e-3)).astype(np.float32)
    packs = [orc.random_packed_weight(n, k, seed=3 * i + m) for i, n in enumerate(ns)]
    frag = layout == "fragment"
    ws = [to_dev(orc.preshuffle_wmma_weight(p, k)) if frag else _row_major(p) for p in packs]
    ys = ext.gemm_from_codes(to_dev(gemm_order(qa)), to_dev(sa), ws, fragment_major=frag)
    for p, y in zip(packs, ys):
        qw, sw = orc.weight_codes_scales(p, k, "row")
        ref = orc.dequant(orc.int_accumulate(qa, qw), sa, sw)
        assert_fp16_equal_and_within_tol(to_np(y), ref)


@pytest.mark.filterwarnings("ignore::RuntimeWarning")
def test_fp16_staging_quant_matches_the_reference_kernel():
    """The CUDA quant (fp16 staging, the timed mode) against the reference's
    own quant_rot_rb compiled for host threads (oracle/_ref): codes and row
    scales bit for bit, an fp16-overflowing row included."""
    import test_oracle_ref_quant as refq

    lib = refq._ref_lib()
    for k in (1024, 2048, 16384):
        x = refq._inputs(k, seed=5)
        codes, sc = refq.ref_quant(lib, x)
        q_dev, s_dev = ext.quantize(to_dev(x), staging=nat.STAGING_FP16)
        np.testing.assert_array_equal(to_np(q_dev), codes)
        np.testing.assert_array_equal(to_np(s_dev).view(np.int32), sc.view(np.int32))


# ----------------------------------------------------------------------------- int8 repack
def repack_int8(w: torch.Tensor, k: int, fragment: bool) -> torch.Tensor:
    layout = nat.LAYOUT_FRAGMENT_MAJOR if fragment else nat.LAYOUT_ROW_MAJOR
    dst = torch.empty((int(w.size(0)), k // 4 + 4), dtype=torch.int32, device=w.device)
    desc = nat.weights_array([(w.data_ptr(), int(w.size(0)), int(w.size(1)), layout)])
    nat.check(nat.lib().w4a4_repack_int8(desc, k, dst.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return dst


def gemm_int8(codes: torch.Tensor, scales, weights, acc_out: bool):
    m, k = codes.shape
    dt = torch.int32 if acc_out else torch.float16
    ys = [torch.empty((m, int(w.size(0))), dtype=dt, device=codes.device) for w in weights]
    descs = nat.weights_array([(w.data_ptr(), int(w.size(0)), int(w.size(1)), nat.LAYOUT_INT8) for w in weights])
    outs = nat.pointer_array([y.data_ptr() for y in ys])
    st = torch.cuda.current_stream().cuda_stream
    if acc_out:
        nat.check(nat.lib().w4a4_gemm_accumulators(codes.data_ptr(), m, k, len(weights), descs, outs, st))
    else:
        nat.check(nat.lib().w4a4_gemm(codes.data_ptr(), scales.data_ptr(), m, k, len(weights), descs, outs, st))
    return ys


def test_repack_int8_layout():
    """Row n of the repack: 16 x code in the GEMM's K byte order, then the
    fp32 scale and three zero words; both source layouts give the same."""
    k, n = 256, 40
    p = orc.random_packed_weight(n, k, seed=9)
    qw, sw = orc.weight_codes_scales(p, k, "row")
    want = np.zeros((n, k // 4 + 4), dtype=np.int32)
    want.view(np.int8)[:, :k] = gemm_order(qw.astype(np.int8)) * 16
    want[:, k // 4] = sw.view(np.int32)
    for frag in (False, True):
        w = to_dev(orc.preshuffle_wmma_weight(p, k)) if frag else _row_major(p)
        np.testing.assert_array_equal(to_np(repack_int8(w, k, frag)), want)


@pytest.mark.parametrize("m,k,ns,layout", GEMM_CASES)
def test_int8_repacked_gemm_bit_exact(m, k, ns, layout):
    """The SS CTA-pair kernel on repacked weights: accumulators bit-exact with
    the oracle, fp16 outputs bit-exact with the dequant contract."""
    rng = np.random.default_rng(m * 7 + k)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    sa = (rng.random(m, dtype=np.float32) * np.float32(0.5) + np.float32(1e-3)).astype(np.float32)
    packs = [orc.random_packed_weight(n, k, seed=5 * i + m) for i, n in enumerate(ns)]
    frag = layout == "fragment"
    ws = [to_dev(orc.preshuffle_wmma_weight(p, k)) if frag else _row_major(p) for p in packs]
    w8 = [repack_int8(w, k, frag) for w in ws]
    codes = to_dev(gemm_order(qa))
    accs = gemm_int8(codes, None, w8, acc_out=True)
    ys = gemm_int8(codes, to_dev(sa), w8, acc_out=False)
    for p, acc, y in zip(packs, accs, ys):
        qw, sw = orc.weight_codes_scales(p, k, "row")
        ia = orc.int_accumulate(qa, qw)
        np.testing.assert_array_equal(to_np(acc), ia)
        assert_fp16_equal_and_within_tol(to_np(y), orc.dequant(ia, sa, sw))


@pytest.mark.parametrize("m", [1, 15, 16, 17, 100, 255, 256, 257, 640, 768, 776, 1000])
def test_gemm_ragged_token_counts(m, variant):
    k, n = 2048, 384
    rng = np.random.default_rng(m)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    p = orc.random_packed_weight(n, k, seed=m)
    acc = gemm_accumulators(to_dev(gemm_order(qa)), [_row_major(p)])[0]
    qw, _ = orc.weight_codes_scales(p, k, "row")
    np.testing.assert_array_equal(to_np(acc), orc.int_accumulate(qa, qw))


def test_gemm_row_stride_variants_agree(variant):
    """Any 16-byte-multiple row stride is read directly (K/8+8 is the default pad)."""
    m, k, n = 50, 2048, 256
    rng = np.random.default_rng(1)
    qa = rng.integers(-7, 8, size=(m, k)).astype(np.int8)
    p = orc.random_packed_weight(n, k, seed=2)
    qw, _ = orc.weight_codes_scales(p, k, "row")
    ref = orc.int_accumulate(qa, qw)
    for words in (k // 8 + 4, k // 8 + 8, k // 8 + 16):
        acc = gemm_accumulators(to_dev(gemm_order(qa)), [_row_major(p, words)])[0]
        np.testing.assert_array_equal(to_np(acc), ref)


def test_bounded_wait_times_out_and_context_survives():
    """A wait on a barrier nothing arrives at must give up, flag the error and
    return; the context must still run correct kernels afterwards."""
    nat.device_error(clear=True)
    nat.check(nat.lib().w4a4_selftest_wait_timeout(50_000_000, torch.cuda.current_stream().cuda_stream))
    bits = nat.device_error(clear=True)
    assert bits & (1 << 4), bits
    m, k, n = 33, 2048, 128
    x = orc.make_activations(m, k, seed=4)
    p = orc.random_packed_weight(n, k, seed=5)
    y = ext.int4_gemm(to_dev(x), _row_major(p))
    assert_fp16_equal_and_within_tol(to_np(y), orc.int4_gemm_ref(x, p, staging="fp16"))
    assert nat.device_error(clear=True) == 0


def test_wide_k_epilogue_matches_float_of_the_accumulator():
    """K = 131072 without rotation and worst-case codes (7 x -8 per term):
    |acc| = 7.3 M > 2^22, past the magic-number conversion's exact range; the
    epilogue must round like the reference's (float)acc."""
    m, n, k = 16, 128, 131072
    x = orc.make_activations(m, k, seed=4)
    x[0] = np.float16(0.5)
    x[1] = np.float16(-0.5)
    payload = np.full((n, k // 8), np.int32(-2004318072), dtype=np.int32)  # 0x88888888: every nibble -8
    payload[n // 2:] = orc.random_packed_weight(n - n // 2, k, 3)[:, : k // 8]
    scales = np.full((n,), 1e-3, dtype=np.float32)
    packed = orc.pad_rows(np.concatenate([payload, scales.view(np.int32)[:, None]], axis=1), k // 8 + 8)
    y = ext.int4_gemm(to_dev(x), to_dev(packed))
    ref = orc.int4_gemm_ref(x, packed, rotate=False, staging="fp32")
    assert abs(int(orc.int_accumulate(*[orc.quant_activation(x[:1], rotate=False)[0],
                                        orc.weight_codes_scales(packed[:1], k)[0]])[0, 0])) > 2 ** 22
    assert_fp16_equal_and_within_tol(to_np(y), ref)
