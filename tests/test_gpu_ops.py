"""The pi05_w4a4::* custom ops on the GPU: drop-in behaviour and end-to-end
parity with the oracle.

Includes the reference project's own GPU tests (tests/test_w4a4.py:45-85),
restated against these kernels: row padding is exact, fragment-major equals
row-major, the tiled op rejects a row-major weight with the reference's
message.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import w4a4_oracle as orc
from pi05_pytorch_fast_b200 import _native as nat
from pi05_pytorch_fast_b200.w4a4 import extension as ext
from pi05_pytorch_fast_b200.w4a4.pack import pack_linear_weight, preshuffle_wmma_weight

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def to_np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    nat.device_error(clear=True)
    yield
    assert nat.device_error(clear=True) == 0


@pytest.fixture(params=["fp16", "fp32"])
def staging(request, monkeypatch):
    monkeypatch.setenv("PI05_W4A4_STAGING", request.param)
    return request.param


def _random_packed(n, k, gen):
    # the reference fixture: random payload (every nibble, -8 included), scales U[0.01, 0.06)
    payload = torch.randint(-(2**31), 2**31 - 1, (n, k // 8), dtype=torch.int32, generator=gen)
    scales = torch.rand(n, dtype=torch.float32, generator=gen) * 0.05 + 0.01
    return torch.cat((payload, scales.view(torch.int32).unsqueeze(1)), dim=1)


# --------------------------------------------------------- the reference's GPU tests
def test_row_padding_is_exact_for_down_projection():
    gen = torch.Generator().manual_seed(20260923)
    x = torch.randn(3, 16384, generator=gen).half().to(DEV)
    packed = _random_packed(128, 16384, gen).to(DEV)
    padded = F.pad(packed, (0, 7))
    a = torch.ops.pi05_w4a4.int4_gemm(x, packed)
    b = torch.ops.pi05_w4a4.int4_gemm(x, padded)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_preshuffled_gate_weight_is_exact():
    gen = torch.Generator().manual_seed(20260923)
    x = torch.randn(272, 2048, generator=gen).half().to(DEV)
    packed = _random_packed(16384, 2048, gen)
    tiled = preshuffle_wmma_weight(packed, 2048).to(DEV)
    a = torch.ops.pi05_w4a4.int4_gemm(x, packed.to(DEV))
    b = torch.ops.pi05_w4a4.int4_gemm_tiled(x, tiled)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_tiled_op_rejects_row_major_weight():
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, 2048, generator=gen).half().to(DEV)
    packed = _random_packed(16384, 2048, gen).to(DEV)
    with pytest.raises(RuntimeError, match=r"K/8\+9 marker stride"):
        torch.ops.pi05_w4a4.int4_gemm_tiled(x, packed)


# --------------------------------------------------------- parity with the oracle
def test_golden_vectors_through_the_op(golden, monkeypatch):
    """fp32 staging reproduces the reference's own int4_gemm_ref outputs bit-exactly."""
    monkeypatch.setenv("PI05_W4A4_STAGING", "fp32")
    for name in ("g2048", "g16384", "g1024", "g128"):
        y = torch.ops.pi05_w4a4.int4_gemm(to_dev(golden[f"{name}_x"]), to_dev(golden[f"{name}_packed"]))
        np.testing.assert_array_equal(to_np(y).view(np.uint16), golden[f"{name}_y"].view(np.uint16))


def test_config0_fused_qkv(staging):
    """Config 0: M=776 x K=2048 activations (1% outlier channels x20), W = N(0, 0.02)
    [2560, 2048] packed and split into Q/K/V, int4_gemm3."""
    for seed in (0, 1, 2):
        x = orc.make_activations(776, 2048, seed)
        w = orc.pack_linear_weight(orc.make_weight(2560, 2048, seed))
        blocks = [w[0:2048], w[2048:2304], w[2304:2560]]
        outs = torch.ops.pi05_w4a4.int4_gemm3(to_dev(x), *[to_dev(orc.pad_rows(b, 264)) for b in blocks])
        ref = orc.int4_gemm_ref(x, w, staging=staging)
        got = np.concatenate([to_np(o) for o in outs], axis=1)
        np.testing.assert_array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_config1_gate_up_and_down(staging):
    seed = 0
    x = orc.make_activations(776, 2048, seed)
    wg = orc.pack_linear_weight(orc.make_weight(16384, 2048, seed + 1))
    wu = orc.pack_linear_weight(orc.make_weight(16384, 2048, seed + 2))
    g, u = torch.ops.pi05_w4a4.int4_gemm2_tiled(
        to_dev(x), to_dev(orc.preshuffle_wmma_weight(wg, 2048)), to_dev(orc.preshuffle_wmma_weight(wu, 2048)))
    np.testing.assert_array_equal(to_np(g).view(np.uint16), orc.int4_gemm_ref(x, wg, staging=staging).view(np.uint16))
    np.testing.assert_array_equal(to_np(u).view(np.uint16), orc.int4_gemm_ref(x, wu, staging=staging).view(np.uint16))
    g2, u2 = torch.ops.pi05_w4a4.int4_gemm2(to_dev(x), to_dev(orc.pad_rows(wg, 264)), to_dev(orc.pad_rows(wu, 264)))
    assert torch.equal(g, g2) and torch.equal(u, u2)
    h = orc.make_activations(776, 16384, seed + 3)
    wd = orc.pack_linear_weight(orc.make_weight(2048, 16384, seed + 4))
    d = torch.ops.pi05_w4a4.int4_gemm(to_dev(h), to_dev(orc.pad_rows(wd, 2056)))
    np.testing.assert_array_equal(to_np(d).view(np.uint16), orc.int4_gemm_ref(h, wd, staging=staging).view(np.uint16))


def test_batched_prefix_rows_sampled(staging):
    """Config 3's largest case (B=64 observations x 776 tokens = 49,664 rows) at
    full size.  Rows are independent, so checking a random sample of rows
    against the oracle is exact; the rest is covered by row-permutation
    equivariance."""
    m, k, n = 64 * 776, 2048, 2560
    gen = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(m, k, device=DEV, generator=gen).half()
    w = orc.pack_linear_weight(orc.make_weight(n, k, 7))
    wd = to_dev(orc.pad_rows(w, 264))
    y = torch.ops.pi05_w4a4.int4_gemm(x, wd)
    rows = np.sort(np.random.default_rng(0).choice(m, 64, replace=False))
    ref = orc.int4_gemm_ref(to_np(x[torch.from_numpy(rows).to(DEV)]), w, staging=staging)
    np.testing.assert_array_equal(to_np(y[torch.from_numpy(rows).to(DEV)]).view(np.uint16), ref.view(np.uint16))
    perm = torch.randperm(m, device=DEV, generator=gen)
    y_perm = torch.ops.pi05_w4a4.int4_gemm(x[perm].contiguous(), wd)
    assert torch.equal(y_perm, y[perm])


# --------------------------------------------------------- shapes, layouts, errors
def test_leading_dims_and_noncontiguous_input(staging):
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(2, 5, 2048, generator=gen).half()
    p = _random_packed(96, 2048, gen)
    y = torch.ops.pi05_w4a4.int4_gemm(x.to(DEV), p.to(DEV))
    assert y.shape == (2, 5, 96) and y.dtype == torch.float16
    ref = orc.int4_gemm_ref(x.numpy(), p.numpy(), staging=staging)
    np.testing.assert_array_equal(to_np(y).view(np.uint16), ref.view(np.uint16))
    xt = x.to(DEV).transpose(0, 1)  # non-contiguous view
    yt = torch.ops.pi05_w4a4.int4_gemm(xt, p.to(DEV))
    assert torch.equal(yt, y.transpose(0, 1))


def test_empty_input():
    p = _random_packed(64, 2048, torch.Generator().manual_seed(0)).to(DEV)
    y = torch.ops.pi05_w4a4.int4_gemm(torch.empty(0, 2048, dtype=torch.float16, device=DEV), p)
    assert y.shape == (0, 64)
    q, k, v = torch.ops.pi05_w4a4.int4_gemm3(torch.empty(2, 0, 2048, dtype=torch.float16, device=DEV), p, p, p)
    assert q.shape == (2, 0, 64)


def test_error_messages_match_reference():
    p = _random_packed(64, 2048, torch.Generator().manual_seed(0)).to(DEV)
    with pytest.raises(RuntimeError, match="activations must be float16"):
        torch.ops.pi05_w4a4.int4_gemm(torch.randn(2, 2048, device=DEV), p)
    with pytest.raises(RuntimeError, match="K must be a multiple of 64, got 100"):
        torch.ops.pi05_w4a4.int4_gemm(torch.randn(2, 100, device=DEV).half(), p)
    with pytest.raises(RuntimeError, match="must be int32"):
        torch.ops.pi05_w4a4.int4_gemm(torch.randn(2, 2048, device=DEV).half(), p.float())
    with pytest.raises(RuntimeError, match="K/8 packed words plus a scale"):
        torch.ops.pi05_w4a4.int4_gemm(torch.randn(2, 2048, device=DEV).half(), p[:, :200].contiguous())
    with pytest.raises(RuntimeError, match="only K=2048, N=16384"):
        torch.ops.pi05_w4a4.int4_gemm_tiled(torch.randn(2, 2048, device=DEV).half(), p)


def test_op_on_fp32_caller_input_matches_oracle(staging):
    """What the reference's W4A4Linear.forward does around the op
    (linear.py:50-59): an fp32 caller tensor cast to fp16, the op, the
    result cast back, plus a bias."""
    lin = torch.nn.Linear(2048, 320, bias=True)
    packed = pack_linear_weight(lin.weight)
    x = orc.make_activations(40, 2048, 11)
    xf = to_dev(x).float()
    y = torch.ops.pi05_w4a4.int4_gemm(xf.half().contiguous(), F.pad(packed, (0, 7)).to(DEV)).float()
    y = y + lin.bias.detach().to(DEV)
    ref = orc.int4_gemm_ref(x, packed.numpy(), staging=staging).astype(np.float32) + lin.bias.detach().numpy()
    np.testing.assert_array_equal(to_np(y), ref)


def test_gpu_pack_matches_cpu_pack():
    w = torch.randn(300, 2048, generator=torch.Generator().manual_seed(5)) * 0.02
    cpu = pack_linear_weight(w)
    gpu = pack_linear_weight(w.to(DEV), device=DEV)
    assert torch.equal(cpu, gpu.cpu())


def test_cuda_graph_capture_replays_identically():
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(776, 2048, generator=gen).half().to(DEV)
    ws = [_random_packed(n, 2048, gen).to(DEV) for n in (2048, 256, 256)]
    ws = [F.pad(w, (0, 7)) for w in ws]
    eager = torch.ops.pi05_w4a4.int4_gemm3(x, *ws)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            torch.ops.pi05_w4a4.int4_gemm3(x, *ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = torch.ops.pi05_w4a4.int4_gemm3(x, *ws)
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, outs):
        assert torch.equal(a, b)
    del g


# ----------------------------------------------------------------------------- GPU weight pack
@pytest.mark.parametrize("n,k", [(1, 64), (7, 1024), (256, 2048), (38, 16384), (12, 4096)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_gpu_weight_pack_equals_the_cpu_pack(n, k, dtype):
    """w4a4_pack_weight (the load-time pack kernel) against the fp32 CPU pack
    (pinned to the reference's golden vectors), in the row-major, padded and
    fragment-major layouts; rotation by K and forced either way."""
    from pi05_pytorch_fast_b200.w4a4 import pack as wpack

    gen = torch.Generator().manual_seed(n * 7 + k)
    w = (torch.randn(n, k, generator=gen) * 0.05).to(dtype)
    w[0, : k // 2] = 0.0                       # a half-zero row
    if n > 2:
        w[2] = (torch.arange(k) % 15 - 7).to(dtype) * 0.125   # ties after the division
    for rotate in (None, False, True):
        if rotate and k & (k - 1):
            continue
        ref = wpack.pack_linear_weight(w.float(), rotate=rotate)
        got = wpack.pack_weight_cuda(w, "row", rotate=rotate, device="cuda:0")
        assert torch.equal(got.cpu(), ref)
        got = wpack.pack_weight_cuda(w, "row", k // 8 + 8, rotate=rotate, device="cuda:0")
        assert torch.equal(got.cpu(), wpack.pad_row_words(ref, k // 8 + 8))
        if n % 2 == 0:
            got = wpack.pack_weight_cuda(w, "fragment", rotate=rotate, device="cuda:0")
            assert torch.equal(got.cpu(), wpack.preshuffle_wmma_weight(ref, k))
