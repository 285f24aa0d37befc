"""GPU parity of the fused prefix-LM layer kernels (w4a4_rmsnorm_quant,
w4a4_geglu_quant, w4a4_rope, w4a4_prefix_attention), called through the C
ABI.

The glue each kernel fuses is floating-point PyTorch in the reference
(pi05_fast/w4a4/apply.py:126-191 over transformers' Gemma layer), so its
check is PyTorch's own eager CUDA result on the same GPU:

* GeGLU (F.gelu(gate, approximate="tanh") * up) and RoPE
  (apply_rotary_pos_emb): bit-exact;
* the residual add: bit-exact; GemmaRMSNorm: within one fp16 ulp (the mean
  of squares is summed in another order), almost always equal;
* the codes and row scales that follow: bit-exact against the CPU oracle fed
  the kernel's own normalised / GeGLU values (written to h_out);
* attention (fp32 scores, one-pass online softmax, fp16 probabilities, fp32
  P V): against
  an fp64 evaluation of the same masked attention, its max error must not
  exceed 1.5 x that of the reference's eager fp16 attention (which rounds the
  scores and the normalised probabilities to fp16), nor 2e-3 where that one
  is smaller.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import w4a4_oracle as orc
from pi05_pytorch_fast_b200 import _native as nat

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
STAGINGS = {"fp16": nat.STAGING_FP16, "fp32": nat.STAGING_FP32}


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    nat.device_error(clear=True)
    yield
    assert nat.device_error(clear=True) == 0, "a kernel's bounded wait ran out"


def _stream():
    return torch.cuda.current_stream(DEV).cuda_stream


def geglu_quant(gate, up, staging, h_out=True):
    m, k = gate.shape
    codes = torch.empty((m, k), dtype=torch.int8, device=DEV)
    scales = torch.empty((m,), dtype=torch.float32, device=DEV)
    h = torch.empty_like(gate) if h_out else None
    nat.check(nat.lib().w4a4_geglu_quant(gate.data_ptr(), up.data_ptr(), m, k, gate.stride(0),
                                         staging, nat.CODES_INT8, codes.data_ptr(), scales.data_ptr(),
                                         h.data_ptr() if h is not None else None, k, _stream()))
    return codes, scales, h


def rmsnorm_quant(x, delta, gain, eps, staging, quant=True, x_out=None):
    m, k = x.shape
    h = torch.empty_like(x)
    codes = torch.empty((m, k), dtype=torch.int8, device=DEV) if quant else None
    scales = torch.empty((m,), dtype=torch.float32, device=DEV) if quant else None
    nat.check(nat.lib().w4a4_rmsnorm_quant(
        x.data_ptr(), x.stride(0), delta.data_ptr() if delta is not None else None, k,
        gain.data_ptr(), eps, x_out.data_ptr() if x_out is not None else None, k, h.data_ptr(), k,
        m, k, staging, nat.CODES_INT8, codes.data_ptr() if quant else None,
        scales.data_ptr() if quant else None, _stream()))
    return h, codes, scales


def assert_half_equal(a: torch.Tensor, b: torch.Tensor):
    """Bit-exact fp16 equality, NaN payloads aside."""
    a16 = a.view(torch.int16).cpu().numpy()
    b16 = b.view(torch.int16).cpu().numpy()
    both_nan = torch.isnan(a).cpu().numpy() & torch.isnan(b).cpu().numpy()
    bad = (a16 != b16) & ~both_nan
    assert not bad.any(), f"{int(bad.sum())} of {bad.size} values differ; first at {np.argwhere(bad)[:3]}"


def assert_codes_match_oracle(h: torch.Tensor, codes, scales, staging):
    qa, sa = orc.quant_activation(h.cpu().numpy(), rotate=True, staging=staging)
    np.testing.assert_array_equal(codes.cpu().numpy(), qa)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.int32), sa.view(np.int32))


# ----------------------------------------------------------------------------- GeGLU
def test_gelu_of_every_fp16_value_matches_torch():
    """gelu_tanh(x) for all 65,536 fp16 bit patterns x, infinities and NaNs
    included (up = 1, so h = fl16(gelu))."""
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16)
    vals = bits.view(torch.float16)
    k = 16384
    m = -(-vals.numel() // k)
    gate = torch.zeros(m * k, dtype=torch.float16)
    gate[: vals.numel()] = vals
    gate = gate.view(m, k).to(DEV)
    up = torch.ones_like(gate)
    _, _, h = geglu_quant(gate, up, nat.STAGING_FP16)
    ref = F.gelu(gate, approximate="tanh")
    torch.cuda.synchronize()
    assert_half_equal(h, ref)


def test_geglu_product_of_every_finite_up_value_matches_torch():
    """fl16(fl16(gelu(g)) * u) for all finite fp16 u, against gates whose GELU
    spans tiny to large magnitudes, so products land in the fp16 subnormal
    range, overflow to infinity and round at every exponent."""
    bits = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16)
    vals = bits.view(torch.float16)
    vals = vals[torch.isfinite(vals)]
    k = 16384
    rows = -(-vals.numel() // k)
    up = torch.zeros(rows * k, dtype=torch.float16)
    up[: vals.numel()] = vals
    gates = [-4.0, -0.75, -1e-3, 3e-5, 0.37, 1.0, 2.5, 300.0]
    up = up.view(rows, k).repeat(len(gates), 1).to(DEV)
    gate = torch.tensor(gates, dtype=torch.float16).repeat_interleave(rows)[:, None].expand(-1, k)
    gate = gate.contiguous().to(DEV)
    _, _, h = geglu_quant(gate, up, nat.STAGING_FP16)
    ref = F.gelu(gate, approximate="tanh") * up
    torch.cuda.synchronize()
    assert_half_equal(h, ref)


@pytest.mark.parametrize("staging", list(STAGINGS))
@pytest.mark.parametrize("m", [1, 5, 776])
def test_geglu_quant_matches_torch_and_oracle(staging, m):
    gen = torch.Generator(device=DEV).manual_seed(11 + m)
    gate = (torch.randn(m, 16384, device=DEV, generator=gen) * 1.5).half()
    up = torch.randn(m, 16384, device=DEV, generator=gen).half()
    codes, scales, h = geglu_quant(gate, up, STAGINGS[staging])
    ref = F.gelu(gate, approximate="tanh") * up
    torch.cuda.synchronize()
    assert_half_equal(h, ref)
    assert_codes_match_oracle(ref, codes, scales, staging)


def test_geglu_quant_without_h_out_gives_the_same_codes():
    gen = torch.Generator(device=DEV).manual_seed(3)
    gate = torch.randn(64, 16384, device=DEV, generator=gen).half()
    up = torch.randn(64, 16384, device=DEV, generator=gen).half()
    c1, s1, _ = geglu_quant(gate, up, nat.STAGING_FP16)
    c2, s2, _ = geglu_quant(gate, up, nat.STAGING_FP16, h_out=False)
    assert torch.equal(c1, c2) and torch.equal(s1, s2)


# ----------------------------------------------------------------------------- RMSNorm
def gemma_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers' GemmaRMSNorm.forward (fp32 math, (1 + w) gain, cast back)."""
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (out * (1.0 + weight.float())).type_as(x)


@pytest.mark.parametrize("staging", list(STAGINGS))
@pytest.mark.parametrize("with_delta", [False, True])
@pytest.mark.parametrize("m", [1, 3, 776])
def test_rmsnorm_quant_matches_torch_and_oracle(staging, with_delta, m):
    gen = torch.Generator(device=DEV).manual_seed(5 * m + with_delta)
    x = (torch.randn(m, 2048, device=DEV, generator=gen) * 3).half()
    x[:, :20] *= 20  # outlier channels
    delta = torch.randn(m, 2048, device=DEV, generator=gen).half() if with_delta else None
    w = (torch.randn(2048, device=DEV, generator=gen) * 0.1).half()
    gain = (1.0 + w.float()).contiguous()
    eps = 1e-6
    x_out = torch.empty_like(x)
    h, codes, scales = rmsnorm_quant(x, delta, gain, eps, STAGINGS[staging], x_out=x_out)
    s_ref = x + delta if with_delta else x
    h_ref = gemma_rmsnorm(s_ref, w, eps)
    torch.cuda.synchronize()
    assert_half_equal(x_out, s_ref)
    d = (h.float() - h_ref.float()).abs()
    ulp = torch.finfo(torch.float16).eps * h_ref.float().abs().clamp_min(2.0 ** -14)
    assert bool((d <= ulp).all()), float((d / ulp).max())
    assert float((d > 0).float().mean()) < 2e-3
    assert_codes_match_oracle(h, codes, scales, staging)


def test_rmsnorm_in_place_residual_and_norm_only():
    gen = torch.Generator(device=DEV).manual_seed(9)
    x = torch.randn(40, 2048, device=DEV, generator=gen).half()
    delta = torch.randn(40, 2048, device=DEV, generator=gen).half()
    w = (torch.randn(2048, device=DEV, generator=gen) * 0.1).half()
    gain = (1.0 + w.float()).contiguous()
    s_ref = x + delta
    h_q, _, _ = rmsnorm_quant(x.clone(), delta, gain, 1e-6, nat.STAGING_FP16)
    h, _, _ = rmsnorm_quant(x, delta, gain, 1e-6, nat.STAGING_FP16, quant=False, x_out=x)
    torch.cuda.synchronize()
    assert_half_equal(x, s_ref)      # x updated in place
    assert_half_equal(h, h_q)        # the norm alone equals the norm inside the fused kernel


# ----------------------------------------------------------------------------- RoPE
def hf_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, heads: int) -> torch.Tensor:
    """transformers' apply_rotary_pos_emb on [1, heads, M, 256] (fp16)."""
    m = x.shape[0]
    xh = x.view(m, heads, 256).transpose(0, 1).unsqueeze(0)
    x1, x2 = xh[..., :128], xh[..., 128:]
    rot = torch.cat((-x2, x1), dim=-1)
    out = (xh * cos[None, None]) + (rot * sin[None, None])
    return out.squeeze(0).transpose(0, 1).reshape(m, heads * 256)


@pytest.mark.parametrize("heads", [1, 8])
def test_rope_matches_transformers(heads):
    m = 776
    gen = torch.Generator(device=DEV).manual_seed(heads)
    x = (torch.randn(m, heads * 256, device=DEV, generator=gen) * 2).half()
    pos = torch.arange(m, device=DEV)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 256, 2, dtype=torch.int64).float() / 256))
    freqs = pos[:, None].float() * inv_freq.to(DEV)[None]
    emb = torch.cat((freqs, freqs), -1)
    cos, sin = emb.cos().half().contiguous(), emb.sin().half().contiguous()
    out = torch.empty_like(x)
    nat.check(nat.lib().w4a4_rope(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0),
                                  cos.data_ptr(), sin.data_ptr(), m, heads, _stream()))
    ref = hf_rope(x, cos, sin, heads)
    torch.cuda.synchronize()
    assert_half_equal(out, ref)
    # in place gives the same
    nat.check(nat.lib().w4a4_rope(x.data_ptr(), x.stride(0), x.data_ptr(), x.stride(0),
                                  cos.data_ptr(), sin.data_ptr(), m, heads, _stream()))
    torch.cuda.synchronize()
    assert_half_equal(x, ref)


# ----------------------------------------------------------------------------- attention
def attention_eager_fp16(q, k, v, pad, heads):
    """transformers' eager_attention_forward in fp16 under lerobot's prefix
    mask (fp32 additive mask value -2.3819763e38): the reference's rounding."""
    from pi05_pytorch_fast_b200.prefix_lm import prefix_positions_and_mask

    b, seq = pad.shape
    _, mask = prefix_positions_and_mask(pad)
    qh = q.view(b, seq, heads, 256).transpose(1, 2)
    kh = k.view(b, seq, 1, 256).transpose(1, 2).expand(b, heads, seq, 256)
    vh = v.view(b, seq, 1, 256).transpose(1, 2).expand(b, heads, seq, 256)
    w = torch.matmul(qh, kh.transpose(2, 3)) * (256 ** -0.5)
    w = torch.softmax(w + mask, dim=-1, dtype=torch.float32).to(torch.float16)
    return torch.matmul(w, vh).transpose(1, 2).reshape(b * seq, heads * 256)


def attention_fp64(q, k, v, pad, heads):
    """The same attention in fp64: real queries over real keys, padded
    queries uniform over all keys."""
    b, seq = pad.shape
    qh = q.view(b, seq, heads, 256).double().transpose(1, 2)
    kh = k.view(b, seq, 1, 256).double().transpose(1, 2)
    vh = v.view(b, seq, 1, 256).double().transpose(1, 2)
    s = (qh @ kh.transpose(2, 3)) / 16.0
    allowed = pad[:, None, :, None] & pad[:, None, None, :]
    s = s.masked_fill(~allowed, float("-inf"))
    s = torch.where((~pad)[:, None, :, None], torch.zeros_like(s), s)
    return (torch.softmax(s, dim=-1) @ vh).transpose(1, 2).reshape(b * seq, heads * 256)


def prefix_attention(q, k, v, pad, heads):
    b, seq = pad.shape
    key_valid = pad.to(torch.uint8).contiguous()
    kv_len = (pad * torch.arange(1, seq + 1, device=DEV)).amax(dim=1).to(torch.int32)
    vt = torch.empty((b, 256, nat.attn_vt_stride(seq)), dtype=torch.float16, device=DEV)
    out = torch.full((b * seq, heads * 256), float("nan"), dtype=torch.float16, device=DEV)
    nat.check(nat.lib().w4a4_prefix_attention(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                                              v.data_ptr(), v.stride(0), key_valid.data_ptr(),
                                              kv_len.data_ptr(), b, seq, heads, vt.data_ptr(),
                                              out.data_ptr(), out.stride(0), None, None, None, 0, _stream()))
    return out


ATTN_CASES = [  # (batch, seq, real tokens per observation, q scale)
    (1, 776, [628], 1.0),
    (1, 776, [628], 4.0),
    (1, 776, [628], 8.0),  # scores spread enough that later key blocks raise the row max (O rescaled)
    (2, 640, [640, 300], 2.0),
    (3, 100, [1, 57, 100], 1.0),
    (1, 1, [1], 1.0),
    (2, 200, [0, 130], 1.0),
]


@pytest.mark.parametrize("batch,seq,real,qscale", ATTN_CASES)
def test_prefix_attention_matches_fp64_at_least_as_well_as_eager(batch, seq, real, qscale):
    heads = 8
    gen = torch.Generator(device=DEV).manual_seed(seq + batch)
    q = (torch.randn(batch * seq, heads * 256, device=DEV, generator=gen) * qscale).half()
    k = torch.randn(batch * seq, 256, device=DEV, generator=gen).half()
    v = torch.randn(batch * seq, 256, device=DEV, generator=gen).half()
    pad = torch.zeros(batch, seq, dtype=torch.bool, device=DEV)
    for i, n in enumerate(real):
        pad[i, :n] = True
    out = prefix_attention(q, k, v, pad, heads)
    truth = attention_fp64(q, k, v, pad, heads)
    eager = attention_eager_fp16(q, k, v, pad, heads)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    rows = pad.reshape(-1)  # real queries; padded ones are checked below
    err = (out.double() - truth).abs()
    err_eager = (eager.double() - truth).abs()
    if rows.any():
        e, e_ref = float(err[rows].max()), float(err_eager[rows].max())
        print(f"attention max |err|: kernel {e:.2e}, eager fp16 {e_ref:.2e}")
        assert e <= max(1.5 * e_ref, 2e-3), (e, e_ref)
    # padded queries: the mean of all seq values of their observation
    if (~rows).any():
        assert float(err[~rows].max()) <= 2e-3


def test_prefix_attention_rows_are_independent_of_the_batch():
    """An observation's output does not depend on the others in the batch."""
    heads, seq = 8, 776
    gen = torch.Generator(device=DEV).manual_seed(1)
    q = torch.randn(2 * seq, heads * 256, device=DEV, generator=gen).half()
    k = torch.randn(2 * seq, 256, device=DEV, generator=gen).half()
    v = torch.randn(2 * seq, 256, device=DEV, generator=gen).half()
    pad = torch.ones(2, seq, dtype=torch.bool, device=DEV)
    pad[:, 628:] = False
    both = prefix_attention(q, k, v, pad, heads)
    second = prefix_attention(q[seq:].contiguous(), k[seq:].contiguous(), v[seq:].contiguous(), pad[1:], heads)
    torch.cuda.synchronize()
    assert torch.equal(both[seq:].view(torch.int16), second.view(torch.int16))


def test_prefix_attention_rescales_when_a_late_key_dominates():
    """The dominant key of every query sits in the last real key block, so
    the running max jumps there and O is rescaled in TMEM."""
    heads, seq = 8, 640
    gen = torch.Generator(device=DEV).manual_seed(2)
    q = torch.randn(seq, heads * 256, device=DEV, generator=gen).half()
    k = (torch.randn(seq, 256, device=DEV, generator=gen) * 0.1).half()
    v = torch.randn(seq, 256, device=DEV, generator=gen).half()
    # key 600 aligned with every head's query direction: score ~ 3 * |q| * ...
    qmean = q.float().view(seq, heads, 256).mean(dim=(0, 1))
    k[600] = (qmean / qmean.norm() * 60).half()
    pad = torch.ones(1, seq, dtype=torch.bool, device=DEV)
    out = prefix_attention(q, k, v, pad, heads)
    truth = attention_fp64(q, k, v, pad, heads)
    eager = attention_eager_fp16(q, k, v, pad, heads)
    torch.cuda.synchronize()
    e = float((out.double() - truth).abs().max())
    e_ref = float((eager.double() - truth).abs().max())
    print(f"late-max attention: kernel {e:.2e}, eager fp16 {e_ref:.2e}")
    assert e <= max(1.5 * e_ref, 2e-3)


def test_prefix_attention_with_fused_rope_equals_rope_then_attention():
    """cos / sin given: q is rotated in place and k into k_out in the
    attention's first launch, exactly as w4a4_rope rotates them, and the
    result is the attention of the rotated inputs."""
    heads, seq, batch = 8, 776, 2
    gen = torch.Generator(device=DEV).manual_seed(4)
    q = torch.randn(batch * seq, heads * 256, device=DEV, generator=gen).half()
    k = torch.randn(batch * seq, 256, device=DEV, generator=gen).half()
    v = torch.randn(batch * seq, 256, device=DEV, generator=gen).half()
    pad = torch.ones(batch, seq, dtype=torch.bool, device=DEV)
    pad[:, 628:] = False
    pos = (torch.cumsum(pad.long(), 1) - 1).reshape(-1)
    inv_freq = (1.0 / (10000.0 ** (torch.arange(0, 256, 2, dtype=torch.int64).float() / 256))).half().float()
    freqs = pos[:, None].float() * inv_freq.to(DEV)[None]
    emb = torch.cat((freqs, freqs), -1)
    cos, sin = emb.cos().half().contiguous(), emb.sin().half().contiguous()
    q_ref, k_ref = hf_rope(q, cos, sin, heads), hf_rope(k, cos, sin, 1)
    expect = prefix_attention(q_ref.contiguous(), k_ref.contiguous(), v, pad, heads)
    key_valid = pad.to(torch.uint8).contiguous()
    kv_len = (pad * torch.arange(1, seq + 1, device=DEV)).amax(dim=1).to(torch.int32)
    vt = torch.empty((batch, 256, nat.attn_vt_stride(seq)), dtype=torch.float16, device=DEV)
    out = torch.empty_like(q)
    k_out = torch.empty_like(k)
    q2 = q.clone()
    nat.check(nat.lib().w4a4_prefix_attention(q2.data_ptr(), q2.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(),
                                              v.stride(0), key_valid.data_ptr(), kv_len.data_ptr(), batch, seq,
                                              heads, vt.data_ptr(), out.data_ptr(), out.stride(0), cos.data_ptr(),
                                              sin.data_ptr(), k_out.data_ptr(), k_out.stride(0), _stream()))
    torch.cuda.synchronize()
    assert_half_equal(q2, q_ref)
    assert_half_equal(k_out, k_ref)
    assert torch.equal(out.view(torch.int16), expect.view(torch.int16))


@pytest.mark.parametrize("seq,fp16_freq", [(776, True), (4096, True), (300, False)])
def test_prefix_tables_match_torch(seq, fp16_freq):
    """Positions, key mask, real-key spans and the rotary tables of
    w4a4_prefix_tables equal PyTorch's evaluation (transformers' rotary
    embedding: fl32(pos * inv_freq), cos / sin on CUDA, rounded to fp16) bit
    for bit, over positions up to 4095."""
    from pi05_pytorch_fast_b200 import prefix_lm as plm

    batch = 3
    pad = torch.ones(batch, seq, dtype=torch.bool, device=DEV)
    pad[0, seq // 2:] = False            # trailing padding
    pad[1, ::7] = False                  # scattered padding
    pad[2, :] = False                    # no real token
    inv_freq = plm.rope_inv_freq(plm.PrefixLMConfig(), fp16_buffer=fp16_freq).to(DEV)
    key_valid = torch.empty(batch, seq, dtype=torch.uint8, device=DEV)
    kv_len = torch.empty(batch, dtype=torch.int32, device=DEV)
    cos = torch.empty(batch * seq, 256, dtype=torch.float16, device=DEV)
    sin = torch.empty_like(cos)
    nat.check(nat.lib().w4a4_prefix_tables(pad.data_ptr(), batch, seq, inv_freq.data_ptr(), 128,
                                           key_valid.data_ptr(), kv_len.data_ptr(), cos.data_ptr(),
                                           sin.data_ptr(), _stream()))
    pos = torch.cumsum(pad.long(), dim=1) - 1
    freqs = pos.reshape(-1, 1).float() * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    torch.cuda.synchronize()
    assert torch.equal(key_valid, pad.to(torch.uint8))
    assert kv_len.tolist() == (pad * torch.arange(1, seq + 1, device=DEV)).amax(dim=1).tolist()
    assert_half_equal(cos, emb.cos().half())
    assert_half_equal(sin, emb.sin().half())
