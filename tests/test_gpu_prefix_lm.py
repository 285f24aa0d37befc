"""The W4A4 prefix LM on the GPU.

* Every W4A4 op inside a real two-layer forward at M = 776 is bit-exact
  against the CPU oracle fed the same activation: the codes, the row scales
  and the fp16 outputs of q/k/v, o_proj, gate/up and down_proj.
* The fused composition IS transformers' Gemma decoder layer: run through
  the stock layers with the same primitives swapped in, the final hidden
  states are bit-identical.
* Against the stock layers with the reference's eager fp16 attention and the
  oracle's projections, the final hidden states differ by no more than two
  variants of that reference differ from each other (an INT4 code moves one
  step when its fp16 input moves one ulp, so no two roundings agree closely).
* The CUDA-graph replay equals the eager forward bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w4a4_oracle as orc
from pi05_pytorch_fast_b200 import _native as nat
from pi05_pytorch_fast_b200 import prefix_lm as plm
from pi05_pytorch_fast_b200.w4a4 import extension as ext

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
STAGINGS = {"fp16": nat.STAGING_FP16, "fp32": nat.STAGING_FP32}


@pytest.fixture(autouse=True, scope="module")
def _no_device_errors():
    nat.device_error(clear=True)
    yield
    assert nat.device_error(clear=True) == 0, "a kernel's bounded wait ran out"


def small_gemma(layers: int = 2, seed: int = 0):
    """A random-init transformers GemmaModel with config 2's widths (Gemma-2B:
    2048 / 16384, 8 q heads, 1 kv head, head_dim 256), few layers, small
    vocabulary (the prefix is given as embeddings), norm weights N(0, 0.1),
    fp16 on the GPU, eager attention."""
    from transformers import GemmaConfig, GemmaModel

    cfg = GemmaConfig(hidden_size=2048, intermediate_size=16384, num_hidden_layers=layers,
                      num_attention_heads=8, num_key_value_heads=1, head_dim=256, vocab_size=1024,
                      hidden_activation="gelu_pytorch_tanh", rms_norm_eps=1e-6)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = GemmaModel(cfg)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.normal_(0.0, 0.1)
    return model.half().to(DEV).eval()


@pytest.fixture(scope="module")
def gemma2():
    return small_gemma(2)


def gemm_order(codes: np.ndarray) -> np.ndarray:
    m, k = codes.shape
    return np.ascontiguousarray(codes.reshape(m, k // 8, 8)[:, :, list(ext.GEMM_GROUP_ORDER)].reshape(m, k))


WEIGHTS = {"qkv": ("q", "k", "v"), "o": ("o",), "gateup": ("gate", "up"), "down": ("down",)}


@pytest.mark.parametrize("staging", list(STAGINGS))
def test_every_w4a4_op_in_the_forward_is_bit_exact(gemma2, staging):
    model = plm.W4A4PrefixLM.from_gemma(gemma2, DEV, staging=STAGINGS[staging])
    embeds, pad = plm.synthetic_prefix(1, device=DEV, seed=1)
    trace: list = []
    with torch.no_grad():
        model.forward(embeds, pad, trace=trace)
    torch.cuda.synchronize()
    assert [t[0] for t in trace] == ["qkv", "o", "gateup", "down"] * 2
    for name, li, x, codes, scales, outs in trace:
        xn = x.cpu().numpy()
        qa, sa = orc.quant_activation(xn, rotate=True, staging=staging)
        np.testing.assert_array_equal(codes.cpu().numpy(), gemm_order(qa), err_msg=f"{name}{li} codes")
        np.testing.assert_array_equal(scales.cpu().numpy().view(np.int32), sa.view(np.int32),
                                      err_msg=f"{name}{li} scales")
        lw = model.layers[li]
        for wname, y in zip(WEIGHTS[name], outs):
            w = getattr(lw, wname).cpu().numpy()
            layout = "fragment" if wname in ("gate", "up") else "row"
            ref = orc.int4_gemm_ref(xn, w, rotate=True, staging=staging, layout=layout)
            np.testing.assert_array_equal(y.cpu().numpy().view(np.uint16), ref.view(np.uint16),
                                          err_msg=f"{name}{li} {wname}")


class OracleLinear(torch.nn.Module):
    """A projection computed by the CPU oracle's W4A4 emulation of the same
    packed weight (int4_gemm_ref): quant, exact integer GEMM, dequant."""

    def __init__(self, packed: torch.Tensor, layout: str, staging: str):
        super().__init__()
        self.packed = packed.cpu().numpy()
        self.layout, self.staging = layout, staging

    def forward(self, x):
        y = orc.int4_gemm_ref(x.detach().cpu().numpy(), self.packed, rotate=True,
                              staging=self.staging, layout=self.layout)
        return torch.from_numpy(y).to(x.device)


class OpLinear(torch.nn.Module):
    """A projection through the pi05_w4a4 torch ops (what the reference's
    W4A4Linear calls), on the same packed weight."""

    def __init__(self, packed: torch.Tensor, fragment: bool):
        super().__init__()
        self.packed, self.fragment = packed, fragment

    def forward(self, x):
        op = torch.ops.pi05_w4a4.int4_gemm_tiled if self.fragment else torch.ops.pi05_w4a4.int4_gemm
        return op(x.contiguous(), self.packed)


class LibRMSNorm(torch.nn.Module):
    """GemmaRMSNorm through the library's norm kernel (w4a4_rmsnorm_quant
    without the quant): the norm the runner's fused kernels compute."""

    def __init__(self, weight: torch.Tensor, eps: float):
        super().__init__()
        self.gain = (1.0 + weight.detach().float()).contiguous()
        self.eps = eps

    def forward(self, x):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        h = torch.empty_like(x2)
        nat.check(nat.lib().w4a4_rmsnorm_quant(
            x2.data_ptr(), x2.stride(0), None, 0, self.gain.data_ptr(), self.eps, None, 0, h.data_ptr(),
            h.stride(0), x2.shape[0], x2.shape[1], 0, nat.CODES_INT8, None, None,
            torch.cuda.current_stream().cuda_stream))
        return h.view_as(x)


def library_attention(pad):
    """transformers attention function running the library's prefix
    attention kernel under the prefix mask of ``pad``."""
    def attn(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
        b, h, seq, d = query.shape
        q = query.transpose(1, 2).reshape(b * seq, h * d).contiguous()
        k = key.transpose(1, 2).reshape(b * seq, d).contiguous()
        v = value.transpose(1, 2).reshape(b * seq, d).contiguous()
        kvalid = pad.to(torch.uint8).contiguous()
        kv_len = (pad * torch.arange(1, seq + 1, device=pad.device)).amax(dim=1).to(torch.int32)
        vt = torch.empty((b, d, nat.attn_vt_stride(seq)), dtype=torch.float16, device=q.device)
        out = torch.empty_like(q)
        nat.check(nat.lib().w4a4_prefix_attention(
            q.data_ptr(), q.stride(0), k.data_ptr(), d, v.data_ptr(), d, kvalid.data_ptr(), kv_len.data_ptr(),
            b, seq, h, vt.data_ptr(), out.data_ptr(), out.stride(0), None, None, None, 0,
            torch.cuda.current_stream().cuda_stream))
        return out.view(b, seq, h, d), None
    return attn


def eager_fp32_attention(module, query, key, value, attention_mask, scaling=None, dropout=0.0, **kwargs):
    """transformers' eager attention evaluated in fp32, rounded to fp16 once."""
    from transformers.models.gemma.modeling_gemma import repeat_kv

    k = repeat_kv(key, module.num_key_value_groups).float()
    v = repeat_kv(value, module.num_key_value_groups).float()
    w = torch.matmul(query.float(), k.transpose(2, 3)) * module.scaling + attention_mask
    w = torch.softmax(w, dim=-1, dtype=torch.float32)
    return torch.matmul(w, v).transpose(1, 2).contiguous().half(), None


def hf_forward(hf, embeds, pad, attn_impl: str):
    """Stock transformers Gemma decoder layers (input norm, attention with
    RoPE, residual, post-attention norm, GeGLU MLP, residual) and final norm."""
    pos, mask = plm.prefix_positions_and_mask(pad)
    hf.config._attn_implementation = attn_impl
    hidden = embeds
    cos_sin = hf.rotary_emb(hidden, pos)
    for layer in hf.layers:
        hidden = layer(hidden, attention_mask=mask, position_ids=pos, position_embeddings=cos_sin)
        if isinstance(hidden, tuple):
            hidden = hidden[0]
    return hf.norm(hidden)


def install_projections(hf, model: plm.W4A4PrefixLM, make):
    for layer, lw in zip(hf.layers, model.layers):
        a, m = layer.self_attn, layer.mlp
        a.q_proj, a.k_proj, a.v_proj, a.o_proj = (make(w, False) for w in (lw.q, lw.k, lw.v, lw.o))
        m.gate_proj, m.up_proj = make(lw.gate, True), make(lw.up, True)
        m.down_proj = make(lw.down, False)


def test_fused_forward_equals_transformers_layers_on_the_same_primitives():
    """The runner's fused composition is exactly transformers' Gemma decoder
    layer (the reference's _fused_attn_forward / _fused_mlp_forward), bit for
    bit, once both use the same primitives: the pi05_w4a4 ops for the seven
    projections, this library's norm and attention kernels; RoPE, GeGLU and
    the residual adds stay transformers' / PyTorch's own (the fused kernels
    round them identically)."""
    from transformers import AttentionInterface

    hf = small_gemma(2, seed=3)
    model = plm.W4A4PrefixLM.from_gemma(hf, DEV)
    embeds, pad = plm.synthetic_prefix(1, device=DEV, seed=4)
    with torch.no_grad():
        ours = model.forward(embeds, pad).hidden.clone()
        install_projections(hf, model, lambda w, frag: OpLinear(w, frag))
        for layer in hf.layers:
            layer.input_layernorm = LibRMSNorm(layer.input_layernorm.weight, 1e-6)
            layer.post_attention_layernorm = LibRMSNorm(layer.post_attention_layernorm.weight, 1e-6)
        hf.norm = LibRMSNorm(hf.norm.weight, 1e-6)
        AttentionInterface.register("w4a4_prefix_test", library_attention(pad))
        ref = hf_forward(hf, embeds, pad, "w4a4_prefix_test")
    torch.cuda.synchronize()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16))


def test_forward_stays_within_the_references_own_rounding_spread():
    """Against the stock composition with the reference's eager fp16
    attention and the oracle's W4A4 projections: INT4 activation codes move
    by one step when an fp16 input moves by one ulp, so any two correct
    roundings of this model differ visibly.  The runner's distance from the
    eager-fp16 reference must stay within 2x the distance between two
    reference variants (eager attention in fp16 vs in fp32)."""
    from transformers import AttentionInterface

    hf = small_gemma(2, seed=3)
    staging = "fp32"  # the reference's CPU emulation arithmetic, pinned to its golden vectors
    model = plm.W4A4PrefixLM.from_gemma(hf, DEV, staging=STAGINGS[staging])
    embeds, pad = plm.synthetic_prefix(1, device=DEV, seed=4)
    with torch.no_grad():
        ours = model.forward(embeds, pad).hidden.clone()
        install_projections(hf, model, lambda w, frag: OracleLinear(w, "fragment" if frag else "row", staging))
        ref16 = hf_forward(hf, embeds, pad, "eager")
        AttentionInterface.register("eager_fp32_test", eager_fp32_attention)
        ref32 = hf_forward(hf, embeds, pad, "eager_fp32_test")
    torch.cuda.synchronize()
    real = pad[0]
    a, r16, r32 = (t[0][real].float() for t in (ours, ref16, ref32))
    rms = float(r16.pow(2).mean().sqrt())
    ours_d = (a - r16).abs()
    spread = (r32 - r16).abs()
    print(f"final hidden vs eager-fp16 reference: ours mean {float(ours_d.mean()) / rms:.2e} "
          f"max {float(ours_d.max()) / rms:.2e}; fp32-attention reference mean "
          f"{float(spread.mean()) / rms:.2e} max {float(spread.max()) / rms:.2e}")
    assert float(ours_d.mean()) <= 2.0 * float(spread.mean()) + 1e-4 * rms
    assert float(ours_d.max()) <= 2.0 * float(spread.max()) + 1e-3 * rms


def test_model_from_the_references_on_disk_pack(gemma2, tmp_path):
    """The reference's offline pack (pack_w4a4_prefix.py: packed.safetensors
    with `{module}.packed` int32 [N, K/8+1] tensors, meta.json with the
    embedl-int4-gemm-v1 format) loads through from_packed_dir, is repacked
    once into the GEMM's layouts and gives the same forward as packing the
    model directly."""
    import json

    from safetensors.torch import save_file

    from pi05_pytorch_fast_b200.w4a4.pack import pack_linear_weight

    prefix = "paligemma_with_expert.paligemma.model.language_model"
    tensors, layers, norms = {}, {}, {}
    for i, layer in enumerate(gemma2.layers):
        mods = {"self_attn.q_proj": layer.self_attn.q_proj, "self_attn.k_proj": layer.self_attn.k_proj,
                "self_attn.v_proj": layer.self_attn.v_proj, "self_attn.o_proj": layer.self_attn.o_proj,
                "mlp.gate_proj": layer.mlp.gate_proj, "mlp.up_proj": layer.mlp.up_proj,
                "mlp.down_proj": layer.mlp.down_proj}
        for name, lin in mods.items():
            key = f"{prefix}.layers.{i}.{name}"
            tensors[key + ".packed"] = pack_linear_weight(lin.weight).contiguous()
            layers[key] = {"in_features": lin.in_features, "out_features": lin.out_features,
                           "rotate": True, "has_bias": False}
        norms[f"layers.{i}.input_layernorm"] = layer.input_layernorm.weight
        norms[f"layers.{i}.post_attention_layernorm"] = layer.post_attention_layernorm.weight
    norms["norm"] = gemma2.norm.weight
    save_file(tensors, str(tmp_path / "packed.safetensors"))
    (tmp_path / "meta.json").write_text(json.dumps({"format": "embedl-int4-gemm-v1", "layers": layers}))
    cfg = plm.PrefixLMConfig.from_gemma(gemma2.config)
    loaded = plm.W4A4PrefixLM.from_packed_dir(tmp_path, norms, cfg, DEV)
    direct = plm.W4A4PrefixLM.from_gemma(gemma2, DEV)
    assert torch.equal(loaded.layers[0].gate, direct.layers[0].gate)
    assert torch.equal(loaded.layers[1].q, direct.layers[1].q)
    embeds, pad = plm.synthetic_prefix(1, device=DEV, seed=9)
    with torch.no_grad():
        a = loaded.forward(embeds, pad).hidden.clone()
        b = direct.forward(embeds, pad).hidden.clone()
    torch.cuda.synchronize()
    # from_packed_dir has no rotary buffer to read: the fp16 LM's table, as
    # from_gemma takes from the fp16 model
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_graph_replay_equals_eager_forward(gemma2):
    model = plm.W4A4PrefixLM.from_gemma(gemma2, DEV)
    embeds, pad = plm.synthetic_prefix(2, device=DEV, seed=7)
    with torch.no_grad():
        eager = model.forward(embeds, pad)
        eager_h = eager.hidden.clone()
        eager_k = [k.clone() for k in eager.keys]
        g = plm.GraphedPrefixLM(model, batch=2, seq=embeds.shape[1])
        out = g.run(embeds, pad)
    torch.cuda.synchronize()
    assert torch.equal(out.hidden.view(torch.int16), eager_h.view(torch.int16))
    for k1, k2 in zip(out.keys, eager_k):
        assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))


@pytest.mark.parametrize("lang_tokens", [64, 192, 200])  # prefixes of 640, 768 and 776 tokens
def test_batched_forward_equals_each_observation_alone(gemma2, lang_tokens):
    """Observations of one batch do not influence each other: a batch of
    three (with 1, 40 and all real language tokens) gives, row for row, the
    bits of each observation run alone -- every kernel works per row or per
    observation, and an integer GEMM's outputs depend only on their row and
    column, whatever the token tiles of the launch."""
    model = plm.W4A4PrefixLM.from_gemma(gemma2, DEV)
    embeds, pad = plm.synthetic_prefix(3, lang_tokens=lang_tokens, device=DEV, seed=11)
    n_img = 576
    pad[0, n_img + 1:] = False
    pad[1, n_img + 40:] = False
    pad[2, n_img:] = True
    with torch.no_grad():
        both = model.forward(embeds, pad)
        hb = both.hidden.clone()
        kb = [k.clone() for k in both.keys]
        for i in range(3):
            one = model.forward(embeds[i:i + 1].contiguous(), pad[i:i + 1].contiguous())
            torch.cuda.synchronize()
            assert torch.equal(one.hidden.view(torch.int16), hb[i:i + 1].view(torch.int16)), i
            for k1, k2 in zip(one.keys, kb):
                assert torch.equal(k1.view(torch.int16), k2[i:i + 1].view(torch.int16)), i


def test_forward_with_int8_repacked_weights_is_bit_identical(gemma2):
    """repack_int8 (the int8 layout run by the SS CTA-pair GEMM) for every
    projection changes no bit of the forward."""
    model = plm.W4A4PrefixLM.from_gemma(gemma2, DEV)
    embeds, pad = plm.synthetic_prefix(2, device=DEV, seed=5)
    with torch.no_grad():
        ref = model.forward(embeds, pad).hidden.clone()
        model.repack_int8(("q", "k", "v", "o", "gate", "up", "down"))
        got = model.forward(embeds, pad).hidden.clone()
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
