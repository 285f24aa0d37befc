"""The W4A4 prefix LM on the GPU.

* Every W4A4 op inside a real two-layer forward at M = 776 is bit-exact
  against the CPU oracle fed the same activation: the codes, the row scales
  and the fp16 outputs of q/k/v, o_proj, gate/up and down_proj.
* The whole forward agrees with the reference's own composition -- stock
  transformers Gemma decoder layers (eager attention, fp16) whose seven
  projections are the oracle's W4A4 emulation -- on the real tokens' final
  hidden states.  The two runs round their glue differently (a fused RMSNorm
  summing in another order, another attention kernel schedule), and a
  one-ulp difference in an fp16 activation can move an INT4 code by one
  step, so the check is a tolerance: max |diff| <= 3e-2 x RMS and mean
  |diff| <= 2e-3 x RMS.
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


def reference_forward(hf, model: plm.W4A4PrefixLM, embeds, pad, staging: str):
    """transformers' Gemma layers (stock forward: RMSNorm, RoPE, eager
    attention, GeGLU MLP, residuals) with every projection replaced by the
    oracle over the packed weights ``model`` uses."""
    for layer, lw in zip(hf.layers, model.layers):
        a, m = layer.self_attn, layer.mlp
        a.q_proj, a.k_proj, a.v_proj, a.o_proj = (OracleLinear(w, "row", staging)
                                                  for w in (lw.q, lw.k, lw.v, lw.o))
        m.gate_proj = OracleLinear(lw.gate, "fragment", staging)
        m.up_proj = OracleLinear(lw.up, "fragment", staging)
        m.down_proj = OracleLinear(lw.down, "row", staging)
    pos, mask = plm.prefix_positions_and_mask(pad)
    hidden = embeds
    cos_sin = hf.rotary_emb(hidden, pos)
    for layer in hf.layers:
        hidden = layer(hidden, attention_mask=mask, position_ids=pos, position_embeddings=cos_sin)
        if isinstance(hidden, tuple):
            hidden = hidden[0]
    return hf.norm(hidden)


def test_forward_matches_transformers_layers_with_oracle_projections():
    hf = small_gemma(2, seed=3)
    staging = "fp32"  # the reference's CPU emulation arithmetic, pinned to its golden vectors
    model = plm.W4A4PrefixLM.from_gemma(hf, DEV, staging=STAGINGS[staging])
    embeds, pad = plm.synthetic_prefix(1, device=DEV, seed=4)
    with torch.no_grad():
        ours = model.forward(embeds, pad).hidden
        ref = reference_forward(hf, model, embeds, pad, staging)
    torch.cuda.synchronize()
    real = pad[0]
    a = ours[0][real].float()
    b = ref[0][real].float()
    rms = float(b.pow(2).mean().sqrt())
    diff = (a - b).abs()
    print(f"final hidden: rms {rms:.4f}, max |diff| / rms {float(diff.max()) / rms:.2e}, "
          f"mean |diff| / rms {float(diff.mean()) / rms:.2e}, equal {float((diff == 0).float().mean()):.4f}")
    assert float(diff.max()) <= 3e-2 * rms
    assert float(diff.mean()) <= 2e-3 * rms


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
