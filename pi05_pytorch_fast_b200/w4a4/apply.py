"""Install the B200 W4A4 path into a PaliGemma / Gemma prefix language model.

Same public functions, environment knobs and behaviour as the reference's
``pi05_fast/w4a4/apply.py:16-243``:

* ``replace_linears_from_packed`` swaps each packed ``nn.Linear`` for a
  ``W4A4Linear``; gate/up (K=2048, N=16384) are stored fragment-major unless
  ``PI05_W4A4_GATE_PRESHUFFLE=0``, other rows are padded to
  ``K/8 + PI05_W4A4_ROW_PAD_WORDS`` words (default 8) -- both layouts are read
  directly by the sm_100a GEMM's TMA, so no further repack is needed;
* ``fuse_shared_activation_quant`` rebinds attention / MLP forwards so that
  q/k/v share one activation quant (``int4_gemm3``) and gate/up share one
  (``int4_gemm2[_tiled]``), unless ``PI05_W4A4_FUSE_QUANT=0``;
* ``apply_w4a4_from_dir`` loads ``packed.safetensors`` + ``meta.json``
  (format ``embedl-int4-gemm-v1``); ``maybe_apply_w4a4_from_env`` reads
  ``PI05_W4A4_PACK``; ``pack_model_linears`` packs a live model.
"""

from __future__ import annotations

import json
import os
import types
from pathlib import Path
from typing import Iterable

import torch
import torch.nn as nn

from .linear import W4A4Linear
from .pack import pack_linear_weight, preshuffle_wmma_weight, should_rotate

DEFAULT_NAME_PREFIXES = ("paligemma_with_expert.paligemma.model.language_model.layers.",)


def _row_pad_words() -> int:
    return max(1, int(os.environ.get("PI05_W4A4_ROW_PAD_WORDS", "8")))


def _set_module(root: nn.Module, dotted: str, new: nn.Module) -> None:
    parent_name, _, leaf = dotted.rpartition(".")
    parent = root.get_submodule(parent_name) if parent_name else root
    setattr(parent, leaf, new)


def iter_packable_linears(
    model: nn.Module, name_prefixes: Iterable[str] = DEFAULT_NAME_PREFIXES
) -> list[tuple[str, nn.Linear]]:
    """nn.Linear modules under the prefixes whose in_features is a multiple of 64."""
    prefixes = tuple(name_prefixes)
    return [
        (name, mod)
        for name, mod in model.named_modules()
        if isinstance(mod, nn.Linear) and name.startswith(prefixes) and mod.in_features % 64 == 0
    ]


def replace_linears_from_packed(
    model: nn.Module,
    packed: dict[str, torch.Tensor],
    meta_layers: dict[str, dict],
    device: torch.device | None = None,
) -> int:
    """Swap every layer listed in ``meta_layers`` that has ``{name}.packed``."""
    pad_words = _row_pad_words()
    preshuffle_gate_up = os.environ.get("PI05_W4A4_GATE_PRESHUFFLE", "1") != "0"
    count = 0
    for name, spec in meta_layers.items():
        w = packed.get(f"{name}.packed")
        if w is None:
            continue
        k, n = int(spec["in_features"]), int(spec["out_features"])
        fragment_major = (preshuffle_gate_up and name.endswith((".mlp.gate_proj", ".mlp.up_proj"))
                          and k == 2048 and n == 16384)
        if fragment_major:
            w = preshuffle_wmma_weight(w, k)
        elif pad_words > 1 and w.shape[1] == k // 8 + 1:
            w = torch.nn.functional.pad(w, (0, pad_words - 1))
        bias = packed.get(f"{name}.bias")
        if device is not None:
            w = w.to(device)
            bias = None if bias is None else bias.to(device)
        _set_module(model, name, W4A4Linear(w, bias=bias, rotate=spec.get("rotate"),
                                            in_features=k, preshuffled=fragment_major))
        count += 1
    return count


def apply_w4a4_from_dir(model: nn.Module, pack_dir: str | Path) -> int:
    pack_dir = Path(pack_dir).expanduser()
    meta_path, st_path = pack_dir / "meta.json", pack_dir / "packed.safetensors"
    if not meta_path.is_file() or not st_path.is_file():
        raise FileNotFoundError(f"need {meta_path} and {st_path}")
    from safetensors.torch import load_file

    from .extension import preload

    meta = json.loads(meta_path.read_text())
    tensors = load_file(str(st_path))
    device = next(model.parameters()).device
    preload()
    n = replace_linears_from_packed(model, tensors, meta["layers"], device=device)
    n_fused = fuse_shared_activation_quant(model)
    n_frag = sum(isinstance(m, W4A4Linear) and m.preshuffled for m in model.modules())
    print(f"w4a4(b200): replaced {n} Linear modules from {pack_dir}; shared-quant fused "
          f"{n_fused} QKV/MLP groups; row stride pad {_row_pad_words()} word(s); "
          f"fragment-major gate/up {n_frag}", flush=True)
    return n


def _fp16_contiguous(x: torch.Tensor) -> torch.Tensor:
    x = x if x.dtype == torch.float16 else x.to(torch.float16)
    return x if x.is_contiguous() else x.contiguous()


def _fused_mlp_forward(self, x: torch.Tensor) -> torch.Tensor:
    from .extension import int4_gemm, int4_gemm2, int4_gemm2_tiled

    xh = _fp16_contiguous(x)
    pair = int4_gemm2_tiled if (self.gate_proj.preshuffled and self.up_proj.preshuffled) else int4_gemm2
    gate, up = pair(xh, self.gate_proj.packed, self.up_proj.packed)
    h = self.act_fn(gate) * up
    y = int4_gemm(h.contiguous(), self.down_proj.packed)
    return y if y.dtype == x.dtype else y.to(x.dtype)


def _fused_attn_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                        past_key_values=None, **kwargs):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    from transformers.models.gemma.modeling_gemma import apply_rotary_pos_emb, eager_attention_forward

    from .extension import int4_gemm3

    lead = hidden_states.shape[:-1]
    heads_shape = (*lead, -1, self.head_dim)
    q, k, v = int4_gemm3(_fp16_contiguous(hidden_states), self.q_proj.packed,
                         self.k_proj.packed, self.v_proj.packed)
    q = q.view(heads_shape).transpose(1, 2)
    k = k.view(heads_shape).transpose(1, 2)
    v = v.view(heads_shape).transpose(1, 2)
    cos, sin = position_embeddings
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    if past_key_values is not None:
        k, v = past_key_values.update(k, v, self.layer_idx)
    attend = ALL_ATTENTION_FUNCTIONS.get_interface(self.config._attn_implementation,
                                                   eager_attention_forward)
    out, weights = attend(self, q, k, v, attention_mask,
                          dropout=0.0 if not self.training else self.attention_dropout,
                          scaling=self.scaling, **kwargs)
    out = self.o_proj(out.reshape(*lead, -1).contiguous())
    return out, weights


def fuse_shared_activation_quant(model: nn.Module) -> int:
    """Rebind attention and MLP forwards to the shared-quant ops."""
    if os.environ.get("PI05_W4A4_FUSE_QUANT", "1") == "0":
        return 0
    fused = 0
    for mod in model.modules():
        projs = [getattr(mod, a, None) for a in ("q_proj", "k_proj", "v_proj")]
        if all(isinstance(p, W4A4Linear) for p in projs):
            mod.forward = types.MethodType(_fused_attn_forward, mod)
            fused += 1
            continue
        mlp = [getattr(mod, a, None) for a in ("gate_proj", "up_proj", "down_proj")]
        if all(isinstance(p, W4A4Linear) for p in mlp) and hasattr(mod, "act_fn"):
            mod.forward = types.MethodType(_fused_mlp_forward, mod)
            fused += 1
    return fused


def maybe_apply_w4a4_from_env(model: nn.Module) -> int:
    path = os.environ.get("PI05_W4A4_PACK", "").strip()
    return apply_w4a4_from_dir(model, path) if path else 0


def pack_model_linears(
    model: nn.Module, name_prefixes: Iterable[str] = DEFAULT_NAME_PREFIXES
) -> tuple[dict[str, torch.Tensor], dict[str, dict]]:
    """Pack every eligible Linear of a live model (CPU, fp32)."""
    tensors: dict[str, torch.Tensor] = {}
    layers: dict[str, dict] = {}
    for name, lin in iter_packable_linears(model, name_prefixes):
        rot = should_rotate(lin.in_features)
        tensors[f"{name}.packed"] = pack_linear_weight(lin.weight, rotate=rot).contiguous()
        if lin.bias is not None:
            tensors[f"{name}.bias"] = lin.bias.detach().cpu().contiguous()
        layers[name] = {"in_features": lin.in_features, "out_features": lin.out_features,
                        "rotate": rot, "has_bias": lin.bias is not None}
    return tensors, layers
