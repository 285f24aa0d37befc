"""The W4A4 prefix language model on B200: PaliGemma's Gemma-2B decoder run
over a robot-observation prefix, every projection an INT4 x INT4 GEMM.

This is the caller the reference builds from transformers' Gemma layers and
its own glue (pi05_fast/w4a4/apply.py:126-191: ``_fused_attn_forward`` and
``_fused_mlp_forward`` over ``GemmaDecoderLayer``; the fp16 LM of
pi05_fast/rocm_pi05_optim.py:146-154), designed here around the library's
C ABI instead of modules:

* one preallocated workspace per token count, so a forward allocates
  nothing and captures into one CUDA graph;
* per layer, ten launches, all of this library: residual add + RMSNorm +
  quant (one kernel), the q/k/v GEMM (one launch, three weights), RoPE of q
  and k with the V transpose (one kernel), the tensor-core attention, quant +
  o_proj GEMM, residual add + RMSNorm + quant, the gate/up GEMM, GeGLU +
  quant (one kernel), the down GEMM; the residual add of each sublayer is
  folded into the next norm;
* the keys after RoPE and the values of every layer stay in a KV cache, the
  prefix state the action expert attends to (apply.py:170-171);
* the positions, key mask and rotary tables come from one kernel per
  forward (w4a4_prefix_tables).

Attention is bidirectional over the prefix with the padding mask of lerobot's
``make_att_2d_masks`` (query i sees key j iff both are real tokens; a padded
query sees nothing, so its softmax is uniform over all keys); position ids
are ``cumsum(pad_mask) - 1``.
"""

from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path

import torch

from . import _native as nat
from .shard import MlpShard, exchange_row_blocks, gather_row_blocks
from .w4a4 import pack as wpack

# lerobot's pi05 mask value for disallowed attention pairs (fp32 additive).
MASK_VALUE = -2.3819763e38


@dataclass(frozen=True)
class PrefixLMConfig:
    """Gemma-2B as PaliGemma's language model."""

    hidden: int = 2048
    intermediate: int = 16384
    layers: int = 18
    heads: int = 8
    kv_heads: int = 1
    head_dim: int = 256
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0

    @classmethod
    def from_gemma(cls, cfg) -> "PrefixLMConfig":
        return cls(hidden=cfg.hidden_size, intermediate=cfg.intermediate_size,
                   layers=cfg.num_hidden_layers, heads=cfg.num_attention_heads,
                   kv_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                   rms_eps=cfg.rms_norm_eps,
                   rope_theta=float(getattr(cfg, "rope_theta", None)
                                    or cfg.rope_parameters["rope_theta"]))


@dataclass
class PackedLayer:
    """One decoder layer's weights on the device, in the layouts the GEMM
    reads in place: q/k/v/o/down row-major with rows padded to K/8+8 words,
    gate/up fragment-major (the reference loader's layouts, apply.py:56-69);
    norms as fp32 gains 1 + weight (GemmaRMSNorm's factor)."""

    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    o: torch.Tensor
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    input_gain: torch.Tensor
    post_gain: torch.Tensor


def _gain(weight: torch.Tensor, device) -> torch.Tensor:
    # GemmaRMSNorm multiplies by (1.0 + weight.float()) in fp32
    return (1.0 + weight.detach().to(device).float()).contiguous()


def _row_major(packed: torch.Tensor) -> torch.Tensor:
    k_words = packed.shape[1] - 1
    return wpack.pad_row_words(packed, k_words + wpack.DEFAULT_ROW_PAD_WORDS).contiguous()


def _fragment_major(packed: torch.Tensor, k: int) -> torch.Tensor:
    return wpack.preshuffle_wmma_weight(packed, k).contiguous()


def pack_layer(lin: dict, input_norm: torch.Tensor, post_norm: torch.Tensor, device,
               shard: MlpShard | None = None) -> PackedLayer:
    """PackedLayer from fp weights {q, k, v, o, gate, up, down: [N, K]} (packed on
    ``device`` in fp32, bit-identical to the reference's CPU pack).  With a
    shard, gate/up keep only this rank's rows (each row packs on its own, so
    packing the slice equals slicing the pack)."""
    if shard is not None and shard.world > 1:
        lin = dict(lin)
        cols = shard.cols(lin["gate"].shape[0])
        lin["gate"], lin["up"] = lin["gate"][cols], lin["up"][cols]
    if torch.device(device).type == "cuda":
        # the GPU pack kernel writes each layout directly
        def row(w):
            return wpack.pack_weight_cuda(w, "row", w.shape[1] // 8 + wpack.DEFAULT_ROW_PAD_WORDS, device=device)

        def frag(w):
            return wpack.pack_weight_cuda(w, "fragment", device=device)

        return PackedLayer(q=row(lin["q"]), k=row(lin["k"]), v=row(lin["v"]), o=row(lin["o"]),
                           gate=frag(lin["gate"]), up=frag(lin["up"]), down=row(lin["down"]),
                           input_gain=_gain(input_norm, device), post_gain=_gain(post_norm, device))
    p = {n: wpack.pack_linear_weight(w, device=device) for n, w in lin.items()}
    return PackedLayer(
        q=_row_major(p["q"]), k=_row_major(p["k"]), v=_row_major(p["v"]), o=_row_major(p["o"]),
        gate=_fragment_major(p["gate"], lin["gate"].shape[1]),
        up=_fragment_major(p["up"], lin["up"].shape[1]),
        down=_row_major(p["down"]),
        input_gain=_gain(input_norm, device), post_gain=_gain(post_norm, device))


def layer_from_packed(packed: dict, prefix: str, input_norm: torch.Tensor, post_norm: torch.Tensor,
                      device) -> PackedLayer:
    """PackedLayer from the reference's on-disk pack (``{module}.packed`` int32
    [N, K/8+1] tensors of pack_w4a4_prefix.py:29-78), repacked once at load
    into the layouts above."""
    def get(name):
        return packed[f"{prefix}.{name}.packed"].to(device)

    gate, up = get("mlp.gate_proj"), get("mlp.up_proj")
    return PackedLayer(
        q=_row_major(get("self_attn.q_proj")), k=_row_major(get("self_attn.k_proj")),
        v=_row_major(get("self_attn.v_proj")), o=_row_major(get("self_attn.o_proj")),
        gate=_fragment_major(gate, (gate.shape[1] - 1) * 8),
        up=_fragment_major(up, (up.shape[1] - 1) * 8),
        down=_row_major(get("mlp.down_proj")),
        input_gain=_gain(input_norm, device), post_gain=_gain(post_norm, device))


def rope_inv_freq(cfg: PrefixLMConfig, fp16_buffer: bool = True) -> torch.Tensor:
    """Rotary inverse frequencies as transformers' default rope computes them
    (fp32 on the CPU: 1 / theta ** (arange(0, d, 2) / d)).  With
    ``fp16_buffer`` they are rounded through fp16, as in the reference's fp16
    prefix LM: its cast converts every floating parameter AND buffer of the
    language model, the rotary ``inv_freq`` included
    (pi05_fast/rocm_pi05_optim.py:136-154), and the rotary embedding then
    computes positions x inv_freq.float()."""
    exps = torch.arange(0, cfg.head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** exps)
    return inv.half().float() if fp16_buffer else inv


def prefix_positions_and_mask(pad_mask: torch.Tensor):
    """(position ids int64 [B, L] = cumsum(pad) - 1, additive fp32 mask
    [B, 1, L, L]: 0 where query and key are both real tokens, MASK_VALUE
    elsewhere; lerobot's make_att_2d_masks for an all-bidirectional prefix)."""
    pad = pad_mask.bool()
    pos = torch.cumsum(pad.to(torch.int64), dim=1) - 1
    allowed = pad[:, None, :, None] & pad[:, None, None, :]
    mask = torch.zeros(allowed.shape, dtype=torch.float32, device=pad.device)
    mask.masked_fill_(~allowed, MASK_VALUE)
    return pos, mask


class _Workspace:
    """Every intermediate of one forward at `rows` tokens, allocated once."""

    def __init__(self, cfg: PrefixLMConfig, batch: int, seq: int, device, trace: bool, world: int = 1):
        f16 = dict(dtype=torch.float16, device=device)
        e = torch.empty
        rows = batch * seq
        self.rows = rows
        mlp = cfg.intermediate // world  # gate/up columns held here
        self.x = e((rows, cfg.hidden), **f16)            # residual stream
        self.codes = e((rows, cfg.intermediate), dtype=torch.int8, device=device)
        self.scales = e((rows,), dtype=torch.float32, device=device)
        self.q = e((rows, cfg.heads * cfg.head_dim), **f16)
        self.k = e((rows, cfg.kv_heads * cfg.head_dim), **f16)
        self.attn = e((rows, cfg.heads * cfg.head_dim), **f16)
        self.o = e((rows, cfg.hidden), **f16)
        self.gate = e((rows, mlp), **f16)
        self.up = e((rows, mlp), **f16)
        self.down = e((rows, cfg.hidden), **f16)
        if world > 1:  # the sharded MLP's exchange buffers
            self.h_part = e((rows, mlp), **f16)            # GeGLU of this rank's columns
            self.h_recv = e((world, rows // world, mlp), **f16)  # this rank's rows, by source rank
            self.down_part = e((rows // world, cfg.hidden), **f16)
        self.out = e((rows, cfg.hidden), **f16)
        self.cos = e((rows, cfg.head_dim), **f16)
        self.sin = e((rows, cfg.head_dim), **f16)
        # attention: V transposed per observation, the key mask, real-key spans
        self.vt = e((batch, cfg.head_dim, nat.attn_vt_stride(seq)), **f16)
        self.key_valid = e((batch, seq), dtype=torch.uint8, device=device)
        self.kv_len = e((batch,), dtype=torch.int32, device=device)
        # debug copies of the quantised activations (traces only)
        self.h = e((rows, cfg.hidden), **f16) if trace else None
        self.h_mlp = e((rows, cfg.intermediate), **f16) if trace else None


@dataclass
class PrefixOutput:
    hidden: torch.Tensor          # [B, L, hidden] after the final norm
    keys: list = field(default_factory=list)    # per layer [B, L, kv_heads * head_dim] (after RoPE)
    values: list = field(default_factory=list)  # per layer [B, L, kv_heads * head_dim]


class W4A4PrefixLM:
    """The W4A4 Gemma prefix LM.  ``forward(embeds, pad_mask)`` takes the
    prefix embeddings fp16 [B, L, hidden] and the real-token mask [B, L] on
    the device and returns the final hidden states and the KV cache.

    ``staging`` selects the activation FWHT rounding (the library's
    W4A4_STAGING_*; fp16 = the reference HIP kernel's)."""

    def __init__(self, cfg: PrefixLMConfig, layers: list[PackedLayer], final_norm: torch.Tensor,
                 device, staging: int = nat.STAGING_FP16, inv_freq: torch.Tensor | None = None,
                 shard: MlpShard | None = None):
        if cfg.hidden != 2048 or cfg.intermediate != 16384 or cfg.head_dim != 256:
            raise ValueError("the fused layer kernels are built for Gemma-2B shapes "
                             "(hidden 2048, MLP 16384, head_dim 256)")
        self.cfg = cfg
        self.layers = layers
        self.device = torch.device(device)
        self.final_gain = _gain(final_norm, self.device)
        self.staging = staging
        # the rotary table: the model's own inv_freq buffer when one is given,
        # else the fp16 LM's (rope_inv_freq)
        self.inv_freq = (rope_inv_freq(cfg) if inv_freq is None else inv_freq.detach().float()).to(self.device)
        # the N-sharded gate/up over several GPUs (shard.py), or None
        self.shard = shard if shard is not None and shard.world > 1 else None
        if self.shard is not None and staging != nat.STAGING_FP16:
            raise ValueError("the sharded MLP quantises its segmented rows with fp16 staging only")
        self._ws: dict = {}
        self._lib = nat.lib()
        self._int8: dict = {}  # data_ptr of a packed weight -> its int8 repack (repack_int8)

    # ------------------------------------------------------------- builders
    @classmethod
    def from_gemma(cls, model, device, staging: int = nat.STAGING_FP16,
                   shard: MlpShard | None = None) -> "W4A4PrefixLM":
        """From a transformers GemmaModel (or anything with .layers / .norm of
        Gemma decoder layers): packs every projection; RoPE uses the model's
        own rotary inv_freq buffer (fp16 once the model is cast to fp16)."""
        cfg = PrefixLMConfig.from_gemma(model.config)
        layers = []
        for layer in model.layers:
            a, m = layer.self_attn, layer.mlp
            lin = {"q": a.q_proj.weight, "k": a.k_proj.weight, "v": a.v_proj.weight,
                   "o": a.o_proj.weight, "gate": m.gate_proj.weight, "up": m.up_proj.weight,
                   "down": m.down_proj.weight}
            layers.append(pack_layer({n: w.detach() for n, w in lin.items()},
                                     layer.input_layernorm.weight, layer.post_attention_layernorm.weight,
                                     device, shard))
        rot = getattr(model, "rotary_emb", None)
        inv_freq = getattr(rot, "inv_freq", None)
        return cls(cfg, layers, model.norm.weight, device, staging, inv_freq=inv_freq, shard=shard)

    @classmethod
    def random(cls, cfg: PrefixLMConfig, device, seed: int = 0, std: float = 0.02,
               norm_std: float = 0.1, staging: int = nat.STAGING_FP16,
               shard: MlpShard | None = None) -> "W4A4PrefixLM":
        """Random-init weights N(0, std), norm weights N(0, norm_std), drawn
        and packed on the device (config 2's random-init model; every rank of
        a shard draws the same weights and keeps its gate/up rows)."""
        gen = torch.Generator(device=device).manual_seed(seed)

        def w(n, k):
            return torch.randn(n, k, device=device, generator=gen) * std

        def nw():
            return (torch.randn(cfg.hidden, device=device, generator=gen) * norm_std).half()

        hd = cfg.head_dim
        layers = []
        for _ in range(cfg.layers):
            lin = {"q": w(cfg.heads * hd, cfg.hidden), "k": w(cfg.kv_heads * hd, cfg.hidden),
                   "v": w(cfg.kv_heads * hd, cfg.hidden), "o": w(cfg.hidden, cfg.heads * hd),
                   "gate": w(cfg.intermediate, cfg.hidden), "up": w(cfg.intermediate, cfg.hidden),
                   "down": w(cfg.hidden, cfg.intermediate)}
            layers.append(pack_layer(lin, nw(), nw(), device, shard))
        return cls(cfg, layers, nw(), device, staging, shard=shard)

    @classmethod
    def from_packed_dir(cls, pack_dir, norms: dict, cfg: PrefixLMConfig, device,
                        prefix: str = "paligemma_with_expert.paligemma.model.language_model",
                        staging: int = nat.STAGING_FP16) -> "W4A4PrefixLM":
        """From the reference's on-disk pack (``packed.safetensors`` +
        ``meta.json``, pack_w4a4_prefix.py:73-77; loader apply.py:91-118).
        The pack holds the projections only; ``norms`` maps
        ``layers.{i}.input_layernorm`` / ``layers.{i}.post_attention_layernorm``
        / ``norm`` to the RMSNorm weights."""
        from safetensors.torch import load_file

        pack_dir = Path(pack_dir).expanduser()
        meta = json.loads((pack_dir / "meta.json").read_text())
        if meta.get("format") != "embedl-int4-gemm-v1":
            raise ValueError(f"unknown pack format {meta.get('format')!r}")
        packed = load_file(str(pack_dir / "packed.safetensors"))
        layers = []
        for i in range(cfg.layers):
            p = f"{prefix}.layers.{i}"
            for name in ("self_attn.q_proj", "mlp.down_proj"):
                spec = meta["layers"][f"{p}.{name}"]
                if spec.get("has_bias"):
                    raise ValueError(f"{p}.{name}: biased projections are not part of Gemma")
            layers.append(layer_from_packed(packed, p, norms[f"layers.{i}.input_layernorm"],
                                            norms[f"layers.{i}.post_attention_layernorm"], device))
        return cls(cfg, layers, norms["norm"], device, staging)

    # ------------------------------------------------------------- forward
    def workspace(self, batch: int, seq: int, trace: bool = False) -> _Workspace:
        key = (batch, seq, trace)
        if key not in self._ws:
            world = self.shard.world if self.shard is not None else 1
            if (batch * seq) % world:
                raise ValueError(f"{batch * seq} token rows do not split over {world} ranks")
            self._ws[key] = _Workspace(self.cfg, batch, seq, self.device, trace, world)
        return self._ws[key]

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def repack_int8(self, names=("gate", "up")) -> None:
        """Repack the named projections of every layer once into the int8
        layout (w4a4_repack_int8: 16 x code bytes + scale per row, twice the
        packed bytes), which the GEMM runs on CTA pairs with both operands in
        shared memory.  Results are bit-identical to the packed weights'."""
        for layer in self.layers:
            for name in names:
                w = getattr(layer, name)
                if w.data_ptr() in self._int8:
                    continue
                fragment = name in ("gate", "up")
                k = self.cfg.intermediate if name == "down" else self.cfg.hidden
                dst = torch.empty((int(w.shape[0]), k // 4 + 4), dtype=torch.int32, device=self.device)
                layout = nat.LAYOUT_FRAGMENT_MAJOR if fragment else nat.LAYOUT_ROW_MAJOR
                desc = nat.weights_array([(w.data_ptr(), int(w.shape[0]), int(w.shape[1]), layout)])
                nat.check(self._lib.w4a4_repack_int8(desc, k, dst.data_ptr(), self._stream()))
                self._int8[w.data_ptr()] = dst
        torch.cuda.synchronize(self.device)

    def _gemm(self, ws: _Workspace, rows: int, k: int, weights, outs, fragment: bool) -> None:
        layout = nat.LAYOUT_FRAGMENT_MAJOR if fragment else nat.LAYOUT_ROW_MAJOR
        if self._int8 and all(w.data_ptr() in self._int8 for w in weights):
            weights = [self._int8[w.data_ptr()] for w in weights]
            layout = nat.LAYOUT_INT8
        descs = nat.weights_array([(w.data_ptr(), int(w.shape[0]), int(w.shape[1]), layout)
                                   for w in weights])
        ptrs = nat.pointer_array([o.data_ptr() for o in outs])
        nat.check(self._lib.w4a4_gemm(ws.codes.data_ptr(), ws.scales.data_ptr(), rows, k,
                                      len(weights), descs, ptrs, self._stream()))

    @staticmethod
    def _codes(ws: _Workspace, rows: int, k: int) -> torch.Tensor:
        return ws.codes.view(-1)[: rows * k].view(rows, k)

    def _norm_quant(self, ws: _Workspace, rows: int, delta, gain, trace, x_in=None) -> None:
        h = ws.h if trace is not None else None
        src = ws.x if x_in is None else x_in
        nat.check(self._lib.w4a4_rmsnorm_quant(
            src.data_ptr(), src.stride(0), delta.data_ptr() if delta is not None else None,
            self.cfg.hidden, gain.data_ptr(), self.cfg.rms_eps, ws.x.data_ptr(), ws.x.stride(0),
            h.data_ptr() if h is not None else None, self.cfg.hidden, rows, self.cfg.hidden,
            self.staging, nat.CODES_GEMM, ws.codes.data_ptr(), ws.scales.data_ptr(), self._stream()))

    def forward(self, embeds: torch.Tensor, pad_mask: torch.Tensor, trace: list | None = None,
                out: PrefixOutput | None = None) -> PrefixOutput:
        """embeds fp16 [B, L, hidden], pad_mask bool [B, L] (True = real token),
        both on the device.  With ``trace`` (a list), every W4A4 op's input
        (fp16, the quantised activation) and output are appended as
        (name, layer, input, codes, scales, outputs) for checking."""
        cfg = self.cfg
        b, seq, hidden = embeds.shape
        if hidden != cfg.hidden or embeds.dtype != torch.float16:
            raise ValueError(f"embeds must be fp16 [B, L, {cfg.hidden}]")
        rows = b * seq
        ws = self.workspace(b, seq, trace is not None)
        x_in = embeds.reshape(rows, hidden)
        if not x_in.is_contiguous():
            x_in = x_in.contiguous()
        pad = pad_mask if pad_mask.dtype in (torch.bool, torch.uint8) else pad_mask.bool()
        pad = pad.contiguous()
        lib, st = self._lib, self._stream()
        # positions cumsum(pad) - 1, key mask, real-key spans, rotary tables
        nat.check(lib.w4a4_prefix_tables(pad.data_ptr(), b, seq, self.inv_freq.data_ptr(),
                                         cfg.head_dim // 2, ws.key_valid.data_ptr(), ws.kv_len.data_ptr(),
                                         ws.cos.data_ptr(), ws.sin.data_ptr(), st))
        kv = cfg.kv_heads * cfg.head_dim
        if out is None:
            out = PrefixOutput(hidden=torch.empty_like(embeds),
                               keys=[torch.empty((b, seq, kv), dtype=torch.float16, device=self.device)
                                     for _ in self.layers],
                               values=[torch.empty((b, seq, kv), dtype=torch.float16, device=self.device)
                                       for _ in self.layers])
        hid, inter = cfg.hidden, cfg.intermediate
        delta = None
        for li, lw in enumerate(self.layers):
            k_cache = out.keys[li].view(rows, kv)
            v_cache = out.values[li].view(rows, kv)
            # --- attention block (layer 0's norm reads the embeddings and
            # starts the residual stream)
            self._norm_quant(ws, rows, delta, lw.input_gain, trace, x_in=x_in if li == 0 else None)
            self._gemm(ws, rows, hid, [lw.q, lw.k, lw.v], [ws.q, ws.k, v_cache], fragment=False)
            if trace is not None:
                trace.append(("qkv", li, ws.h.clone(), self._codes(ws, rows, hid).clone(), ws.scales.clone(),
                              (ws.q.clone(), ws.k.clone(), v_cache.clone())))
            # RoPE of q (in place) and k (into the KV cache), V^T, then attention
            nat.check(lib.w4a4_prefix_attention(
                ws.q.data_ptr(), ws.q.stride(0), ws.k.data_ptr(), ws.k.stride(0), v_cache.data_ptr(), kv,
                ws.key_valid.data_ptr(), ws.kv_len.data_ptr(), b, seq, cfg.heads, ws.vt.data_ptr(),
                ws.attn.data_ptr(), ws.attn.stride(0), ws.cos.data_ptr(), ws.sin.data_ptr(),
                k_cache.data_ptr(), kv, st))
            nat.check(lib.w4a4_quant(ws.attn.data_ptr(), rows, cfg.hidden, cfg.hidden, nat.ROTATE_BY_K,
                                     self.staging, nat.CODES_GEMM, ws.codes.data_ptr(),
                                     ws.scales.data_ptr(), st))
            self._gemm(ws, rows, hid, [lw.o], [ws.o], fragment=False)
            if trace is not None:
                trace.append(("o", li, ws.attn.clone(), self._codes(ws, rows, hid).clone(), ws.scales.clone(),
                              (ws.o.clone(),)))
            # --- MLP block (the attention output is added inside the norm)
            self._norm_quant(ws, rows, ws.o, lw.post_gain, trace)
            self._gemm(ws, rows, hid, [lw.gate, lw.up], [ws.gate, ws.up], fragment=True)
            if trace is not None:
                trace.append(("gateup", li, ws.h.clone(), self._codes(ws, rows, hid).clone(), ws.scales.clone(),
                              (ws.gate.clone(), ws.up.clone())))
            if self.shard is not None:
                self._sharded_mlp_tail(ws, rows, lw)
            else:
                h_mlp = ws.h_mlp if trace is not None else None
                nat.check(lib.w4a4_geglu_quant(
                    ws.gate.data_ptr(), ws.up.data_ptr(), rows, cfg.intermediate, cfg.intermediate,
                    self.staging, nat.CODES_GEMM, ws.codes.data_ptr(), ws.scales.data_ptr(),
                    h_mlp.data_ptr() if h_mlp is not None else None, cfg.intermediate, st))
                self._gemm(ws, rows, inter, [lw.down], [ws.down], fragment=False)
                if trace is not None:
                    trace.append(("down", li, ws.h_mlp.clone(), self._codes(ws, rows, inter).clone(),
                                  ws.scales.clone(), (ws.down.clone(),)))
            delta = ws.down
        # final residual add + norm
        nat.check(lib.w4a4_rmsnorm_quant(
            ws.x.data_ptr(), ws.x.stride(0), delta.data_ptr(), cfg.hidden, self.final_gain.data_ptr(),
            cfg.rms_eps, ws.x.data_ptr(), ws.x.stride(0), out.hidden.data_ptr(), cfg.hidden, rows,
            cfg.hidden, self.staging, nat.CODES_GEMM, None, None, st))
        return out

    def _sharded_mlp_tail(self, ws: _Workspace, rows: int, lw: PackedLayer) -> None:
        """GeGLU of this rank's gate/up columns, the row-block exchange, the
        quant of this rank's complete rows from their segments, down_proj on
        them, and the all-gather of the results (shard.py)."""
        sh, cfg, st = self.shard, self.cfg, self._stream()
        part = cfg.intermediate // sh.world
        mine = rows // sh.world
        nat.check(self._lib.w4a4_geglu(ws.gate.data_ptr(), ws.up.data_ptr(), rows, part, part,
                                       ws.h_part.data_ptr(), part, st))
        exchange_row_blocks(ws.h_part, ws.h_recv, sh)
        nat.check(self._lib.w4a4_quant_segments(ws.h_recv.data_ptr(), mine, cfg.intermediate, part, part,
                                                mine * part, self.staging, nat.CODES_GEMM,
                                                ws.codes.data_ptr(), ws.scales.data_ptr(), st))
        self._gemm(ws, mine, cfg.intermediate, [lw.down], [ws.down_part], fragment=False)
        gather_row_blocks(ws.down_part, ws.down, sh)

    __call__ = forward

    def launches_per_forward(self) -> int:
        """Kernels of this library per forward: the prefix tables; per layer 2
        norm+quant, 1 quant, 4 GEMMs, RoPE of q and k + V transpose, attention, 1
        GeGLU+quant (the sharded MLP: GeGLU, then the segment quant); then the
        final norm.  Nothing else runs on the device."""
        return (10 + (1 if self.shard is not None else 0)) * len(self.layers) + 2


class GraphedPrefixLM:
    """A W4A4PrefixLM forward at a fixed (batch, seq) captured in one CUDA
    graph, with static input and output buffers: ``run(embeds, pad_mask)``
    copies the inputs in (host or device tensors), replays the graph and
    returns the static output (valid until the next run)."""

    def __init__(self, model: W4A4PrefixLM, batch: int, seq: int):
        dev = model.device
        self.model = model
        self.embeds = torch.zeros((batch, seq, model.cfg.hidden), dtype=torch.float16, device=dev)
        self.pad = torch.ones((batch, seq), dtype=torch.bool, device=dev)
        kv = model.cfg.kv_heads * model.cfg.head_dim
        self.out = PrefixOutput(
            hidden=torch.empty_like(self.embeds),
            keys=[torch.empty((batch, seq, kv), dtype=torch.float16, device=dev) for _ in model.layers],
            values=[torch.empty((batch, seq, kv), dtype=torch.float16, device=dev) for _ in model.layers])
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                model.forward(self.embeds, self.pad, out=self.out)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            model.forward(self.embeds, self.pad, out=self.out)

    def replay(self) -> None:
        self.graph.replay()

    def run(self, embeds: torch.Tensor, pad_mask: torch.Tensor) -> PrefixOutput:
        self.embeds.copy_(embeds, non_blocking=True)
        self.pad.copy_(pad_mask, non_blocking=True)
        self.graph.replay()
        return self.out


def synthetic_prefix(batch: int, lang_tokens: int = 200, real_lang: int = 52, device="cpu",
                     seed: int = 0, vocab: int = 257152, hidden: int = 2048,
                     embed_table: torch.Tensor | None = None):
    """Config 2's prefix: 3 camera blocks of 256 + 256 + 64 image-token
    embeddings ~ N(0, 1), then ``lang_tokens`` language tokens of which the
    first ``real_lang`` are real ids ~ U[0, vocab) and the rest padding.
    Language embeddings are rows of ``embed_table`` (random N(0, 1) rows
    drawn per id when None) times sqrt(hidden), as Gemma scales them.
    Returns (embeds fp16 [B, L, hidden], pad_mask bool [B, L])."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    n_img = 256 + 256 + 64
    seq = n_img + lang_tokens
    img = torch.randn(batch, n_img, hidden, generator=gen)
    ids = torch.randint(0, vocab, (batch, lang_tokens), generator=gen)
    ids[:, real_lang:] = 0
    if embed_table is None:
        # one N(0,1) row per distinct id: a random-init embedding table sampled lazily
        uniq, inv = torch.unique(ids, return_inverse=True)
        rows = torch.randn(len(uniq), hidden, generator=gen)
        lang = rows[inv]
    else:
        lang = embed_table[ids].float()
    lang = lang * math.sqrt(hidden)
    embeds = torch.cat((img, lang), dim=1).half()
    pad = torch.ones(batch, seq, dtype=torch.bool)
    pad[:, n_img + real_lang:] = False
    return embeds.to(device), pad.to(device)
