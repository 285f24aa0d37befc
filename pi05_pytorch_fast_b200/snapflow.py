"""Config 4: one pi0.5 SnapFlow 1-NFE action chunk around the W4A4 prefix LM.

The reference runs this step through lerobot's ``PI05Pytorch`` with the
SnapFlow student subclass (pi05_fast/snapflow_pi05.py:127-195:
``sample_actions_1step`` -> ``embed_prefix`` -> prefix LM with a KV cache ->
``denoise_step`` at time 1 with the target-time MLP -> ``x_t - v_t``) and the
batched SigLIP prefix of pi05_fast/rocm_pi05_optim.py:88-133 (the real
cameras through SigLIP in one batch; the empty camera is a constant -1 image
whose embedding is computed once and sum-pooled 4:1 to 64 tokens, so the
prefix is 256 + 256 + 64 image tokens + 200 language tokens = 776).  The
prefix LM runs fp16 (rocm_pi05_optim.py:146-154); SigLIP and the action
expert run bf16.

lerobot is not part of the reference, so the neighbours of the W4A4 path are
rebuilt here from their published structure, with random weights:

* SigLIP-So400m (width 1152, 27 layers, 16 heads, MLP 4304, patch 14 at
  224 x 224 -> 256 tokens, no pooling head): ``SiglipTower``, the
  computation of transformers' ``SiglipVisionModel`` with fewer launches
  (it loads that model's weights), and PaliGemma's multi-modal projector
  (1152 -> 2048), bf16 through cuBLAS and PyTorch's SDPA;
* the language embedding table (257,152 x 2048) scaled by sqrt(2048), as
  Gemma scales embeddings;
* the W4A4 prefix LM of this package (``prefix_lm.W4A4PrefixLM``), whose
  per-layer keys (after RoPE) and values are the expert's prefix KV cache,
  cast to bf16 as ``clone_kv_cache(..., dtype=expert dtype)`` does
  (snapflow_pi05.py:155-157);
* the Gemma-300M action expert (width 1024, 18 layers, MLP 4096 GeGLU, 8
  query heads / 1 KV head, head_dim 256) with pi0.5's adaptive RMSNorm (scale,
  shift and a residual gate from the time condition); its 50 action tokens
  attend to every real prefix token and to each other (the suffix attention
  mask [1, 0, ..., 0] of snapflow_pi05.py:114 makes one bidirectional block),
  at positions ``sum(prefix mask) + i`` (snapflow_pi05.py:150-151);
* the suffix embedding of snapflow_pi05.py:67-116: the sinusoidal time
  embedding (periods log-spaced from min_period to max_period), plus the
  SnapFlow target-time MLP (Linear, SiLU, Linear) of the target time, then
  the time MLP (Linear, SiLU, Linear, SiLU) -> the adaptive-norm condition;
  ``action_in_proj`` / ``action_out_proj`` (32 <-> 1024).

The exact lerobot module layout (and so a checkpoint's tensor names) is not
reproduced; shapes, dtypes, masks, positions and the order of operations
are.  ``GraphedSnapFlow`` captures the whole step (SigLIP, the prefix
assembly, the W4A4 prefix LM, the expert) in one CUDA graph.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from . import _native as nat
from . import prefix_lm as plm


@dataclass(frozen=True)
class SnapFlowConfig:
    """BASELINE config 4's shapes."""

    # SigLIP-So400m
    vision_hidden: int = 1152
    vision_intermediate: int = 4304
    vision_layers: int = 27
    vision_heads: int = 16
    image_size: int = 224
    patch: int = 14
    real_cameras: int = 2
    empty_pool: int = 4          # the empty camera's 256 tokens sum-pooled 4:1 -> 64
    # language
    lang_tokens: int = 200
    vocab: int = 257152
    # the W4A4 prefix LM (Gemma-2B)
    lm: plm.PrefixLMConfig = field(default_factory=plm.PrefixLMConfig)
    # the action expert (Gemma-300M)
    expert_hidden: int = 1024
    expert_intermediate: int = 4096
    expert_layers: int = 18
    expert_heads: int = 8
    expert_kv_heads: int = 1
    head_dim: int = 256
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    # the flow step
    chunk: int = 50
    action_dim: int = 32
    min_period: float = 4e-3
    max_period: float = 4.0

    @property
    def image_tokens(self) -> int:
        return (self.image_size // self.patch) ** 2

    @property
    def prefix_len(self) -> int:
        return self.real_cameras * self.image_tokens + self.image_tokens // self.empty_pool + self.lang_tokens


def sinusoidal_time_embedding(t: torch.Tensor, dim: int, min_period: float, max_period: float) -> torch.Tensor:
    """[B] times -> [B, dim]: sin and cos of t * 2 pi / period for dim / 2
    periods spaced geometrically from min_period to max_period (computed in
    float64, returned float32)."""
    if dim % 2:
        raise ValueError("dim must be even")
    frac = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64, device=t.device)
    period = min_period * (max_period / min_period) ** frac
    arg = (2.0 * math.pi / period)[None, :] * t.to(torch.float64)[:, None]
    return torch.cat((torch.sin(arg), torch.cos(arg)), dim=1).float()


def pool_tokens(emb: torch.Tensor, pool: int) -> torch.Tensor:
    """[B, T, D] -> [B, T / pool, D]: the sum of each run of `pool`
    consecutive tokens (the empty camera's 4:1 pool)."""
    b, t, d = emb.shape
    if t % pool:
        raise ValueError(f"{t} tokens do not pool {pool}:1")
    return emb.reshape(b, t // pool, pool, d).sum(dim=2)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """positions [B, S] -> cos, sin [B, 1, S, head_dim] (fp32 angles, cast to
    dtype), the rotary tables of transformers' Gemma."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=positions.device) / head_dim))
    ang = positions.float()[..., None] * inv
    emb = torch.cat((ang, ang), dim=-1)[:, None]
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _on_kernels(x: torch.Tensor) -> bool:
    """bf16 CUDA tensors go through the library's neighbour kernels; the
    PyTorch forms below serve CPU tensors (the small-shape CPU tests)."""
    return x.is_cuda and x.dtype == torch.bfloat16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ada_rms_norm(x: torch.Tensor, mod: tuple, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """pi0.5's adaptive RMSNorm: mod = (1 + scale, shift) in fp32 and gate,
    each [B, h], from a Linear of the flow-time condition; y = rms_norm(x) *
    (1 + scale) + shift in fp32, cast back to x's dtype; the gate multiplies
    the sublayer's output on the residual.  x [B, S, h]."""
    scale1, shift, gate = mod
    if _on_kernels(x):
        b, s, h = x.shape
        x = x.contiguous()
        y = torch.empty_like(x)
        nat.check(nat.lib().w4a4_ada_rms_norm_bf16(x.data_ptr(), y.data_ptr(), b * s, h, s, scale1.data_ptr(),
                                                   shift.data_ptr(), scale1.stride(0), eps, _stream()))
        return y, gate[:, None]
    y = F.rms_norm(x.float(), (x.shape[-1],), eps=eps)
    return torch.addcmul(shift[:, None], y, scale1[:, None]).to(x.dtype), gate[:, None]


def layer_norm(ln: nn.LayerNorm, x: torch.Tensor) -> torch.Tensor:
    """``ln(x)``, through the library's LayerNorm kernel for bf16 on CUDA."""
    if _on_kernels(x) and x.shape[-1] % 8 == 0 and x.shape[-1] <= 2048:
        x = x.contiguous()
        y = torch.empty_like(x)
        h = x.shape[-1]
        nat.check(nat.lib().w4a4_layer_norm_bf16(x.data_ptr(), y.data_ptr(), x.numel() // h, h,
                                                 ln.weight.data_ptr(), ln.bias.data_ptr(), ln.eps, _stream()))
        return y
    return ln(x)


def signed_sin(sin: torch.Tensor) -> torch.Tensor:
    """sin with its first half (over the last dim) negated: rotate_half(x) *
    sin == roll(x, half) * signed_sin(sin)."""
    h = sin.shape[-1] // 2
    return torch.cat((-sin[..., :h], sin[..., h:]), dim=-1)


class ExpertLayer(nn.Module):
    """One Gemma-300M decoder layer of the action expert with adaptive norms;
    attention over [prefix KV cache ; own keys] as transformers' eager
    attention computes it (bf16 scores with the additive mask, softmax in
    fp32, rounded to bf16, times V), the query heads of a KV head stacked
    as rows of one matrix product."""

    def __init__(self, cfg: SnapFlowConfig):
        super().__init__()
        h, hd = cfg.expert_hidden, cfg.head_dim
        self.heads, self.kv_heads, self.hd, self.eps = cfg.expert_heads, cfg.expert_kv_heads, hd, cfg.rms_eps
        self.q = nn.Linear(h, self.heads * hd, bias=False)
        self.k = nn.Linear(h, self.kv_heads * hd, bias=False)
        self.v = nn.Linear(h, self.kv_heads * hd, bias=False)
        self.o = nn.Linear(self.heads * hd, h, bias=False)
        self.gate = nn.Linear(h, cfg.expert_intermediate, bias=False)
        self.up = nn.Linear(h, cfg.expert_intermediate, bias=False)
        self.down = nn.Linear(cfg.expert_intermediate, h, bias=False)

    def forward(self, x, mod_in, mod_post, rope, prefix_k, prefix_v, mask_add):
        """x [B, S, h]; mod_* (1 + scale, shift, gate) of the two norms (see
        ``ada_rms_norm``); rope = (cos, sin) [B * S, hd] for the RoPE kernel,
        or on CPU (cos, sin with its first half negated (``signed_sin``)), each
        [B, S, 1, hd]; prefix_k / prefix_v [B, kv_heads, L, hd] (keys after
        RoPE); mask_add [B, 1, L + S] (0 or the dtype's lowest value)."""
        b, s, _ = x.shape
        kvh, g, hd = self.kv_heads, self.heads // self.kv_heads, self.hd
        n, g1 = ada_rms_norm(x, mod_in, self.eps)
        q, k, v = self.q(n), self.k(n), self.v(n)
        if _on_kernels(q):
            # q and k rotated in place (the Linear outputs are contiguous rows)
            nat.check(nat.lib().w4a4_rope_qk_bf16(q.data_ptr(), self.heads * hd, self.heads, k.data_ptr(),
                                                  kvh * hd, kvh, rope[0].data_ptr(), rope[1].data_ptr(), b * s,
                                                  hd, _stream()))
            q, k = q.view(b, s, self.heads, hd), k.view(b, s, kvh, hd)
        else:
            # x cos + rotate_half(x) sin, with rotate_half(x) = roll(x, hd / 2)
            # times the sign carried by sin (negated first half)
            cos, sin = rope
            q, k = q.view(b, s, self.heads, hd), k.view(b, s, kvh, hd)
            q = torch.addcmul(q * cos, torch.roll(q, hd // 2, dims=-1), sin)
            k = torch.addcmul(k * cos, torch.roll(k, hd // 2, dims=-1), sin)
        v = v.view(b, s, kvh, hd)
        # rows (KV head, query head of the group, token); keys [prefix ; suffix]
        q = q.view(b, s, kvh, g, hd).permute(0, 2, 3, 1, 4).reshape(b * kvh, g * s, hd)
        k = torch.cat((prefix_k, k.transpose(1, 2)), dim=2).view(b * kvh, -1, hd)
        v = torch.cat((prefix_v, v.transpose(1, 2)), dim=2).view(b * kvh, -1, hd)
        mask = mask_add if kvh == 1 else mask_add.repeat_interleave(kvh, dim=0)
        scores = torch.baddbmm(mask, q, k.transpose(1, 2), alpha=hd ** -0.5)
        p = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q.dtype)
        a = torch.bmm(p, v).view(b, kvh, g, s, hd).permute(0, 3, 1, 2, 4).reshape(b, s, self.heads * hd)
        x = torch.addcmul(x, g1, self.o(a))
        n, g2 = ada_rms_norm(x, mod_post, self.eps)
        return torch.addcmul(x, g2, self.down(F.gelu(self.gate(n), approximate="tanh") * self.up(n)))


class ActionExpert(nn.Module):
    """The suffix path of the SnapFlow step: time embedding (+ target-time
    MLP), the time MLP -> condition, action_in_proj, the expert layers over
    the prefix KV cache, the final adaptive norm and action_out_proj.  The
    [scale, shift, gate] of all 2 x layers + 1 adaptive norms come from one
    Linear of the condition (``modulation``: norm i's at rows 3 h i ..)."""

    def __init__(self, cfg: SnapFlowConfig):
        super().__init__()
        h = cfg.expert_hidden
        self.cfg = cfg
        self.action_in_proj = nn.Linear(cfg.action_dim, h)
        self.action_out_proj = nn.Linear(h, cfg.action_dim)
        self.time_mlp_in = nn.Linear(h, h)
        self.time_mlp_out = nn.Linear(h, h)
        hid = max(h, 256)
        self.target_time_mlp = nn.Sequential(nn.Linear(h, hid), nn.SiLU(), nn.Linear(hid, h))
        self.layers = nn.ModuleList(ExpertLayer(cfg) for _ in range(cfg.expert_layers))
        self.n_norms = 2 * cfg.expert_layers + 1
        self.modulation = nn.Linear(h, self.n_norms * 3 * h)

    def condition(self, t: torch.Tensor, target_t: torch.Tensor | None) -> torch.Tensor:
        cfg, dt = self.cfg, self.time_mlp_in.weight.dtype
        emb = sinusoidal_time_embedding(t, cfg.expert_hidden, cfg.min_period, cfg.max_period).to(dt)
        if target_t is not None:
            tt = sinusoidal_time_embedding(target_t, cfg.expert_hidden, cfg.min_period, cfg.max_period)
            emb = emb + self.target_time_mlp(tt.to(dt))
        return F.silu(self.time_mlp_out(F.silu(self.time_mlp_in(emb))))

    def forward(self, x_t, t, target_t, prefix_pad, keys, values) -> torch.Tensor:
        """x_t [B, chunk, action_dim] in the expert's dtype; prefix_pad bool
        [B, L]; keys / values: per layer [B, L, kv_heads * hd] (any float
        dtype).  Returns v_t [B, chunk, action_dim] in the expert's dtype."""
        cfg = self.cfg
        dt = self.action_in_proj.weight.dtype
        b, s, h = x_t.shape[0], cfg.chunk, cfg.expert_hidden
        mods = self.modulation(self.condition(t, target_t)).view(b, self.n_norms, 3, h)
        # every norm's (1 + scale, shift) in fp32 at once, and its gate
        scale1 = (mods[:, :, 0].float() + 1.0).contiguous()
        shift, gate = mods[:, :, 1].float().contiguous(), mods[:, :, 2]
        mod = [(scale1[:, i], shift[:, i], gate[:, i]) for i in range(self.n_norms)]
        x = self.action_in_proj(x_t)
        # suffix positions continue after the real prefix tokens
        pos = prefix_pad.sum(dim=1, keepdim=True) + torch.arange(s, device=x.device)[None, :]
        cos, sin = rope_tables(pos, cfg.head_dim, cfg.rope_theta, dt)
        if _on_kernels(x):
            rope = (cos[:, 0].reshape(b * s, cfg.head_dim).contiguous(),
                    sin[:, 0].reshape(b * s, cfg.head_dim).contiguous())
        else:
            rope = (cos.transpose(1, 2), signed_sin(sin.transpose(1, 2)))
        # the prefix's real tokens and every suffix token are visible
        visible = torch.cat((prefix_pad, torch.ones((b, s), dtype=torch.bool, device=x.device)), dim=1)
        mask_add = torch.zeros(visible.shape, dtype=dt, device=x.device).masked_fill_(
            ~visible, torch.finfo(dt).min)[:, None, :]
        kvh, hd = cfg.expert_kv_heads, cfg.head_dim
        for i, (layer, k, v) in enumerate(zip(self.layers, keys, values)):
            pk = k.view(b, -1, kvh, hd).transpose(1, 2).to(dt)
            pv = v.view(b, -1, kvh, hd).transpose(1, 2).to(dt)
            x = layer(x, mod[2 * i], mod[2 * i + 1], rope, pk, pv, mask_add)
        x, _ = ada_rms_norm(x, mod[-1], cfg.rms_eps)
        return self.action_out_proj(x[:, -s:])


class SiglipTower(nn.Module):
    """SigLIP vision encoder without the pooling head, the computation of
    transformers' ``SiglipVisionModel`` (patch convolution, position
    embedding, pre-norm layers: LayerNorm -> attention -> residual, LayerNorm
    -> fc1 -> tanh GELU -> fc2 -> residual, final LayerNorm) laid out for
    fewer launches: the residual stream token-major from the patch
    embedding on, and q, k and v from one GEMM whose output is viewed as
    [N, T, 3, heads, d] and handed to scaled-dot-product attention as strided
    views."""

    def __init__(self, cfg: SnapFlowConfig, eps: float = 1e-6):
        super().__init__()
        h, self.heads = cfg.vision_hidden, cfg.vision_heads
        self.patch = nn.Conv2d(3, h, kernel_size=cfg.patch, stride=cfg.patch)
        self.pos = nn.Parameter(torch.zeros(cfg.image_tokens, h))
        self.ln1 = nn.ModuleList(nn.LayerNorm(h, eps=eps) for _ in range(cfg.vision_layers))
        self.qkv = nn.ModuleList(nn.Linear(h, 3 * h) for _ in range(cfg.vision_layers))
        self.out = nn.ModuleList(nn.Linear(h, h) for _ in range(cfg.vision_layers))
        self.ln2 = nn.ModuleList(nn.LayerNorm(h, eps=eps) for _ in range(cfg.vision_layers))
        self.fc1 = nn.ModuleList(nn.Linear(h, cfg.vision_intermediate) for _ in range(cfg.vision_layers))
        self.fc2 = nn.ModuleList(nn.Linear(cfg.vision_intermediate, h) for _ in range(cfg.vision_layers))
        self.post_ln = nn.LayerNorm(h, eps=eps)

    @torch.no_grad()
    def load_transformers(self, model) -> "SiglipTower":
        """Copies the weights of a transformers ``SiglipVisionModel``."""
        vm = model.vision_model
        self.patch.load_state_dict(vm.embeddings.patch_embedding.state_dict())
        self.pos.copy_(vm.embeddings.position_embedding.weight)
        for i, layer in enumerate(vm.encoder.layers):
            at = layer.self_attn
            self.qkv[i].weight.copy_(torch.cat((at.q_proj.weight, at.k_proj.weight, at.v_proj.weight)))
            self.qkv[i].bias.copy_(torch.cat((at.q_proj.bias, at.k_proj.bias, at.v_proj.bias)))
            self.out[i].load_state_dict(at.out_proj.state_dict())
            self.ln1[i].load_state_dict(layer.layer_norm1.state_dict())
            self.ln2[i].load_state_dict(layer.layer_norm2.state_dict())
            self.fc1[i].load_state_dict(layer.mlp.fc1.state_dict())
            self.fc2[i].load_state_dict(layer.mlp.fc2.state_dict())
        self.post_ln.load_state_dict(vm.post_layernorm.state_dict())
        return self

    def forward(self, pixels: torch.Tensor) -> torch.Tensor:
        """[N, 3, H, W] -> [N, tokens, hidden] in the tower's dtype."""
        # the patch grid made token-major once: the convolution's [N, h, T]
        # viewed as [N, T, h] would keep every later residual add and Linear
        # input channel-major (non-vectorised adds, a copy before each GEMM)
        x = self.patch(pixels.to(self.patch.weight.dtype)).flatten(2).transpose(1, 2).contiguous() + self.pos
        n, t, h = x.shape
        d = h // self.heads
        for i in range(len(self.qkv)):
            qkv = self.qkv[i](layer_norm(self.ln1[i], x)).view(n, t, 3, self.heads, d)
            q, k, v = (qkv[:, :, j].transpose(1, 2) for j in range(3))
            a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(n, t, h)
            x = x + self.out[i](a)
            x = x + self.fc2[i](F.gelu(self.fc1[i](layer_norm(self.ln2[i], x)), approximate="tanh"))
        return layer_norm(self.post_ln, x)


class VisionPrefix(nn.Module):
    """SigLIP-So400m + PaliGemma's projector, and the prefix assembly of
    rocm_pi05_optim.py:88-133 (real cameras batched, the empty camera's
    cached embedding pooled 4:1, then the language embeddings)."""

    def __init__(self, cfg: SnapFlowConfig):
        super().__init__()
        self.cfg = cfg
        self.siglip = SiglipTower(cfg)
        self.projector = nn.Linear(cfg.vision_hidden, cfg.lm.hidden)
        self.register_buffer("empty_cam", torch.zeros(0), persistent=False)

    def embed_images(self, images: torch.Tensor) -> torch.Tensor:
        """[N, 3, H, W] -> [N, tokens, lm hidden] in the tower's dtype."""
        return self.projector(self.siglip(images))

    @torch.no_grad()
    def cache_empty_camera(self) -> None:
        """The empty camera is a constant -1 image: its pooled embedding is
        computed once (rocm_pi05_optim.py:72-87)."""
        cfg, dev = self.cfg, self.projector.weight.device
        blank = torch.full((1, 3, cfg.image_size, cfg.image_size), -1.0, device=dev)
        self.empty_cam = pool_tokens(self.embed_images(blank), cfg.empty_pool)

    def forward(self, images: torch.Tensor, lang_emb: torch.Tensor, lang_mask: torch.Tensor):
        """images [B, real_cameras, 3, H, W]; lang_emb [B, T, hidden] (already
        scaled); lang_mask bool [B, T] -> (embeds fp16 [B, L, hidden], pad bool
        [B, L])."""
        b, ncam = images.shape[:2]
        emb = self.embed_images(images.transpose(0, 1).reshape(ncam * b, *images.shape[2:]))
        emb = emb.view(ncam, b, emb.shape[1], emb.shape[2])
        parts = [emb[i] for i in range(ncam)] + [self.empty_cam.expand(b, -1, -1)]
        n_img = sum(p.shape[1] for p in parts)
        embeds = torch.cat([p.to(torch.float16) for p in parts] + [lang_emb.to(torch.float16)], dim=1)
        pad = torch.cat((torch.ones((b, n_img), dtype=torch.bool, device=lang_mask.device), lang_mask), dim=1)
        return embeds, pad


class SnapFlowPolicy:
    """The config-4 step on one GPU: ``sample_actions(images, lang_ids,
    lang_mask, noise)`` -> actions [B, chunk, action_dim] = x_t - v_t, x_t the
    noise in the expert's dtype and v_t the expert's velocity at t = target
    t = 1, in the noise's dtype (snapflow_pi05.py:170-195)."""

    def __init__(self, cfg: SnapFlowConfig, lm: plm.W4A4PrefixLM, device, seed: int = 0,
                 dtype=torch.bfloat16, std: float = 0.02):
        self.cfg, self.lm, self.device, self.dtype = cfg, lm, torch.device(device), dtype
        torch.manual_seed(seed)
        with torch.device(self.device):
            self.vision = VisionPrefix(cfg)
            self.expert = ActionExpert(cfg)
        for mod in (self.vision, self.expert):
            for name, p in mod.named_parameters():
                if p.dim() >= 2 and "embeddings" not in name:
                    nn.init.normal_(p, std=std)
            mod.to(dtype).eval()
        gen = torch.Generator(device=self.device).manual_seed(seed + 1)
        self.lang_table = torch.randn(cfg.vocab, cfg.lm.hidden, device=self.device, generator=gen,
                                      dtype=torch.float16)
        self.lang_scale = torch.tensor(math.sqrt(cfg.lm.hidden), dtype=torch.float16, device=self.device)
        self.vision.cache_empty_camera()
        self._prefix_out: dict = {}

    def _out(self, b: int, seq: int) -> plm.PrefixOutput:
        key = (b, seq)
        if key not in self._prefix_out:
            kv = self.lm.cfg.kv_heads * self.lm.cfg.head_dim
            f16 = dict(dtype=torch.float16, device=self.device)
            self._prefix_out[key] = plm.PrefixOutput(
                hidden=torch.empty((b, seq, self.lm.cfg.hidden), **f16),
                keys=[torch.empty((b, seq, kv), **f16) for _ in self.lm.layers],
                values=[torch.empty((b, seq, kv), **f16) for _ in self.lm.layers])
        return self._prefix_out[key]

    @torch.no_grad()
    def embed_prefix(self, images, lang_ids, lang_mask):
        lang = self.lang_table[lang_ids] * self.lang_scale
        return self.vision(images, lang, lang_mask)

    @torch.no_grad()
    def sample_actions(self, images, lang_ids, lang_mask, noise) -> torch.Tensor:
        embeds, pad = self.embed_prefix(images, lang_ids, lang_mask)
        out = self.lm.forward(embeds, pad, out=self._out(*pad.shape))
        b = noise.shape[0]
        t = torch.ones(b, dtype=torch.float32, device=self.device)
        x_t = noise.to(self.dtype)
        v = self.expert(x_t, t, t, pad, out.keys, out.values)
        return (x_t - v).to(noise.dtype)


class GraphedSnapFlow:
    """``SnapFlowPolicy.sample_actions`` at a fixed batch captured in one CUDA
    graph with static inputs: ``run(images, lang_ids, lang_mask, noise)``
    copies the inputs in and replays; the result is ``self.actions``."""

    def __init__(self, policy: SnapFlowPolicy, batch: int):
        cfg, dev = policy.cfg, policy.device
        self.policy = policy
        self.images = torch.zeros((batch, cfg.real_cameras, 3, cfg.image_size, cfg.image_size),
                                  dtype=torch.float32, device=dev)
        self.lang_ids = torch.zeros((batch, cfg.lang_tokens), dtype=torch.long, device=dev)
        self.lang_mask = torch.ones((batch, cfg.lang_tokens), dtype=torch.bool, device=dev)
        self.noise = torch.zeros((batch, cfg.chunk, cfg.action_dim), dtype=torch.float32, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                policy.sample_actions(self.images, self.lang_ids, self.lang_mask, self.noise)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.actions = policy.sample_actions(self.images, self.lang_ids, self.lang_mask, self.noise)

    def replay(self) -> None:
        self.graph.replay()

    def run(self, images, lang_ids, lang_mask, noise) -> torch.Tensor:
        self.images.copy_(images, non_blocking=True)
        self.lang_ids.copy_(lang_ids, non_blocking=True)
        self.lang_mask.copy_(lang_mask, non_blocking=True)
        self.noise.copy_(noise, non_blocking=True)
        self.graph.replay()
        return self.actions


def synthetic_observation(cfg: SnapFlowConfig, batch: int, real_lang: int = 52, seed: int = 0, device="cpu"):
    """Config 4's inputs: real-camera images with pixels ~ U[-1, 1], language
    ids (the first ``real_lang`` real, uniform over the vocabulary; the rest
    padding) and the flow noise ~ N(0, 1).  Returns (images fp32 [B, cams, 3,
    H, W], lang_ids [B, T], lang_mask bool [B, T], noise fp32 [B, chunk,
    action_dim])."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    images = torch.rand(batch, cfg.real_cameras, 3, cfg.image_size, cfg.image_size, generator=gen) * 2 - 1
    ids = torch.randint(0, cfg.vocab, (batch, cfg.lang_tokens), generator=gen)
    ids[:, real_lang:] = 0
    mask = torch.zeros(batch, cfg.lang_tokens, dtype=torch.bool)
    mask[:, :real_lang] = True
    noise = torch.randn(batch, cfg.chunk, cfg.action_dim, generator=gen)
    return images.to(device), ids.to(device), mask.to(device), noise.to(device)
