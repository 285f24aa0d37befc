"""Config 4 (the SnapFlow 1-NFE step around the W4A4 prefix LM): the expert's
masks, positions and prefix-KV attention against a direct restatement, the
time embedding, the empty-camera pool and the prefix assembly on CPU (tiny
shapes, fp32); the full-size step on a B200 (graph replay against eager,
the KV handoff from the W4A4 prefix LM)."""

from __future__ import annotations

import math
from dataclasses import replace

import pytest
import torch
import torch.nn.functional as F

from pi05_pytorch_fast_b200 import prefix_lm as plm
from pi05_pytorch_fast_b200 import snapflow as sf

TINY = sf.SnapFlowConfig(vision_hidden=32, vision_intermediate=64, vision_layers=2, vision_heads=4,
                         image_size=56, patch=14, lang_tokens=6, vocab=100,
                         lm=replace(plm.PrefixLMConfig(), hidden=48),
                         expert_hidden=40, expert_intermediate=96, expert_layers=2, expert_heads=4,
                         expert_kv_heads=1, head_dim=16, chunk=5, action_dim=3)


def test_time_embedding_matches_the_formula():
    t = torch.tensor([1.0, 0.25, 0.0])
    emb = sf.sinusoidal_time_embedding(t, 8, 4e-3, 4.0)
    for b, tb in enumerate(t.tolist()):
        for i in range(4):
            period = 4e-3 * (4.0 / 4e-3) ** (i / 3)
            assert emb[b, i].item() == pytest.approx(math.sin(2 * math.pi * tb / period), abs=1e-6)
            assert emb[b, 4 + i].item() == pytest.approx(math.cos(2 * math.pi * tb / period), abs=1e-6)


def test_roll_with_signed_sin_is_rotate_half():
    x = torch.randn(2, 3, 4, 16, dtype=torch.float64)
    sin = torch.randn(2, 3, 1, 16, dtype=torch.float64)
    torch.testing.assert_close(torch.roll(x, 8, dims=-1) * sf.signed_sin(sin), sf.rotate_half(x) * sin,
                               rtol=0, atol=0)


def test_pool_sums_runs_of_tokens():
    x = torch.arange(2 * 8 * 3, dtype=torch.float32).view(2, 8, 3)
    p = sf.pool_tokens(x, 4)
    assert p.shape == (2, 2, 3)
    assert torch.equal(p[1, 1], x[1, 4:8].sum(0))
    with pytest.raises(ValueError):
        sf.pool_tokens(x, 3)


def test_prefix_length_of_config_4_is_config_2s():
    assert sf.SnapFlowConfig().prefix_len == 776


def _expert_direct(expert: sf.ActionExpert, x_t, pad, keys, values):
    """The expert restated over the whole [prefix ; suffix] sequence: an
    additive fp64 mask (prefix key j visible iff real, every suffix key
    visible), explicit softmax, positions sum(pad) + i, GQA by repetition."""
    cfg = expert.cfg
    dev = x_t.device
    b, s = x_t.shape[0], cfg.chunk
    t = torch.ones(b, device=dev)
    cond = expert.condition(t, t).double()
    x = F.linear(x_t.double(), expert.action_in_proj.weight.double(), expert.action_in_proj.bias.double())
    pos = pad.sum(1, keepdim=True).double() + torch.arange(s, dtype=torch.float64, device=dev)[None]
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, dtype=torch.float32, device=dev)
                                    / cfg.head_dim))
    ang = (pos.float()[..., None] * inv).double()
    cos = torch.cat((ang, ang), -1).cos()[:, None]
    sin = torch.cat((ang, ang), -1).sin()[:, None]
    visible = torch.cat((pad, torch.ones(b, s, dtype=torch.bool, device=dev)), 1)
    add = torch.where(visible, 0.0, -math.inf)[:, None, None, :]

    mods = F.linear(cond, expert.modulation.weight.double(), expert.modulation.bias.double())
    mods = mods.view(b, expert.n_norms, 3, -1)

    def norm(i, x):
        scale, shift, gate = mods[:, i, 0, None], mods[:, i, 1, None], mods[:, i, 2, None]
        y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)
        return y * (1 + scale) + shift, gate

    def lin(m, x):
        return F.linear(x, m.weight.double(), None if m.bias is None else m.bias.double())

    for li, (layer, k, v) in enumerate(zip(expert.layers, keys, values)):
        n, g1 = norm(2 * li, x)
        q = lin(layer.q, n).view(b, s, cfg.expert_heads, -1).transpose(1, 2)
        kk = lin(layer.k, n).view(b, s, 1, -1).transpose(1, 2)
        vv = lin(layer.v, n).view(b, s, 1, -1).transpose(1, 2)
        q = q * cos + sf.rotate_half(q) * sin
        kk = kk * cos + sf.rotate_half(kk) * sin
        kk = torch.cat((k.double().view(b, -1, 1, cfg.head_dim).transpose(1, 2), kk), 2)
        vv = torch.cat((v.double().view(b, -1, 1, cfg.head_dim).transpose(1, 2), vv), 2)
        sc = q @ kk.transpose(-1, -2) / math.sqrt(cfg.head_dim) + add
        a = torch.softmax(sc, -1) @ vv
        x = x + g1 * lin(layer.o, a.transpose(1, 2).reshape(b, s, -1))
        n, g2 = norm(2 * li + 1, x)
        x = x + g2 * lin(layer.down, F.gelu(lin(layer.gate, n), approximate="tanh") * lin(layer.up, n))
    x, _ = norm(-1, x)
    return lin(expert.action_out_proj, x)


def test_expert_over_the_prefix_cache_matches_the_direct_restatement():
    torch.manual_seed(0)
    expert = sf.ActionExpert(TINY).eval()
    b, L = 2, 9
    pad = torch.ones(b, L, dtype=torch.bool)
    pad[0, 6:] = False
    pad[1, 3:] = False
    keys = [torch.randn(b, L, TINY.head_dim) for _ in range(TINY.expert_layers)]
    values = [torch.randn(b, L, TINY.head_dim) for _ in range(TINY.expert_layers)]
    x_t = torch.randn(b, TINY.chunk, TINY.action_dim)
    t = torch.ones(b)
    with torch.no_grad():
        v = expert(x_t, t, t, pad, keys, values)
        ref = _expert_direct(expert, x_t, pad, keys, values)
    torch.testing.assert_close(v.double(), ref, rtol=1e-4, atol=1e-5)
    # a padded prefix key never matters
    keys2 = [k.clone() for k in keys]
    keys2[0][0, 7] += 100.0
    values2 = [x.clone() for x in values]
    values2[1][1, 5] -= 50.0
    with torch.no_grad():
        torch.testing.assert_close(expert(x_t, t, t, pad, keys2, values2), v)


def test_siglip_tower_matches_transformers_siglip():
    from transformers import SiglipVisionConfig, SiglipVisionModel

    torch.manual_seed(2)
    hf = SiglipVisionModel(SiglipVisionConfig(
        hidden_size=TINY.vision_hidden, intermediate_size=TINY.vision_intermediate,
        num_hidden_layers=TINY.vision_layers, num_attention_heads=TINY.vision_heads,
        image_size=TINY.image_size, patch_size=TINY.patch, vision_use_head=False)).eval()
    with torch.no_grad():
        for p in hf.parameters():  # non-trivial norms and biases
            p.add_(torch.randn_like(p) * 0.05)
    tower = sf.SiglipTower(TINY).eval().load_transformers(hf)
    px = torch.rand(3, 3, TINY.image_size, TINY.image_size) * 2 - 1
    with torch.no_grad():
        torch.testing.assert_close(tower(px), hf(pixel_values=px).last_hidden_state, rtol=1e-5, atol=1e-5)


def test_vision_prefix_assembles_cameras_empty_camera_and_language():
    torch.manual_seed(1)
    vis = sf.VisionPrefix(TINY).eval()
    vis.cache_empty_camera()
    tok = TINY.image_tokens
    assert vis.empty_cam.shape == (1, tok // TINY.empty_pool, TINY.lm.hidden)
    b = 2
    images, ids, mask, _ = sf.synthetic_observation(TINY, b, real_lang=4, seed=3)
    lang = torch.randn(b, TINY.lang_tokens, TINY.lm.hidden)
    with torch.no_grad():
        embeds, pad = vis(images, lang, mask)
        cam1 = vis.embed_images(images[:, 1])
        blank = vis.embed_images(torch.full((1, 3, TINY.image_size, TINY.image_size), -1.0))
    assert embeds.shape == (b, TINY.prefix_len, TINY.lm.hidden) and embeds.dtype == torch.float16
    assert torch.equal(embeds[:, tok:2 * tok], cam1.half())
    torch.testing.assert_close(embeds[0, 2 * tok:2 * tok + tok // 4].float(),
                               sf.pool_tokens(blank, 4)[0].half().float())
    assert torch.equal(embeds[:, -TINY.lang_tokens:], lang.half())
    assert pad[:, :2 * tok + tok // 4].all()
    assert torch.equal(pad[:, -TINY.lang_tokens:], mask)


def test_neighbour_kernels_check_their_arguments():
    """Shape and alignment checks run on the host, before any device work."""
    from pi05_pytorch_fast_b200 import _native as nat

    lib = nat.lib()
    fake = 1 << 40

    def err(rc):
        assert rc != nat.W4A4_OK
        return nat.last_error()

    assert "multiple of 256" in err(lib.w4a4_ada_rms_norm_bf16(fake, fake, 4, 1000, 2, fake, fake, 1000, 1e-6, None))
    assert "mod_stride" in err(lib.w4a4_ada_rms_norm_bf16(fake, fake, 4, 1024, 2, fake, fake, 512, 1e-6, None))
    assert "aligned" in err(lib.w4a4_ada_rms_norm_bf16(fake + 2, fake, 4, 1024, 2, fake, fake, 1024, 1e-6, None))
    assert lib.w4a4_ada_rms_norm_bf16(None, None, 0, 1024, 1, None, None, 1024, 1e-6, None) == nat.W4A4_OK
    assert "multiple of 16" in err(lib.w4a4_rope_qk_bf16(fake, 2040, 8, fake, 255, 1, fake, fake, 4, 255, None))
    assert "strides" in err(lib.w4a4_rope_qk_bf16(fake, 1024, 8, fake, 256, 1, fake, fake, 4, 256, None))
    assert "aligned" in err(lib.w4a4_rope_qk_bf16(fake, 2052, 8, fake, 256, 1, fake, fake, 4, 256, None))
    assert "multiple of 8" in err(lib.w4a4_layer_norm_bf16(fake, fake, 4, 1150, fake, fake, 1e-6, None))
    assert "null" in err(lib.w4a4_layer_norm_bf16(fake, None, 4, 1152, fake, fake, 1e-6, None))


# ----------------------------------------------------------------------------- B200
def _bf16_close(got: torch.Tensor, ref: torch.Tensor):
    """Within one bf16 rounding of an fp64 reference (plus fp32 reduction
    order): |got - ref| <= 2^-7 |ref| + 1e-6."""
    got, ref = got.double(), ref.double()
    bad = (got - ref).abs() > ref.abs() * 2.0 ** -7 + 1e-6
    assert not bad.any(), f"{int(bad.sum())} of {bad.numel()} values off"


@pytest.mark.gpu
def test_ada_rms_norm_kernel_matches_the_formula():
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(11)
    b, s, h, n = 3, 50, 1024, 5
    x = (torch.randn(b, s, h, device=dev, generator=g) * 3).bfloat16()
    scale1 = (1 + torch.randn(b, n, h, device=dev, generator=g) * 0.3).contiguous()
    shift = (torch.randn(b, n, h, device=dev, generator=g) * 0.5).contiguous()
    gate = torch.randn(b, n, h, device=dev, generator=g).bfloat16()
    y, gt = sf.ada_rms_norm(x, (scale1[:, 2], shift[:, 2], gate[:, 2]), 1e-6)
    xd = x.double()
    ref = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-6) * scale1[:, 2, None].double() \
        + shift[:, 2, None].double()
    assert y.dtype == torch.bfloat16 and torch.equal(gt, gate[:, 2, None])
    _bf16_close(y, ref)


@pytest.mark.gpu
def test_rope_kernel_matches_rotate_half():
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(12)
    rows, hq, hk, hd = 100, 8, 1, 256
    q = torch.randn(rows, hq * hd, device=dev, generator=g).bfloat16()
    k = torch.randn(rows, hk * hd, device=dev, generator=g).bfloat16()
    pos = torch.arange(rows, device=dev)[None] + 700
    cos, sin = sf.rope_tables(pos, hd, 10000.0, torch.bfloat16)
    cos, sin = cos[0, 0].contiguous(), sin[0, 0].contiguous()
    q0, k0 = q.clone(), k.clone()
    from pi05_pytorch_fast_b200 import _native as nat

    nat.check(nat.lib().w4a4_rope_qk_bf16(q.data_ptr(), hq * hd, hq, k.data_ptr(), hk * hd, hk, cos.data_ptr(),
                                          sin.data_ptr(), rows, hd, torch.cuda.current_stream().cuda_stream))
    for got, x0, heads in ((q, q0, hq), (k, k0, hk)):
        xd = x0.double().view(rows, heads, hd)
        ref = xd * cos.double()[:, None] + sf.rotate_half(xd) * sin.double()[:, None]
        _bf16_close(got.view(rows, heads, hd), ref)


@pytest.mark.gpu
def test_layer_norm_kernel_matches_torch():
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(13)
    ln = torch.nn.LayerNorm(1152, eps=1e-6).to(dev)
    with torch.no_grad():
        ln.weight.normal_(1.0, 0.2, generator=g)
        ln.bias.normal_(0.0, 0.2, generator=g)
    ln = ln.bfloat16()
    x = (torch.randn(2, 300, 1152, device=dev, generator=g) * 2 + 0.5).bfloat16()
    with torch.no_grad():
        y = sf.layer_norm(ln, x)
        ref = F.layer_norm(x.double(), (1152,), ln.weight.double(), ln.bias.double(), 1e-6)
    _bf16_close(y, ref)



@pytest.fixture(scope="module")
def policy():
    dev = torch.device("cuda:0")
    lm = plm.W4A4PrefixLM.random(plm.PrefixLMConfig(), dev, seed=5)
    return sf.SnapFlowPolicy(sf.SnapFlowConfig(), lm, dev, seed=6)


@pytest.mark.gpu
def test_snapflow_step_graph_replay_equals_eager(policy):
    cfg = policy.cfg
    obs = sf.synthetic_observation(cfg, 2, seed=7, device="cuda:0")
    eager = policy.sample_actions(*obs)
    g = sf.GraphedSnapFlow(policy, 2)
    out = g.run(*obs)
    torch.cuda.synchronize()
    assert out.shape == (2, cfg.chunk, cfg.action_dim) and out.dtype == torch.float32
    assert torch.isfinite(out).all()
    assert torch.equal(out, eager)
    # a second observation batch through the same graph
    obs2 = sf.synthetic_observation(cfg, 2, seed=8, device="cuda:0")
    out2 = g.run(*obs2).clone()
    torch.testing.assert_close(out2, policy.sample_actions(*obs2), rtol=0, atol=0)
    assert not torch.equal(out2, eager)


@pytest.mark.gpu
def test_snapflow_expert_reads_the_w4a4_prefix_cache(policy):
    """The expert's velocity from the W4A4 prefix LM's KV cache, against the
    fp64 restatement over the same cache (bf16 expert: loose tolerance), and
    the observations of a batch stay independent (the two have different
    language lengths, so different prefix masks and suffix positions)."""
    cfg = policy.cfg
    images, ids, mask, noise = sf.synthetic_observation(cfg, 2, seed=9, device="cuda:0")
    mask[1, 17:] = False
    ids[1, 17:] = 0
    with torch.no_grad():
        embeds, pad = policy.embed_prefix(images, ids, mask)
        out = policy.lm.forward(embeds, pad)
        x_t = noise.to(policy.dtype)
        t = torch.ones(2, device="cuda:0")
        v = policy.expert(x_t, t, t, pad, out.keys, out.values).double()
        expert64 = sf.ActionExpert(cfg).to("cuda:0")
        expert64.load_state_dict(policy.expert.state_dict())
        ref = _expert_direct(expert64.double(), x_t.double(), pad, out.keys, out.values)
        one = policy.sample_actions(images[1:], ids[1:], mask[1:], noise[1:])
        both = policy.sample_actions(images, ids, mask, noise)
    rel = (v - ref).norm() / ref.norm()
    assert rel < 0.05, float(rel)
    # bf16 library GEMMs may pick other kernels for another batch size
    rel_b = (both[1:] - one).norm() / one.norm()
    assert rel_b < 0.02, float(rel_b)
