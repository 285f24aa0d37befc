"""CPU-only tests: the C-ABI library loads and exports every declared symbol,
host-side argument validation (no CUDA call is reached), the packed-format
helpers against the reference's golden vectors, and the op layer's
refusal of CPU tensors (there is no CPU fallback)."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from pi05_pytorch_fast_b200 import _native as nat
from pi05_pytorch_fast_b200.w4a4 import pack as bpack

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions() -> list[str]:
    text = open(os.path.join(ROOT, "include", "w4a4_sm100.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*int\s+(w4a4_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_binding_symbols():
    assert declared_functions() == sorted(nat.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(nat.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert nat.lib().w4a4_version() == 100


def _err(status):
    assert status != nat.W4A4_OK
    return nat.last_error()


def test_quant_argument_validation_without_gpu():
    lib = nat.lib()
    assert "multiple of 64, got 100" in _err(lib.w4a4_quant(None, 4, 100, 100, -1, 0, 0, None, None, None))
    assert "positive" in _err(lib.w4a4_quant(None, 4, 0, 0, -1, 0, 0, None, None, None))
    assert "staging" in _err(lib.w4a4_quant(None, 4, 64, 64, -1, 7, 0, None, None, None))
    assert "rotation" in _err(lib.w4a4_quant(None, 4, 4096, 4096, 1, 0, 0, None, None, None))
    # M == 0 is a no-op that succeeds before any device call
    assert lib.w4a4_quant(None, 0, 2048, 2048, -1, 0, 0, None, None, None) == nat.W4A4_OK


def test_gemm_argument_validation_without_gpu():
    lib = nat.lib()
    k = 2048
    fake = 0x1000  # never dereferenced: validation fails first
    w = nat.weights_array([(fake, 16384, k // 8 + 1, nat.LAYOUT_FRAGMENT_MAJOR)])
    y = nat.pointer_array([fake])
    assert "K/8+9 marker stride" in _err(lib.w4a4_gemm(fake, fake, 4, k, 1, w, y, None))
    w = nat.weights_array([(fake, 64, k // 8 + 1, nat.LAYOUT_ROW_MAJOR)])
    assert "multiple of 4 words" in _err(lib.w4a4_gemm(fake, fake, 4, k, 1, w, y, None))
    w = nat.weights_array([(fake, 64, k // 8, nat.LAYOUT_ROW_MAJOR)])
    assert "K/8 packed words plus a scale" in _err(lib.w4a4_gemm(fake, fake, 4, k, 1, w, y, None))
    w = nat.weights_array([(fake, 64, 264, 0), (fake, 64, 265, 1)])
    assert "share a layout" in _err(lib.w4a4_gemm(fake, fake, 4, k, 2, w, nat.pointer_array([fake, fake]), None))
    assert "n_weights" in _err(lib.w4a4_gemm(fake, fake, 4, k, 4, w, y, None))
    w = nat.weights_array([(fake + 4, 64, 264, nat.LAYOUT_ROW_MAJOR)])
    assert "16-byte aligned" in _err(lib.w4a4_gemm(fake, fake, 4, k, 1, w, y, None))


def test_gemm_variant_selection_validated():
    lib = nat.lib()
    assert "unknown GEMM variant 7" in _err(lib.w4a4_set_gemm_variant(7))
    for v in (nat.GEMM_NO_SPLIT, nat.GEMM_SPLIT_K):
        assert lib.w4a4_set_gemm_variant(v) == nat.W4A4_OK
    assert lib.w4a4_set_gemm_variant(nat.GEMM_CTA_PAIR) == nat.W4A4_OK
    assert lib.w4a4_set_gemm_variant(nat.GEMM_SINGLE_CTA) == nat.W4A4_OK


# The launch plans of the prefix's GEMMs at M = 776 on 148 SMs (as the ncu
# launch list shows them): q/k/v, o, gate/up, down.
# gate/up (fragment-major, 776 tokens) runs on the CTA pair: 128 weight tiles
# of 256 rows.
PREFIX_PLANS = [
    ("qkv", 776, 2048, [2048, 256, 256], nat.LAYOUT_ROW_MAJOR,
     dict(tok_tile=112, split=False, grid=140, tok_group=7, w_tiles=20)),
    ("o", 776, 2048, [2048], nat.LAYOUT_ROW_MAJOR,
     dict(tok_tile=96, split=False, grid=144, tok_group=9, w_tiles=16)),
    ("gate/up", 776, 2048, [16384, 16384], nat.LAYOUT_FRAGMENT_MAJOR,
     dict(tok_tile=208, split=False, grid=148, tok_group=4, w_tiles=128)),
    ("down", 776, 16384, [2048], nat.LAYOUT_ROW_MAJOR,
     dict(tok_tile=208, split=True, grid=128, tok_group=4, w_tiles=16)),
]


@pytest.mark.parametrize("name,m,k,ns,layout,want", PREFIX_PLANS)
def test_prefix_gemm_plans(name, m, k, ns, layout, want):
    plan = nat.gemm_plan(m, k, ns, layout=layout)
    assert {key: plan[key] for key in want} == want, (name, plan)


def test_default_variant_pairs_only_large_fragment_major_gemms():
    """The default variant runs fragment-major GEMMs of 768 or more tokens on
    the CTA pair (256-row weight tiles, no split-K) and everything else on
    single CTAs."""
    ns = [16384, 16384]
    assert nat.gemm_plan(767, 2048, ns, layout=nat.LAYOUT_FRAGMENT_MAJOR)["w_tiles"] == 256
    big = nat.gemm_plan(768, 2048, ns, layout=nat.LAYOUT_FRAGMENT_MAJOR)
    assert big["w_tiles"] == 128 and not big["split"] and big["grid"] % 2 == 0
    assert nat.gemm_plan(6208, 2048, ns, layout=nat.LAYOUT_ROW_MAJOR)["w_tiles"] == 256
    for v in (nat.GEMM_NO_SPLIT, nat.GEMM_SPLIT_K):
        assert nat.gemm_plan(6208, 2048, ns, variant=v,
                             layout=nat.LAYOUT_FRAGMENT_MAJOR)["w_tiles"] == 256


@pytest.mark.parametrize("m", [1, 15, 16, 17, 208, 209, 640, 768, 776, 6208, 24832])
@pytest.mark.parametrize("k,ns", [(2048, [2048, 256, 256]), (2048, [16384, 16384]),
                                  (16384, [2048]), (1024, [384, 128]), (64, [24])])
@pytest.mark.parametrize("variant", [nat.GEMM_SINGLE_CTA, nat.GEMM_CTA_PAIR, nat.GEMM_NO_SPLIT,
                                     nat.GEMM_SPLIT_K])
@pytest.mark.parametrize("layout", [nat.LAYOUT_ROW_MAJOR, nat.LAYOUT_FRAGMENT_MAJOR])
def test_gemm_plan_invariants(m, k, ns, variant, layout):
    """Whatever the shape, the plan covers every token with at most 208-token
    MMA tiles, launches no more CTAs than SMs (pairs and split-K clusters: an
    even grid, one tile per cluster for split-K), splits K only into two even
    halves, and groups token tiles so one group's codes stay within ~48 MB."""
    sms = 148
    plan = nat.gemm_plan(m, k, ns, sms=sms, variant=variant, layout=layout)
    pair = variant == nat.GEMM_CTA_PAIR or (
        variant == nat.GEMM_SINGLE_CTA and layout == nat.LAYOUT_FRAGMENT_MAJOR and m >= 768)
    rows = 256 if pair else 128
    assert plan["w_tiles"] == sum(-(-n // rows) for n in ns)
    t = plan["tok_tile"]
    assert t % 16 == 0 and 16 <= t <= 208
    assert plan["tok_tiles"] == -(-m // t)
    total = plan["tok_tiles"] * plan["w_tiles"]
    assert 1 <= plan["grid"] <= sms
    k_steps = -(-k // 128)
    if plan["split"]:
        assert variant != nat.GEMM_NO_SPLIT and not pair
        assert k_steps % 2 == 0 and plan["grid"] == 2 * total <= sms
    elif variant == nat.GEMM_SPLIT_K:
        assert k_steps % 2 == 1 or k_steps < 2 or total > sms // 2  # could not split
    if pair:
        assert plan["grid"] % 2 == 0
    g = plan["tok_group"]
    assert 1 <= g <= plan["tok_tiles"]
    assert g == plan["tok_tiles"] or g * t * k <= 48 << 20


def test_gemm_plan_rejects_bad_queries():
    for args in ((0, 2048, [64]), (4, 100, [64]), (4, 2048, [0]), (4, 2048, [64, 64, 64, 64])):
        with pytest.raises(nat.W4A4Error):
            nat.gemm_plan(*args)
    with pytest.raises(nat.W4A4Error, match="unknown GEMM variant"):
        nat.gemm_plan(4, 2048, [64], variant=9)
    with pytest.raises(nat.W4A4Error, match="unknown weight layout"):
        nat.gemm_plan(4, 2048, [64], layout=7)


def test_ops_refuse_cpu_tensors():
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    x = torch.randn(3, 2048).half()
    w = torch.zeros(16, 264, dtype=torch.int32)
    for op in (lambda: ext.int4_gemm(x, w), lambda: ext.int4_gemm3(x, w, w, w),
               lambda: ext.int4_gemm2(x, w, w)):
        with pytest.raises(RuntimeError, match="expects CUDA/HIP tensors"):
            op()


def test_repack_int8_argument_validation_without_gpu():
    lib = nat.lib()
    dst = ctypes.c_void_p(16)
    row = nat.weights_array([(16, 8, 2048 // 8 + 8, nat.LAYOUT_ROW_MAJOR)])
    frag = nat.weights_array([(16, 8, 2048 // 8 + 9, nat.LAYOUT_FRAGMENT_MAJOR)])
    already = nat.weights_array([(16, 8, 2048 // 4 + 4, nat.LAYOUT_INT8)])
    assert lib.w4a4_repack_int8(row, 2000, dst, None) != 0          # K not a multiple of 64
    assert lib.w4a4_repack_int8(row, 131072, dst, None) != 0        # above the magic-number K
    assert lib.w4a4_repack_int8(already, 2048, dst, None) != 0      # already int8
    assert lib.w4a4_repack_int8(row, 2048, ctypes.c_void_p(8), None) != 0  # unaligned dst
    assert lib.w4a4_repack_int8(None, 2048, dst, None) != 0
    bad_frag = nat.weights_array([(16, 8, 2048 // 8 + 8, nat.LAYOUT_FRAGMENT_MAJOR)])
    assert lib.w4a4_repack_int8(bad_frag, 2048, dst, None) != 0     # fragment-major needs K/8+9
    del frag


def test_pack_weight_argument_validation_without_gpu():
    lib = nat.lib()
    out = ctypes.c_void_p(16)
    w = ctypes.c_void_p(16)
    bad = [
        (w, 0, 64, 4, 60, -1, nat.LAYOUT_ROW_MAJOR, out, 9),        # K not a multiple of 64
        (w, 0, 32768, 4, 32768, -1, nat.LAYOUT_ROW_MAJOR, out, 4097),  # K above 16384
        (w, 3, 64, 4, 64, -1, nat.LAYOUT_ROW_MAJOR, out, 9),        # dtype
        (w, 0, 64, 4, 64, 2, nat.LAYOUT_ROW_MAJOR, out, 9),         # rotate
        (w, 0, 192, 4, 192, 1, nat.LAYOUT_ROW_MAJOR, out, 25),      # rotation of a non-power-of-two K
        (w, 0, 32, 4, 64, -1, nat.LAYOUT_ROW_MAJOR, out, 9),        # row stride below K
        (w, 0, 64, 4, 64, -1, nat.LAYOUT_ROW_MAJOR, out, 8),        # rows without the scale word
        (w, 0, 64, 4, 64, -1, nat.LAYOUT_FRAGMENT_MAJOR, out, 16),  # not the K/8+9 stride
        (w, 0, 64, 3, 64, -1, nat.LAYOUT_FRAGMENT_MAJOR, out, 17),  # odd N
        (w, 0, 64, 4, 64, -1, 7, out, 9),                           # layout
    ]
    for args in bad:
        assert lib.w4a4_pack_weight(*args, None) != 0, args


def test_gemm_from_codes_checks_codes_and_scales():
    """Codes must be contiguous int8 [M, K] and scales fp32 [M]: a sliced or
    mistyped view is refused before anything reaches the library."""
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    codes = torch.zeros(4, 128, dtype=torch.int8)
    scales = torch.ones(4)
    w = [torch.zeros(16, 25, dtype=torch.int32)]
    bad = [
        (codes.float(), scales),
        (torch.zeros(4, 256, dtype=torch.int8)[:, :128], scales),
        (codes[0], scales),
        (codes, scales.half()),
        (codes, torch.ones(3)),
        (codes, torch.ones(8)[::2]),
    ]
    for c, sc in bad:
        with pytest.raises(ValueError, match="gemm_from_codes"):
            ext.gemm_from_codes(c, sc, w)


def test_extension_module_serves_as_the_reference_compiled_module():
    """The integration binding assigns this module to the reference's `_mod`
    (the object load_int4_gemm() returns): it must expose the compiled
    module's five functions, and the ops must already be registered so the
    reference's registration returns early."""
    import inspect

    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    for name, n_weights in (("int4_gemm", 1), ("int4_gemm_tiled", 1), ("int4_gemm2", 2),
                            ("int4_gemm2_tiled", 2), ("int4_gemm3", 3)):
        fn = getattr(ext, name)
        assert callable(fn)
        assert len(inspect.signature(fn).parameters) == 1 + n_weights
        assert hasattr(torch.ops.pi05_w4a4, name)
    assert callable(ext.preload)


def test_op_bodies_come_from_the_cpp_op_library():
    """The five ops run the C++ bodies of _w4a4_ops.so (csrc/torch_ops.cpp),
    not a Python body and not the not-built stub."""
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    assert ext._load_ops()
    for name, _, _ in ext._OPS:
        table = torch._C._dispatch_dump(f"pi05_w4a4::{name}")
        line = next(ln for ln in table.splitlines() if ln.startswith("CompositeExplicitAutograd"))
        assert "torch_ops.cpp" in line, table


def test_ops_raise_when_the_op_library_is_not_built(tmp_path):
    """A package copy without _w4a4_ops.so registers raising stubs (no CPU
    fallback); building and loading the library afterwards in the same
    process replaces them without a duplicate-kernel registration."""
    import shutil
    import subprocess
    import sys

    pkg = os.path.join(ROOT, "pi05_pytorch_fast_b200")
    shutil.copytree(pkg, tmp_path / "pi05_pytorch_fast_b200",
                    ignore=shutil.ignore_patterns("_w4a4_ops.so", "__pycache__", "csrc"))
    script = (
        "import os, shutil, torch\n"
        "from pi05_pytorch_fast_b200.w4a4 import extension as ext\n"
        "try:\n"
        "    torch.ops.pi05_w4a4.int4_gemm(torch.zeros(1, 8, dtype=torch.float16),"
        " torch.zeros(1, 2, dtype=torch.int32))\n"
        "    raise SystemExit('stub did not raise')\n"
        "except RuntimeError as e:\n"
        "    assert 'is not built' in str(e), e\n"
        f"shutil.copy({os.path.join(pkg, '_w4a4_ops.so')!r}, ext.OPS_LIB_PATH)\n"
        "ext.preload()\n"
        "table = torch._C._dispatch_dump('pi05_w4a4::int4_gemm')\n"
        "line = next(l for l in table.splitlines() if l.startswith('CompositeExplicitAutograd'))\n"
        "assert 'torch_ops.cpp' in line, table\n"
        "print('ok')\n")
    env = dict(os.environ, PYTHONPATH=str(tmp_path))
    r = subprocess.run([sys.executable, "-c", script], cwd=tmp_path, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
    assert "Overriding a previously registered kernel" not in r.stderr, r.stderr


def test_op_library_uses_the_shared_cxx_runtime():
    """_w4a4_ops.so must take libstdc++ from libstdc++.so.6, like torch: a
    second, statically linked C++ runtime in it makes every exception torch
    throws through an op body (a TORCH_CHECK with a formatted message) crash
    the process while unwinding."""
    import shutil
    import subprocess

    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    if shutil.which("readelf") is None:
        pytest.skip("readelf not installed")
    dyn = subprocess.run(["readelf", "-d", ext.OPS_LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    assert "[libstdc++.so.6]" in dyn


def test_fake_impls_give_reference_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(2, 776, 2048, dtype=torch.float16, device="cuda")
        w = torch.empty(2048, 264, dtype=torch.int32, device="cuda")
        y = torch.ops.pi05_w4a4.int4_gemm(x, w)
        q, k, v = torch.ops.pi05_w4a4.int4_gemm3(x, w, w[:256], w[:256])
    assert y.shape == (2, 776, 2048) and y.dtype == torch.float16
    assert k.shape == (2, 776, 256)


@pytest.mark.parametrize("name", ["w2048", "w1024", "w16384", "w128", "wzero"])
def test_product_packer_matches_reference(golden, name):
    packed = bpack.pack_linear_weight(torch.from_numpy(golden[f"{name}_w"]))
    np.testing.assert_array_equal(packed.numpy(), golden[f"{name}_packed"])


@pytest.mark.parametrize("name,k", [("pre64", 64), ("pre2048", 2048)])
def test_product_preshuffle_matches_reference(golden, name, k):
    tiled = bpack.preshuffle_wmma_weight(torch.from_numpy(golden[f"{name}_packed"]), k)
    np.testing.assert_array_equal(tiled.numpy(), golden[f"{name}_tiled"])


REFERENCE = os.environ.get("PI05_REFERENCE_CHECKOUT", "/root/reference")

# Runs in a fresh interpreter: applies the two-line binding a maintainer adds
# (mark the reference's op registration done, point its module handle at this
# package) to the UNMODIFIED reference extension module, then installs W4A4
# on a small transformers Gemma with the reference's own apply.py / linear.py
# and traces one forward under FakeTensorMode (CUDA fake tensors; no GPU).
_BINDING_SCRIPT = r"""
import sys, torch
import pi05_pytorch_fast_b200
from pi05_pytorch_fast_b200.w4a4 import extension as ours
sys.path.insert(0, sys.argv[1])
import pi05_fast.w4a4.extension as ref_ext
assert ref_ext.__file__.startswith(sys.argv[1]), ref_ext.__file__
ref_ext._mod = ours                         # the binding a maintainer adds
ref_ext._register_custom_op()
assert ref_ext._op_registered, "the reference did not take its early-out"
assert ref_ext.load_int4_gemm() is ours
ref_ext.preload()                           # no HIP JIT: returns the bound module
from pi05_fast.w4a4 import apply as ref_apply
from pi05_fast.w4a4.linear import W4A4Linear as RefLinear
from transformers import GemmaConfig
from transformers.models.gemma.modeling_gemma import GemmaModel
cfg = GemmaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                  num_attention_heads=2, num_key_value_heads=1, head_dim=64, vocab_size=64)
cfg._attn_implementation = "eager"
model = GemmaModel(cfg).half()
tensors, layers = ref_apply.pack_model_linears(model, name_prefixes=("layers.",))
assert ref_apply.replace_linears_from_packed(model, tensors, layers) == 14
assert ref_apply.fuse_shared_activation_quant(model) == 4
assert isinstance(model.layers[0].mlp.down_proj, RefLinear)
from collections import Counter
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.utils._python_dispatch import TorchDispatchMode

class OpLog(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.calls = Counter()
    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        name = str(func.overloadpacket)
        if name.startswith("pi05_w4a4."):
            self.calls[name] += 1
        return func(*args, **(kwargs or {}))

with FakeTensorMode(allow_non_fake_inputs=True), OpLog() as log:
    model = model.to("cuda")
    x = torch.empty(1, 8, 128, dtype=torch.float16, device="cuda")
    pos = torch.arange(8, device="cuda")[None]
    out = model(inputs_embeds=x, position_ids=pos).last_hidden_state
assert tuple(out.shape) == (1, 8, 128) and out.dtype == torch.float16, (out.shape, out.dtype)
# per layer: int4_gemm3 (q/k/v), int4_gemm (o_proj, down_proj), int4_gemm2 (gate/up)
assert log.calls == {"pi05_w4a4.int4_gemm3": 2, "pi05_w4a4.int4_gemm": 4, "pi05_w4a4.int4_gemm2": 2}, log.calls
print("binding ok", dict(log.calls))
"""


@pytest.mark.skipif(not os.path.isdir(os.path.join(REFERENCE, "pi05_fast", "w4a4")),
                    reason="reference checkout not present (only in the build container)")
def test_unmodified_reference_caller_runs_on_these_ops():
    import subprocess
    import sys

    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    res = subprocess.run([sys.executable, "-c", _BINDING_SCRIPT, REFERENCE], capture_output=True,
                         text=True, env=env, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "binding ok" in res.stdout


def test_layer_glue_argument_validation_without_gpu():
    lib = nat.lib()
    fake = 0x1000  # never dereferenced: validation fails first
    assert "K = 2048" in _err(lib.w4a4_rmsnorm_quant(fake, 1024, None, 0, fake, 1e-6, None, 0, None, 0,
                                                     4, 1024, 0, 2, fake, fake, None))
    assert "codes or h_out" in _err(lib.w4a4_rmsnorm_quant(fake, 2048, None, 0, fake, 1e-6, None, 0, None,
                                                           0, 4, 2048, 0, 2, None, None, None))
    assert "16-byte aligned" in _err(lib.w4a4_rmsnorm_quant(fake + 2, 2048, None, 0, fake, 1e-6, None, 0,
                                                            None, 0, 4, 2048, 0, 2, fake, fake, None))
    assert "staging" in _err(lib.w4a4_rmsnorm_quant(fake, 2048, None, 0, fake, 1e-6, None, 0, None, 0,
                                                    4, 2048, 9, 2, fake, fake, None))
    assert "K = 16384" in _err(lib.w4a4_geglu_quant(fake, fake, 4, 2048, 2048, 0, 2, fake, fake, None, 0,
                                                    None))
    assert "16-byte aligned" in _err(lib.w4a4_geglu_quant(fake + 2, fake, 4, 16384, 16384, 0, 2, fake, fake,
                                                          None, 0, None))
    assert "codes format" in _err(lib.w4a4_geglu_quant(fake, fake, 4, 16384, 16384, 0, 7, fake, fake,
                                                       None, 0, None))
    assert "rope rows" in _err(lib.w4a4_rope(fake, 100, fake, 256, fake, fake, 4, 1, None))
    assert "invalid rope shape" in _err(lib.w4a4_rope(fake, 256, fake, 256, fake, fake, 4, 0, None))
    # empty inputs succeed before any device call
    assert lib.w4a4_rmsnorm_quant(None, 2048, None, 0, None, 1e-6, None, 0, fake, 2048, 0, 2048, 0, 2,
                                  None, None, None) == nat.W4A4_OK
    assert lib.w4a4_geglu_quant(None, None, 0, 16384, 16384, 0, 2, None, None, None, 0, None) == nat.W4A4_OK
    assert lib.w4a4_rope(None, 256, None, 256, None, None, 0, 8, None) == nat.W4A4_OK


def test_prefix_positions_and_mask_follow_lerobot():
    from pi05_pytorch_fast_b200 import prefix_lm as plm

    pad = torch.tensor([[1, 1, 0, 1, 0], [1, 1, 1, 1, 1]], dtype=torch.bool)
    pos, mask = plm.prefix_positions_and_mask(pad)
    assert pos.tolist() == [[0, 1, 1, 2, 2], [0, 1, 2, 3, 4]]
    allowed = mask[:, 0] == 0
    expect = pad[:, :, None] & pad[:, None, :]  # make_att_2d_masks with an all-zero att mask
    assert torch.equal(allowed, expect)
    assert float(mask.min()) == float(torch.tensor(plm.MASK_VALUE, dtype=torch.float32))


def test_rope_tables_match_transformers_rotary_embedding():
    """cos / sin as the model computes them equal transformers' Gemma rotary
    embedding bit for bit (CPU, config 2's head_dim and theta)."""
    from transformers import GemmaConfig
    from transformers.models.gemma.modeling_gemma import GemmaRotaryEmbedding

    from pi05_pytorch_fast_b200 import prefix_lm as plm

    cfg = plm.PrefixLMConfig()
    hf = GemmaRotaryEmbedding(GemmaConfig(hidden_size=2048, num_attention_heads=8, num_key_value_heads=1,
                                          head_dim=256))
    assert torch.equal(hf.inv_freq, plm.rope_inv_freq(cfg, fp16_buffer=False))
    pad = torch.ones(1, 776, dtype=torch.bool)
    pad[0, 628:] = False
    pos, _ = plm.prefix_positions_and_mask(pad)
    x = torch.empty(1, 776, 2048, dtype=torch.float16)
    for fp16_buffer in (False, True):
        if fp16_buffer:  # the reference's fp16 LM cast (buffers included)
            hf.inv_freq.data = hf.inv_freq.data.half()
        cos_hf, sin_hf = hf(x, pos)
        freqs = pos.reshape(-1, 1).float() * plm.rope_inv_freq(cfg, fp16_buffer)[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        assert torch.equal(emb.cos().half(), cos_hf[0]) and torch.equal(emb.sin().half(), sin_hf[0])


def test_synthetic_prefix_layout():
    from pi05_pytorch_fast_b200 import prefix_lm as plm

    emb, pad = plm.synthetic_prefix(2, lang_tokens=200, seed=3)
    assert emb.shape == (2, 776, 2048) and emb.dtype == torch.float16
    assert pad.shape == (2, 776) and int(pad.sum()) == 2 * 628 and not bool(pad[:, 628:].any())
    emb2, _ = plm.synthetic_prefix(1, lang_tokens=64, seed=3)
    assert emb2.shape == (1, 640, 2048)


def test_attention_argument_validation_without_gpu():
    lib = nat.lib()
    fake = 0x1000
    args = lambda **kw: [kw.get("q", fake), kw.get("ldq", 2048), fake, 256, fake, 256, fake, fake,  # noqa: E731
                         kw.get("batch", 1), kw.get("seq", 776), kw.get("heads", 8), fake, fake,
                         kw.get("ldo", 2048), kw.get("cos"), fake, None, 256, None]
    assert "heads must divide 128" in _err(lib.w4a4_prefix_attention(*args(heads=3)))
    assert "exceeds 4096" in _err(lib.w4a4_prefix_attention(*args(seq=5000)))
    assert "16-byte aligned" in _err(lib.w4a4_prefix_attention(*args(q=fake + 2)))
    assert "16-byte aligned" in _err(lib.w4a4_prefix_attention(*args(ldq=1000)))
    assert "invalid attention shape" in _err(lib.w4a4_prefix_attention(*args(batch=-1)))
    assert "RoPE needs" in _err(lib.w4a4_prefix_attention(*args(cos=fake)))
    assert lib.w4a4_prefix_attention(*args(batch=0)) == nat.W4A4_OK
    assert nat.attn_vt_stride(776) == 776 and nat.attn_vt_stride(100) == 104
