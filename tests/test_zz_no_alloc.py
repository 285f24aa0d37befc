"""w4a4_int4_gemm_noalloc: the op path with library-owned static scratch.

The file is named to be collected last: the no-allocation entry point shares
one static scratch per device, so it runs after every other test and must
also pass alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w4a4_oracle as orc
from pi05_pytorch_fast_b200 import _native as nat


def _descs(weights, layout=nat.LAYOUT_ROW_MAJOR):
    return nat.weights_array([(w.data_ptr(), int(w.size(0)), int(w.size(1)), layout) for w in weights])


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    lib = nat.lib()
    fake = 0x1000  # never dereferenced: the size check comes first
    w = nat.weights_array([(fake, 64, 2048 // 8 + 8, nat.LAYOUT_ROW_MAJOR)])
    y = nat.pointer_array([fake])
    rows = nat.NOALLOC_MAX_ROWS + 1
    assert lib.w4a4_int4_gemm_noalloc(fake, rows, 64, 64, -1, 0, 1, w, y, None) == nat.W4A4_ERR_UNSUPPORTED
    assert "exceeds its static scratch" in nat.last_error()
    m = nat.NOALLOC_MAX_CODES // 16384 + 1  # m * k just past the code limit
    assert lib.w4a4_int4_gemm_noalloc(fake, m, 16384, 16384, -1, 0, 1, w, y, None) == nat.W4A4_ERR_UNSUPPORTED
    assert "exceeds its static scratch" in nat.last_error()


def _run_both(x: torch.Tensor, weights):
    """Outputs of the existing entry point (torch scratch) and of the
    no-allocation one, on the same inputs."""
    m, k = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    descs = _descs(weights)
    ref = [torch.empty((m, int(w.size(0))), dtype=torch.float16, device=x.device) for w in weights]
    codes = torch.empty((m, k), dtype=torch.int8, device=x.device)
    scales = torch.empty((m,), dtype=torch.float32, device=x.device)
    nat.check(nat.lib().w4a4_int4_gemm(x.data_ptr(), m, k, k, nat.ROTATE_BY_K, nat.STAGING_FP16,
                                       len(weights), descs, nat.pointer_array([t.data_ptr() for t in ref]),
                                       codes.data_ptr(), scales.data_ptr(), stream))
    out = [torch.empty_like(t) for t in ref]
    nat.check(nat.lib().w4a4_int4_gemm_noalloc(x.data_ptr(), m, k, k, nat.ROTATE_BY_K, nat.STAGING_FP16,
                                               len(weights), descs,
                                               nat.pointer_array([t.data_ptr() for t in out]), stream))
    return ref, out


@pytest.mark.gpu
def test_noalloc_matches_the_scratch_entry_point_on_consecutive_calls():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # call 1: a fused q/k/v-like GEMM (K = 2048, three weights)
    x1 = torch.from_numpy(orc.make_activations(776, 2048, seed=11)).to(dev)
    w1 = [torch.from_numpy(orc.pad_rows(orc.random_packed_weight(n, 2048, seed=20 + i), 2048 // 8 + 8)).to(dev)
          for i, n in enumerate((2048, 256, 256))]
    # call 2, right after: a down_proj-like GEMM (K = 16384, other rows)
    x2 = torch.from_numpy(orc.make_activations(300, 16384, seed=12)).to(dev)
    w2 = [torch.from_numpy(orc.pad_rows(orc.random_packed_weight(2048, 16384, seed=30), 16384 // 8 + 8)).to(dev)]
    ref1, out1 = _run_both(x1, w1)
    ref2, out2 = _run_both(x2, w2)
    torch.cuda.synchronize()
    for a, b in zip(ref1 + ref2, out1 + out2):
        assert torch.equal(a, b)
    # and the first shape again, after the scratch held the second call's codes
    ref3, out3 = _run_both(x1, w1)
    torch.cuda.synchronize()
    for a, b in zip(ref3, out3):
        assert torch.equal(a, b)
    assert nat.device_error(clear=True) == 0
