"""Kernels launched on a second GPU of the same process: kernel attributes (dynamic shared memory above 48 KB) and
cached per-device state must be set up per device, not once per process."""

import pytest
import torch

from economize_b200 import ops
from economize_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gemm_and_attention_on_device_1_after_device_0():
    ops.require()
    for dev in (0, 1):
        d = torch.device("cuda", dev)
        with torch.cuda.device(d):
            g = torch.Generator(device=d).manual_seed(7)
            for M in (1, 61, 300):  # cluster split-K, cluster split-K, persistent stream-K
                x = torch.randn(M, 4096, device=d, generator=g).bfloat16()
                w = (torch.randn(6144, 4096, device=d, generator=g) * 0.02).bfloat16()
                y = ops.linear(x, w)
                expect = x.float() @ w.float().T
                torch.testing.assert_close(y.float(), expect, atol=2e-2 * expect.abs().max().item() / 4 + 1e-3,
                                           rtol=2e-2)
            B, T, H, Hkv, S, D = 1, 61, 32, 8, 1024, 128
            k = torch.randn(B, Hkv, S, D, device=d, generator=g).bfloat16()
            v = torch.randn(B, Hkv, S, D, device=d, generator=g).bfloat16()
            q = torch.randn(B, T, H, D, device=d, generator=g).bfloat16()
            kv_len = torch.tensor([700], dtype=torch.int32, device=d)
            n_new = torch.tensor([T], dtype=torch.int32, device=d)
            out = ops.attention(q, k, v, kv_len, n_new)
            want = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, None)
            torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=2e-2)
            torch.cuda.synchronize(d)
            assert ops.require().status(dev) == 0
