"""The allocation-free C entry point ``ecz_linear_bf16_noalloc`` (declared in economize_b200/csrc/noalloc.h).

It exists for callers that cannot allocate GPU memory (a host runtime that owns all device memory, a
latency-critical path where a synchronizing cudaMalloc would stall the device, C code without PyTorch's
allocator): its split-K partials live in a fixed device array inside the library. The test calls it through its
exported C symbol and checks two calls in a row against the regular entry point (``ops.linear``), on shapes that
use the scratch array (split-K) and one that does not, and that an oversized request is refused without a launch.
This file is named to be collected last."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def noalloc(cuda):
    import economize_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.ecz_linear_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p]
    return fn


def _call(fn, x, w, y):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.shape[0], w.shape[0], x.shape[1], stream)


@pytest.mark.parametrize("M,N,K", [(61, 4096, 4096), (7, 6144, 4096), (200, 1024, 512), (300, 16384, 256)])
def test_noalloc_matches_linear(noalloc, cuda, M, N, K):
    from economize_b200 import ops

    g = torch.Generator(device=cuda).manual_seed(11)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    for call in range(2):  # two calls in a row share (and reuse) the scratch array
        x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
        y = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
        assert _call(noalloc, x, w, y) == 0
        torch.cuda.synchronize()
        expect = ops.linear(x, w)
        torch.testing.assert_close(y.float(), expect.float(), atol=2e-2 * expect.abs().max().item() / 4 + 1e-3,
                                   rtol=2e-2)


def test_noalloc_rejects_oversized(noalloc, cuda):
    # on 148 SMs this shape takes 3 K-splits: 3 x 256 x 6144 fp32 partials exceed the 4 Mi-float array
    M, N, K = 256, 6144, 4096
    from economize_b200 import ops

    splits = ops.require().gemm_splits(M, N, K, torch.cuda.get_device_properties(0).multi_processor_count)
    x = torch.zeros(M, K, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(N, K, device=cuda, dtype=torch.bfloat16)
    y = torch.full((M, N), 7.0, device=cuda, dtype=torch.bfloat16)
    rc = _call(noalloc, x, w, y)
    if splits > 1 and splits * M * N > (4 << 20):
        assert rc == -2
        torch.cuda.synchronize()
        assert bool((y == 7.0).all())  # nothing was launched
    else:
        assert rc == 0
    bad = torch.zeros(5, 12, device=cuda, dtype=torch.bfloat16)  # K not a multiple of 8
    assert _call(noalloc, bad, torch.zeros(8, 12, device=cuda, dtype=torch.bfloat16),
                 torch.empty(5, 8, device=cuda, dtype=torch.bfloat16)) == -1


@pytest.fixture(scope="module")
def noalloc_status(cuda):
    import economize_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    status = lib.ecz_linear_bf16_noalloc_status
    status.restype = ctypes.c_int
    status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    selftest = lib.ecz_noalloc_wait_selftest
    selftest.restype = ctypes.c_int
    selftest.argtypes = [ctypes.c_ulonglong, ctypes.c_void_p]
    return status, selftest


def _status(status_fn) -> int:
    word = ctypes.c_uint(12345)
    assert status_fn(ctypes.byref(word)) == 0
    return word.value


def test_noalloc_status_word(noalloc, noalloc_status, cuda):
    """The status word a bounded wait writes reaches the caller: a clean call reads 0, a wait that runs out (the
    self-test waits 1 ms on a barrier nothing completes) reads its code, and the next call clears it again."""
    from economize_b200 import ops

    status_fn, selftest = noalloc_status
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(61, 4096, device=cuda, generator=g).bfloat16()
    w = (torch.randn(4096, 4096, device=cuda, generator=g) * 0.02).bfloat16()
    y = torch.empty(61, 4096, device=cuda, dtype=torch.bfloat16)
    assert _call(noalloc, x, w, y) == 0
    torch.cuda.synchronize()
    assert _status(status_fn) == 0
    assert selftest(1_000_000, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert _status(status_fn) == 1
    assert _call(noalloc, x, w, y) == 0
    torch.cuda.synchronize()
    assert _status(status_fn) == 0
    expect = ops.linear(x, w)
    torch.testing.assert_close(y.float(), expect.float(), atol=2e-2 * expect.abs().max().item() / 4 + 1e-3,
                               rtol=2e-2)
    assert selftest(0, None) == -1  # the limit must be positive


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_second_device(noalloc, cuda):
    """Each device gets its own scratch address and kernel attributes: the entry point on cuda:1 after cuda:0."""
    from economize_b200 import ops

    for dev in (0, 1):
        d = torch.device("cuda", dev)
        with torch.cuda.device(d):
            g = torch.Generator(device=d).manual_seed(5)
            x = torch.randn(61, 4096, device=d, generator=g).bfloat16()
            w = (torch.randn(6144, 4096, device=d, generator=g) * 0.02).bfloat16()
            y = torch.empty(61, 6144, device=d, dtype=torch.bfloat16)
            assert _call(noalloc, x, w, y) == 0
            torch.cuda.synchronize(d)
            expect = ops.linear(x, w)
            torch.testing.assert_close(y.float(), expect.float(),
                                       atol=2e-2 * expect.abs().max().item() / 4 + 1e-3, rtol=2e-2)
