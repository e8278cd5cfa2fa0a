"""The no-allocation C entry point of the W8A16 GEMM, called through its exported C symbol.

That entry point serves callers that cannot allocate device memory (a plain C host program without PyTorch's
allocator, or a serving loop whose memory plan is frozen): its stream-K scratch lives in static device arrays.
Its output must match the PyTorch entry point (``ops.w8a16_linear``: the same kernel, scratch from a tensor) on two
calls in a row; the second call checks that the first returned every ticket to zero. The file name makes pytest
collect it last, so a run that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from hrm_flashrenderer_b200 import ops

ERR_ARG, ERR_TOO_BIG = 1, 2


def _lib():
    if not ops.has_ext():
        pytest.skip("CUDA extension not built")
    import hrm_flashrenderer_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    f = lib.hrm_w8a16_gemm_f16_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.hrm_w8a16_noalloc_last_error.restype = ctypes.c_char_p
    lib.hrm_w8a16_noalloc_check.restype = ctypes.c_int
    lib.hrm_w8a16_noalloc_check.argtypes = [ctypes.POINTER(ctypes.c_int)]
    return lib


def _call(lib, x, w, s, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.hrm_w8a16_gemm_f16_noalloc(x.data_ptr(), x.stride(0), w.data_ptr(), s.data_ptr(), out.data_ptr(),
                                          out.stride(0), x.shape[0], w.shape[0], x.shape[1], stream)


def test_noalloc_rejects_bad_arguments_before_touching_the_device():
    lib = _lib()
    fake = 1 << 20   # never dereferenced: every call below fails its argument checks first
    f = lib.hrm_w8a16_gemm_f16_noalloc
    assert f(fake, 100, fake, fake, fake, 64, 4, 64, 100, None) == ERR_ARG      # K not a multiple of 64
    assert b"multiple of 64" in lib.hrm_w8a16_noalloc_last_error()
    assert f(fake, 60, fake, fake, fake, 64, 4, 64, 64, None) == ERR_ARG       # ldx < K
    assert f(fake, 64, fake, fake, fake, 32, 4, 64, 64, None) == ERR_ARG       # ldo < N
    assert f(None, 64, fake, fake, fake, 64, 4, 64, 64, None) == ERR_ARG       # null pointer
    assert f(fake + 8, 64, fake, fake, fake, 64, 4, 64, 64, None) == ERR_ARG   # x not 16-byte aligned
    assert b"16-byte aligned" in lib.hrm_w8a16_noalloc_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(16, 8192, 8192), (5, 1000, 1024), (1, 4096, 7168), (64, 2048, 2048)])
def test_noalloc_matches_torch_entry_point_twice(M, N, K):
    lib = _lib()
    torch.manual_seed(M * 7 + N)
    dev = torch.device("cuda", 0)
    x = torch.randn(M, K, device=dev).half()
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
    s = torch.rand(N, device=dev) * 1e-3 + 1e-4
    ref = ops.w8a16_linear(x, w, s)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float16, device=dev)
        rc = _call(lib, x, w, s, out)
        assert rc == 0, lib.hrm_w8a16_noalloc_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=1e-3, atol=1e-3)
    code = ctypes.c_int(-1)
    assert lib.hrm_w8a16_noalloc_check(ctypes.byref(code)) == 0
    assert code.value == 0
    # and against plain fp32 math of the same op
    want = x.float() @ (w.float() * s[:, None]).t()
    torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2)


MAX_WS_FLOATS, MAX_TILES = 4 * 1024 * 1024, 4096   # HRM_NOALLOC_MAX_WS_FLOATS / HRM_NOALLOC_MAX_TILES


def _fits(M, N, K):
    """Whether this GPU's stream-K plan of (M, N, K) fits the static scratch (the plan depends on the SM count)."""
    p = ops.gemm_plan(M, N, K)
    return p["ws_floats"] <= MAX_WS_FLOATS and p["counters"] <= MAX_TILES


@pytest.mark.gpu
def test_noalloc_rejects_plans_beyond_the_static_scratch():
    """The expected answer comes from this GPU's own plan, so the test holds on any SM count.  Real buffers of the
    full shape back the call, so an accepted plan would still run within bounds."""
    lib = _lib()
    dev = torch.device("cuda", 0)
    M, N, K = 256, 16384, 4096
    x = torch.zeros(M, K, dtype=torch.float16, device=dev)
    w = torch.zeros(N, K, dtype=torch.int8, device=dev)
    s = torch.ones(N, device=dev)
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    rc = _call(lib, x, w, s, out)
    torch.cuda.synchronize()
    if _fits(M, N, K):
        assert rc == 0, lib.hrm_w8a16_noalloc_last_error()
    else:
        assert rc == ERR_TOO_BIG
        assert b"static limits" in lib.hrm_w8a16_noalloc_last_error()


@pytest.mark.gpu
def test_noalloc_accepts_the_70b_lm_head_at_16_tokens():
    """The header's promise: every decode GEMM of a 70B-class model fits at up to 16 tokens, the widest being the
    128256-row lm_head (K = 8192)."""
    lib = _lib()
    dev = torch.device("cuda", 0)
    M, N, K = 16, 128256, 8192
    assert _fits(M, N, K)
    torch.manual_seed(3)
    x = torch.randn(M, K, device=dev).half()
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev)
    s = torch.rand(N, device=dev) * 1e-3 + 1e-4
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    assert _call(lib, x, w, s, out) == 0, lib.hrm_w8a16_noalloc_last_error()
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), ops.w8a16_linear(x, w, s).float(), rtol=1e-3, atol=1e-3)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_noalloc_on_a_second_device_after_the_first():
    """Per-device set-up: the scratch address and the kernel's shared-memory limit are set on each device the first
    time a call runs with it current, so a call on device 1 after device 0 works."""
    lib = _lib()
    for d in (0, 1):
        with torch.cuda.device(d):
            dev = torch.device("cuda", d)
            torch.manual_seed(d)
            x = torch.randn(16, 4096, device=dev).half()
            w = torch.randint(-127, 128, (8192, 4096), dtype=torch.int8, device=dev)
            s = torch.rand(8192, device=dev) * 1e-3 + 1e-4
            out = torch.empty(16, 8192, dtype=torch.float16, device=dev)
            assert _call(lib, x, w, s, out) == 0, lib.hrm_w8a16_noalloc_last_error()
            torch.cuda.synchronize(dev)
            want = x.float() @ (w.float() * s[:, None]).t()
            torch.testing.assert_close(out.float(), want, rtol=2e-2, atol=2e-2)
