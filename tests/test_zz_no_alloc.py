"""``pp_quad_gemm_static_scratch``: the split-K scratch in a device array of
the library, for callers that cannot call cudaMalloc (plugin hosts whose own
pool owns all device memory, code that must not allocate because cudaMalloc
can synchronise the device).

Compared with ``pp_quad_gemm`` (caller workspace) on two calls in a row.
The file name sorts last, so the test also runs after every other GPU test
has used the library; it passes alone as well.
"""
import ctypes

import numpy as np
import pytest
import torch

from polar_pack_b200 import _lib

pytestmark = pytest.mark.gpu


def _problem(K, N, M, layout, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    codes = torch.randint(-2**31, 2**31 - 1, (N, K), generator=g, dtype=torch.int32)
    if layout == "kn":
        codes = codes.t().contiguous()                           # (K, N), N contiguous
    luts = [torch.rand(256, generator=g).half()] + [(torch.rand(256, generator=g) * 2 - 1).half()
                                                     for _ in range(6)]
    x = torch.randn(M, K, generator=g).half()
    return codes, luts, x


def _views(codes, layout):
    # (K, N) view of the codes and its element strides
    if layout == "kn":
        return codes, codes.stride(0), codes.stride(1)
    v = codes.t()                                                # file layout: K contiguous
    return v, v.stride(0), v.stride(1)


def _run(fn_name, dev, codes, luts, x, layout, use_ws):
    L = _lib.load()
    cv, ldk, ldn = _views(codes, layout)
    K, N = cv.shape
    M = x.shape[0]
    outs = [torch.full((M, N), float("nan"), dtype=torch.half, device=dev) for _ in range(4)]
    args = [x.data_ptr(), x.stride(0), x.stride(1), cv.data_ptr(), ldk, ldn, _lib.ptrs(luts, 7),
            _lib.floats4([0.5, 1.0, 1.5, 2.0]), _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1),
            M, N, K]
    stream = _lib.stream_handle(dev)
    if use_ws:
        nb = ctypes.c_size_t()
        _lib.check(L.pp_quad_gemm_workspace_bytes(M, N, K, ldk, ldn, ctypes.byref(nb)))
        ws = torch.zeros(nb.value + 256, dtype=torch.uint8, device=dev)
        _lib.check(getattr(L, fn_name)(*args, ws.data_ptr(), nb.value, stream))
    else:
        _lib.check(getattr(L, fn_name)(*args, stream))
    torch.cuda.synchronize(dev)
    return [o.cpu() for o in outs]


@pytest.mark.parametrize("layout,K,N,M", [("nk", 2048, 2048, 1), ("nk", 2048, 11008, 3), ("nk", 1024, 512, 16),
                                          ("kn", 2048, 1024, 2), ("kn", 512, 2048, 6)])
def test_static_scratch_matches_workspace_entry_point(cuda, layout, K, N, M):
    codes, luts, x = _problem(K, N, M, layout, seed=K + N + M)
    codes, luts, x = codes.to(cuda), [t.to(cuda) for t in luts], x.to(cuda)
    ref = _run("pp_quad_gemm", cuda, codes, luts, x, layout, use_ws=True)
    for _ in range(2):                                            # two calls in a row
        got = _run("pp_quad_gemm_static_scratch", cuda, codes, luts, x, layout, use_ws=False)
        for k in range(4):
            assert not torch.isnan(got[k]).any()
            np.testing.assert_array_equal(got[k].numpy().view(np.uint16), ref[k].numpy().view(np.uint16))


def test_static_scratch_allocates_no_device_memory(cuda):
    """The entry point's reason to exist: free device memory (cudaMemGetInfo)
    is the same before and after two calls, with every buffer allocated
    before the first measurement."""
    codes, luts, x = _problem(2048, 11008, 3, "nk", seed=9)
    codes, luts, x = codes.to(cuda), [t.to(cuda) for t in luts], x.to(cuda)
    cv, ldk, ldn = _views(codes, "nk")
    K, N = cv.shape
    outs = [torch.empty((3, N), dtype=torch.half, device=cuda) for _ in range(4)]
    L = _lib.load()
    args = (x.data_ptr(), x.stride(0), x.stride(1), cv.data_ptr(), ldk, ldn, _lib.ptrs(luts, 7),
            _lib.floats4([0.5, 1.0, 1.5, 2.0]), _lib.ptrs(outs, 4), outs[0].stride(0), outs[0].stride(1),
            3, N, K, _lib.stream_handle(cuda))
    _lib.check(L.pp_quad_gemm_static_scratch(*args))            # warm-up: the first call's set-up
    torch.cuda.synchronize(cuda)
    free0 = torch.cuda.mem_get_info(cuda)[0]
    for _ in range(2):
        _lib.check(L.pp_quad_gemm_static_scratch(*args))
    torch.cuda.synchronize(cuda)
    assert torch.cuda.mem_get_info(cuda)[0] == free0


def test_static_scratch_rejects_plans_beyond_its_size(cuda):
    # kernel layout at 16 batch rows: ~2.4 MB of partial slots on a 148-SM part
    codes, luts, x = _problem(4096, 8192, 16, "kn", seed=5)
    codes, luts, x = codes.to(cuda), [t.to(cuda) for t in luts], x.to(cuda)
    cv, ldk, ldn = _views(codes, "kn")
    nb = ctypes.c_size_t()
    L = _lib.load()
    _lib.check(L.pp_quad_gemm_workspace_bytes(16, 8192, 4096, ldk, ldn, ctypes.byref(nb)))
    if nb.value <= (1 << 20):
        pytest.skip("device too small for the plan to exceed the static scratch")
    outs = [torch.empty(16, 8192, dtype=torch.half, device=cuda) for _ in range(4)]
    rc = L.pp_quad_gemm_static_scratch(x.data_ptr(), x.stride(0), x.stride(1), cv.data_ptr(), ldk, ldn,
                                       _lib.ptrs(luts, 7), _lib.floats4([1, 1, 1, 1]), _lib.ptrs(outs, 4),
                                       8192, 1, 16, 8192, 4096, _lib.stream_handle(cuda))
    assert rc == _lib.PP_ERR_WORKSPACE
    assert b"static scratch" in L.pp_last_error()
