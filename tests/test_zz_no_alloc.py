"""rb_mm_int4_static, the prefill entry point that allocates nothing (its split-K scratch is a file-scope
device array of 8 MiB): the same results as rb_mm_int4_ws with a caller-provided workspace, on two calls in a
row, and RB_ERR_SHAPE for a split that would need more scratch than it has. Collected last on purpose."""
import ctypes

import pytest
import torch

SCRATCH = 8 << 20


def _call(L, fn, x, q, s, m, y, *extra):
    from rumik_fast_b200 import _lib
    T, K = x.shape
    N = q.shape[0]
    args = [x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0), q.data_ptr(), s.data_ptr(), m.data_ptr(),
            y.data_ptr(), _lib.dtype_code(y.dtype), y.stride(0), T, N, K, *extra, 0, _lib.stream_ptr(x.device)]
    return getattr(L, fn)(*args)


def _inputs(M, N, K, seed, dtype=torch.float16):
    from rumik_fast_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    gen = syn.generator(seed, dev)
    q, s, m = syn.int4_weights(N, K, gen, dev)
    x = syn.activations((M, K), gen, dev, dtype=dtype)
    return x, q, s, m


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,xdt,ydt", [
    (34, 3072, 3072, torch.float16, torch.float16),
    (34, 3072, 8192, torch.float16, torch.float16),
    (1024, 3072, 3072, torch.float16, torch.float16),
    (34, 3072, 8192, torch.bfloat16, torch.bfloat16),   # the engine's dtype, converted to fp16 in the kernel
    (34, 3072, 3072, torch.float16, torch.bfloat16),
    (1, 3072, 8192, torch.float16, torch.float16),      # one token: the GEMV path, no scratch used
])
def test_static_scratch_matches_workspace_entry(native_lib, M, N, K, xdt, ydt):
    from rumik_fast_b200 import device_error
    L = native_lib
    x, q, s, m = _inputs(M, N, K, 3, xdt)
    ws_bytes = L.rb_mm_int4_workspace(M, N, K)
    assert ws_bytes <= SCRATCH
    ws = torch.empty(max(ws_bytes // 4, 1), device=x.device, dtype=torch.float32)
    y_ref = torch.empty(M, N, device=x.device, dtype=ydt)
    assert _call(L, "rb_mm_int4_ws", x, q, s, m, y_ref, ctypes.c_void_p(ws.data_ptr()), ws_bytes) == 0
    ys = [torch.full((M, N), float("nan"), device=x.device, dtype=ydt) for _ in range(2)]
    for y in ys:  # two calls in a row on one stream reuse the same scratch
        assert _call(L, "rb_mm_int4_static", x, q, s, m, y) == 0
    torch.cuda.synchronize()
    for y in ys:
        assert torch.equal(y, y_ref)
    assert device_error(x.device) == 0


@pytest.mark.gpu
def test_static_scratch_rejects_oversize_split(native_lib):
    L = native_lib
    M, N, K = 128, 1152, 8192  # 9 row blocks x 16 slices: 9.4 MB of partials, more than 8 MiB
    assert L.rb_mm_int4_workspace(M, N, K) > SCRATCH
    x, q, s, m = _inputs(M, N, K, 4)
    y = torch.empty(M, N, device=x.device, dtype=torch.float16)
    assert _call(L, "rb_mm_int4_static", x, q, s, m, y) == 2  # RB_ERR_SHAPE


@pytest.mark.gpu
def test_static_scratch_rejects_bad_dtype(native_lib):
    L = native_lib
    x, q, s, m = _inputs(34, 3072, 3072, 5)
    y = torch.empty(34, 3072, device=x.device, dtype=torch.float16)
    from rumik_fast_b200 import _lib
    args = [x.data_ptr(), _lib.F32, x.stride(0), q.data_ptr(), s.data_ptr(), m.data_ptr(), y.data_ptr(),
            _lib.F16, y.stride(0), 34, 3072, 3072, 0, _lib.stream_ptr(x.device)]
    assert L.rb_mm_int4_static(*args) == 3  # RB_ERR_DTYPE: X must be fp16 or bf16
