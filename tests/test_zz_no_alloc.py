"""The allocation-free LM-head/argmax entry point, called through its C symbol.

Some callers of this library cannot allocate device memory (they run inside a
pre-planned memory budget, or inside another runtime that owns the device
allocator).  ``sc_lm_head_argmax_noalloc`` serves them: it keeps its scratch
in a fixed device array inside the library.  This test calls the exported C
symbol with ctypes and checks it against the regular entry point, which takes
caller-provided scratch, on two calls in a row (the shared scratch and its
counter must be reusable).  The file sorts last so that a run stopping at the
first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    from sparsecache_b200 import ops

    lib = ctypes.CDLL(ops.loaded_library_path())
    fn = lib.sc_lm_head_argmax_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.sc_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _regular(x, w, nw, eps):
    from sparsecache_b200 import ops

    ext = ops.ext()
    M = x.shape[0]
    grid = ext.gemv_argmax_grid(w.shape[0])
    pv = torch.empty(M * grid, device=x.device)
    pi = torch.empty(M * grid, device=x.device, dtype=torch.int32)
    counter = torch.zeros(1, device=x.device, dtype=torch.int32)
    tok = torch.empty(M, device=x.device, dtype=torch.int32)
    ext.gemv_argmax(x, w, nw, eps, pv, pi, counter, tok, None, None, None, None, None)
    return tok


def test_noalloc_entry_point_matches_regular(cuda_device):
    fn, err = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    eps = 1e-5
    for call, (M, N, K) in enumerate([(3, 32000, 4096), (8, 4096, 1024)]):
        g = torch.Generator(device="cpu").manual_seed(100 + call)
        x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
        nw = (1 + 0.1 * torch.randn(K, generator=g)).to(cuda_device, torch.bfloat16)
        expect = _regular(x, w, nw, eps)
        got = torch.full((M,), -1, device=cuda_device, dtype=torch.int32)
        rc = fn(x.data_ptr(), w.data_ptr(), nw.data_ptr(), eps, M, N, K, got.data_ptr(), stream)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert torch.equal(got, expect), (got.tolist(), expect.tolist())


def test_noalloc_without_norm_and_ties(cuda_device):
    """norm_w = NULL uses x as given; tied logits resolve to the lowest row index."""
    fn, err = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cpu").manual_seed(7)
    M, N, K = 4, 4096, 512
    x = torch.randn(M, K, generator=g).to(cuda_device, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.05).to(cuda_device, torch.bfloat16)
    for call in range(2):
        expect = _regular(x, w, None, 1e-5)
        got = torch.full((M,), -1, device=cuda_device, dtype=torch.int32)
        rc = fn(x.data_ptr(), w.data_ptr(), None, 1e-5, M, N, K, got.data_ptr(), stream)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        assert torch.equal(got, expect), (call, got.tolist(), expect.tolist())
    # rows 17, 900 and 3000 become copies of row 0's winning row: their
    # logits tie exactly, and the lowest index of the tied rows must win
    w2 = w.clone()
    logits = (x.float() @ w2.float().t())
    best = int(logits[0].argmax())
    for j in (17, 900, 3000):
        w2[j] = w2[best]
    got = torch.full((M,), -1, device=cuda_device, dtype=torch.int32)
    rc = fn(x.data_ptr(), w2.data_ptr(), None, 1e-5, M, N, K, got.data_ptr(), stream)
    assert rc == 0, err(rc).decode()
    torch.cuda.synchronize()
    expect = _regular(x, w2, None, 1e-5)
    assert torch.equal(got, expect)
    assert int(got[0]) == min(17, best)


def test_noalloc_rejects_oversized_calls(cuda_device):
    fn, err = _symbol()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(9, 64, device=cuda_device, dtype=torch.bfloat16)
    w = torch.zeros(64, 64, device=cuda_device, dtype=torch.bfloat16)
    out = torch.zeros(9, device=cuda_device, dtype=torch.int32)
    rc = fn(x.data_ptr(), w.data_ptr(), None, 1e-5, 9, 64, 64, out.data_ptr(), stream)
    assert rc == 1 and b"M <= 8" in err(rc)
    rc = fn(x.data_ptr(), w.data_ptr(), None, 1e-5, 1, 64, 60, out.data_ptr(), stream)
    assert rc == 1
    # misaligned x (a view starting 1 element into the buffer) and NULL x
    xa = torch.zeros(2, 72, device=cuda_device, dtype=torch.bfloat16)
    rc = fn(xa.data_ptr() + 2, w.data_ptr(), None, 1e-5, 1, 64, 64, out.data_ptr(), stream)
    assert rc == 5 and b"16-byte aligned" in err(rc)
    rc = fn(None, w.data_ptr(), None, 1e-5, 1, 64, 64, out.data_ptr(), stream)
    assert rc == 5
