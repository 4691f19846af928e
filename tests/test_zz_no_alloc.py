"""The allocation-free decode attention entry point, called through its
exported C symbol, must match the regular (allocating) op.

The C entry point exists for callers that cannot allocate device memory
(a host runtime that owns all allocations, a plugin behind a plain C ABI):
its split-KV partials live in a static device array inside the library.
This file is collected last so that a failure here cannot hide another
test's result in a run that stops at the first failure.
"""

import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from afd_demo_b200 import ops

    ops.ext()  # loads the extension into the process
    pkg = os.path.dirname(os.path.abspath(ops.__file__ + "/.."))
    path = glob.glob(os.path.join(pkg, "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.afd_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 7 + [ctypes.c_void_p]
    err = lib.afd_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, q, kc, vc, out, pos, batch_offset, n_split):
    B, nq, D = q.shape
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), pos.data_ptr(), B, nq,
              kc.shape[1], D, kc.shape[2], batch_offset, n_split,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")
def test_noalloc_matches_regular_entry_point_twice():
    from afd_demo_b200 import ops

    fn, err = _lib()
    dev = "cuda"
    nq, nkv, D, S = 32, 4, 128, 1024
    g = torch.Generator(device=dev).manual_seed(0)
    for call, (B, kv_len, n_split) in enumerate([(8, 300, 4), (16, 777, 8)]):
        kc = torch.randn(B + 2, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(B + 2, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn(B, nq, D, generator=g, device=dev).to(torch.bfloat16)
        pos = torch.tensor([kv_len - 1], device=dev, dtype=torch.int32)
        ref = ops.attention(q, kc, vc, 2, 1, kv_len - 1, pos).view(B, nq, D)
        out = torch.empty_like(q)
        rc = _call(fn, q, kc, vc, out, pos, 2, n_split)
        assert rc == 0, err(rc).decode()
        torch.cuda.synchronize()
        rel = float((out.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 1e-2, (call, rel)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")
def test_noalloc_rejects_oversized_request():
    fn, err = _lib()
    dev = "cuda"
    B, nq, nkv, D, S = 64, 32, 4, 128, 64
    kc = torch.zeros(B, nkv, S, D, device=dev, dtype=torch.bfloat16)
    q = torch.zeros(B, nq, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    pos = torch.zeros(1, device=dev, dtype=torch.int32)
    rc = _call(fn, q, kc, kc, out, pos, 0, 64)  # 64*32*64*130*4 bytes > 8 MiB
    assert rc == 1 and b"8 MiB" in err(rc)
