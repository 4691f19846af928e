"""The allocation-free decode attention entry point, called through its
exported C symbol.

The C entry point exists for callers that cannot allocate device memory
(a host runtime that owns all allocations, a plugin behind a plain C ABI):
its split-KV partials live in a static device array inside the library.
Its results are checked against the fp32 PyTorch statement of the op
(``torch_ref.attention`` on CPU copies) and against the regular allocating
op, on consecutive calls that reuse the static scratch.

This file is collected last so that a failure here cannot hide another
test's result in a run that stops at the first failure.
"""

import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="no CUDA device")

OK, TOO_LARGE, BAD_ARG = 0, 1, 2
BAD_POSITION = 3  # status word code for a start position outside the cache


def _lib():
    from afd_demo_b200 import ops

    ops.ext()  # loads the extension into the process
    pkg = os.path.dirname(os.path.abspath(ops.__file__ + "/.."))
    path = glob.glob(os.path.join(pkg, "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.afd_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 8 + [ctypes.c_void_p]
    err = lib.afd_noalloc_error_string
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return fn, err


def _call(fn, q, kc, vc, out, pos, batch_offset, n_split, status=None, max_seq=None,
          max_batch=None):
    B, nq, D = q.shape
    return fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), pos.data_ptr(),
              status.data_ptr() if status is not None else None, B, nq, kc.shape[1], D,
              kc.shape[0] if max_batch is None else max_batch,
              kc.shape[2] if max_seq is None else max_seq, batch_offset, n_split,
              torch.cuda.current_stream().cuda_stream)


def _oracle(q, kc, vc, batch_offset, kv_len):
    """fp32 statement of the op on CPU copies."""
    from afd_demo_b200.ops import torch_ref

    B, nq, D = q.shape
    return torch_ref.attention(q.cpu(), kc.cpu(), vc.cpu(), batch_offset, 1,
                               kv_len - 1).view(B, nq, D).float()


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm())


@needs_cuda
def test_noalloc_matches_fp32_statement_and_regular_op_twice():
    from afd_demo_b200 import ops

    fn, err = _lib()
    dev = "cuda"
    nq, nkv, D, S = 32, 4, 128, 1024
    g = torch.Generator(device=dev).manual_seed(0)
    # two calls in a row share the static scratch; the second is larger
    for call, (B, kv_len, n_split) in enumerate([(8, 300, 4), (16, 777, 8)]):
        kc = torch.randn(B + 2, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(B + 2, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn(B, nq, D, generator=g, device=dev).to(torch.bfloat16)
        pos = torch.tensor([kv_len - 1], device=dev, dtype=torch.int32)
        status = torch.zeros(2, device=dev, dtype=torch.int32)
        out = torch.empty_like(q)
        rc = _call(fn, q, kc, vc, out, pos, 2, n_split, status)
        assert rc == OK, err(rc).decode()
        torch.cuda.synchronize()
        assert status.tolist() == [0, 0]
        ref32 = _oracle(q, kc, vc, 2, kv_len)
        assert _rel(out, ref32) < 1e-2, (call, _rel(out, ref32))
        regular = ops.attention(q, kc, vc, 2, 1, kv_len - 1, pos).view(B, nq, D)
        assert _rel(out, regular) < 1e-2, (call, _rel(out, regular))


@needs_cuda
@pytest.mark.parametrize("n_split", [1, 40])
def test_noalloc_unsplit_and_more_splits_than_key_tiles(n_split):
    """n_split = 1 writes the output directly (no scratch); n_split larger
    than the number of 64-key tiles leaves some splits empty."""
    fn, err = _lib()
    dev = "cuda"
    B, nq, nkv, D, S, kv_len = 4, 16, 2, 64, 512, 130  # 3 key tiles
    g = torch.Generator(device=dev).manual_seed(1)
    kc = torch.randn(B, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(B, nkv, S, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, nq, D, generator=g, device=dev).to(torch.bfloat16)
    pos = torch.tensor([kv_len - 1], device=dev, dtype=torch.int32)
    out = torch.empty_like(q)
    rc = _call(fn, q, kc, vc, out, pos, 0, n_split)
    assert rc == OK, err(rc).decode()
    torch.cuda.synchronize()
    assert _rel(out, _oracle(q, kc, vc, 0, kv_len)) < 1e-2


@needs_cuda
def test_noalloc_start_position_past_the_cache_is_an_error_not_a_read():
    """*start_pos >= max_seq: the kernel must read no key. The buffer is
    allocated longer than the declared layout, so even a broken guard would
    read allocated memory; the guard turns it into zeros plus a status."""
    fn, err = _lib()
    dev = "cuda"
    B, nq, nkv, D, S = 2, 32, 4, 128, 256
    # declared [B, nkv, S, D]; allocated with 2 extra sequences of slack
    kc = torch.randn(B + 2, nkv, S, D, device=dev).to(torch.bfloat16)
    vc = torch.randn(B + 2, nkv, S, D, device=dev).to(torch.bfloat16)
    q = torch.randn(B, nq, D, device=dev).to(torch.bfloat16)
    for n_split in (1, 4):
        pos = torch.tensor([S + 40], device=dev, dtype=torch.int32)
        status = torch.zeros(2, device=dev, dtype=torch.int32)
        out = torch.full_like(q, 7.0)
        rc = _call(fn, q, kc, vc, out, pos, 0, n_split, status, max_seq=S, max_batch=B)
        assert rc == OK, err(rc).decode()
        torch.cuda.synchronize()
        assert int(status[0]) == BAD_POSITION, status.tolist()
        assert torch.count_nonzero(out) == 0
    # a negative position is refused the same way
    pos = torch.tensor([-3], device=dev, dtype=torch.int32)
    status = torch.zeros(2, device=dev, dtype=torch.int32)
    out = torch.full_like(q, 7.0)
    assert _call(fn, q, kc, vc, out, pos, 0, 2, status, max_seq=S, max_batch=B) == OK
    torch.cuda.synchronize()
    assert int(status[0]) == BAD_POSITION and torch.count_nonzero(out) == 0


@needs_cuda
def test_noalloc_rejects_bad_arguments_on_the_host():
    fn, err = _lib()
    dev = "cuda"
    B, nkv, D, S = 4, 4, 128, 64
    kc = torch.zeros(B, nkv, S, D, device=dev, dtype=torch.bfloat16)
    pos = torch.zeros(1, device=dev, dtype=torch.int32)
    q3 = torch.zeros(B, 12, D, device=dev, dtype=torch.bfloat16)  # 12 / 4 = 3 heads per group
    assert _call(fn, q3, kc, kc, torch.empty_like(q3), pos, 0, 1) == BAD_ARG
    q = torch.zeros(B, 32, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    # rows past the cache's sequences
    assert _call(fn, q, kc, kc, out, pos, 1, 1) == BAD_ARG
    assert b"max_batch" in err(BAD_ARG)
    # an empty batch is a no-op
    q0 = torch.zeros(0, 32, D, device=dev, dtype=torch.bfloat16)
    assert _call(fn, q0, kc, kc, torch.empty_like(q0), pos, 0, 1) == OK


@needs_cuda
def test_noalloc_rejects_oversized_request():
    fn, err = _lib()
    dev = "cuda"
    B, nq, nkv, D, S = 64, 32, 4, 128, 64
    kc = torch.zeros(B, nkv, S, D, device=dev, dtype=torch.bfloat16)
    q = torch.zeros(B, nq, D, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    pos = torch.zeros(1, device=dev, dtype=torch.int32)
    rc = _call(fn, q, kc, kc, out, pos, 0, 64)  # 64*32*64*130*4 bytes > 8 MiB
    assert rc == TOO_LARGE and b"8 MiB" in err(rc)
