"""The native ops refuse host tensors with a clear error before any CUDA call
(each launching binding checks its tensors' device first and then makes that
device current). Runs without a GPU; skipped when the extension is not built."""

import re

import pytest
import torch


@pytest.fixture(scope="module")
def C():
    try:
        from afd_demo_b200 import _C  # noqa: F401
    except ImportError:
        pytest.skip("afd_demo_b200._C is not built")
    from afd_demo_b200 import ops

    return ops.ext()


def _bf(*shape):
    return torch.zeros(*shape, dtype=torch.bfloat16)


def _i32(*shape):
    return torch.zeros(*shape, dtype=torch.int32)


@pytest.mark.parametrize("name,call,arg", [
    ("argmax", lambda C: C.argmax(_bf(2, 8), torch.zeros(2, dtype=torch.long), None, None),
     "logits"),
    ("moe_gather", lambda C: C.moe_gather(_bf(2, 8), _i32(2), _i32(1), _bf(2, 8), 2), "x"),
    ("add_i32", lambda C: C.add_i32(_i32(1), 1), "t"),
    ("peer_copy", lambda C: C.peer_copy(_bf(4, 8), [], [], 1, None, None, 1), "src"),
    ("sum_rmsnorm", lambda C: C.sum_rmsnorm([_bf(2, 8)], _bf(8), None, _bf(2, 8), 1e-6, [], 0,
                                            None, 0, None), "parts[0]"),
])
def test_host_tensors_are_refused(C, name, call, arg):
    with pytest.raises(RuntimeError, match=re.escape(f"{arg} must be a CUDA tensor")):
        call(C)
