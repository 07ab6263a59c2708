"""The drop-in of the extension module on its own: the reference's unmodified
python/sparse_attention.py imported with this repository's shim standing in
as ``sparse_attn_cuda`` (the "keep the reference's Python file, swap only
the extension" integration).

Runs on the CPU machine where the reference checkout is present; its root is
the one oracle/build_ref.py recorded when it built the reference kernel
(oracle/_ref/reference_root.txt).  The module is imported read-only from
there.  No GPU is needed: with CPU tensors the shim raises the reference
binding's own errors, which shows each call site reached it with arguments
it accepts (a wrong arity would raise TypeError instead).
"""

import ast
import importlib
import importlib.util
import inspect
import math
import os
import sys

import pytest
import torch

from conftest import REPO
from python import sparse_attn_cuda as shim


def _reference_root():
    spec = importlib.util.spec_from_file_location("build_ref", os.path.join(REPO, "oracle", "build_ref.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.recorded_reference_root()


@pytest.fixture(scope="module")
def ref_module():
    root = _reference_root()
    if root is None:
        pytest.skip("reference checkout not present (oracle/_ref/reference_root.txt)")
    saved = {name: sys.modules.get(name) for name in ("sparse_attn_cuda", "python", "python.sparse_attention")}
    sys.modules["sparse_attn_cuda"] = shim
    # The reference module is loaded under its own name from its own file, so
    # this repository's `python` package is left alone.
    path = os.path.join(root, "python", "sparse_attention.py")
    spec = importlib.util.spec_from_file_location("reference_sparse_attention", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    yield mod, path
    for name, m in saved.items():
        if m is None:
            sys.modules.pop(name, None)
        else:
            sys.modules[name] = m


def _extension_calls(path):
    """(line, function name, positional argument count) of every
    sparse_attn_cuda.<fn>(...) call in the reference module."""
    tree = ast.parse(open(path).read())
    calls = []
    for node in ast.walk(tree):
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and isinstance(node.func.value, ast.Name) and node.func.value.id == "sparse_attn_cuda"):
            calls.append((node.lineno, node.func.attr, len(node.args), [k.arg for k in node.keywords]))
    return sorted(calls)


def test_reference_sees_the_extension(ref_module):
    mod, _ = ref_module
    assert mod.HAS_CUDA_EXT is True
    assert mod.sparse_attn_cuda is shim


def test_every_call_site_binds_the_shim_signature(ref_module):
    """forward at :66 and :173, backward at :93, pack_mask at :196."""
    _, path = ref_module
    calls = _extension_calls(path)
    names = sorted({c[1] for c in calls})
    assert names == ["backward", "forward", "pack_mask"], calls
    for line, name, nargs, kwargs in calls:
        sig = inspect.signature(getattr(shim, name))
        sig.bind(*range(nargs), **{k: None for k in kwargs})  # raises TypeError on a mismatch
    assert {(c[1], c[2]) for c in calls} == {("forward", 8), ("backward", 11), ("pack_mask", 1)}


def test_pack_mask_reaches_the_shim(ref_module):
    mod, _ = ref_module
    mask = torch.rand(1, 2, 64, 64) < 0.5
    with pytest.raises(RuntimeError, match="mask must be CUDA tensor"):
        mod.pack_mask(mask)


def test_forward_reaches_the_shim(ref_module):
    """SparseAttentionFunction.forward (:66) hands its CPU tensors to the shim,
    which rejects them with the reference binding's TORCH_CHECK message."""
    mod, _ = ref_module
    B, H, N, D = 1, 2, 64, 64
    q, k, v = (torch.randn(B, H, N, D).half() for _ in range(3))
    mask = torch.rand(B, H, N, N) < 0.5
    packed = torch.zeros(B, H, N, N // 32, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="q must be CUDA tensor"):
        mod.SparseAttentionFunction.apply(q, k, v, packed, mask, 1.0 / math.sqrt(D), N)


def test_cpu_tensors_keep_the_reference_cpu_path(ref_module):
    """sparse_attention() with CPU tensors still takes the reference's own
    FP32 path (:146-151) with the shim installed."""
    mod, _ = ref_module
    B, H, N, D = 1, 1, 32, 64
    q, k, v = (torch.randn(B, H, N, D).half() for _ in range(3))
    mask = torch.rand(B, H, N, N) < 0.5
    out = mod.sparse_attention(q, k, v, mask)
    assert out.dtype == torch.float16
    assert torch.equal(out, mod.sparse_attention_ref(q.float(), k.float(), v.float(), mask).half())
