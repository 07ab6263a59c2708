"""sparse_attention_from_host: host inputs streamed through the GPU in
slices give what sparse_attention gives on the same inputs on the device
(bit for bit where both run the same kernels), for one to several slices,
ragged slice bounds, pageable inputs and a caller-provided output."""

import math

import numpy as np
import pytest
import torch

from conftest import out_bound
from oracle import oracle
from python import sparse_attention, workloads
from python.streaming import sparse_attention_from_host

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _host_inputs(name, B=None, H=None, seed=0, pin=True):
    over = {key: val for key, val in (("B", B), ("H", H)) if val is not None}
    q, k, v, m = workloads.make_inputs(name, seed=seed, device=DEV, **over)
    host = tuple(x.cpu() for x in (q, k, v, m))
    if pin:
        host = tuple(x.pin_memory() for x in host)
    return (q, k, v, m), host


@pytest.mark.parametrize("slices", [1, 2, 3, 5])
def test_c1_equals_device_api(slices):
    (q, k, v, m), (hq, hk, hv, hm) = _host_inputs("c1")
    ref = sparse_attention(q, k, v, m).cpu()
    out = sparse_attention_from_host(hq, hk, hv, hm, slices=slices)
    torch.cuda.current_stream().synchronize()
    assert out.is_pinned()
    assert torch.equal(out, ref)


def test_bf16_head_dim_128_ragged_slices_and_out():
    # 2 x 7 = 14 heads in 4 slices (5, 4, 3, 2 heads): every slice smaller than the GPU.
    (q, k, v, m), (hq, hk, hv, hm) = _host_inputs("c3", B=2, H=7, seed=1)
    out = torch.empty(hq.shape, dtype=hq.dtype).pin_memory()
    res = sparse_attention_from_host(hq, hk, hv, hm, slices=4, out=out)
    torch.cuda.synchronize()
    assert res is out
    D = q.shape[-1]
    ref = oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                           m.cpu().numpy(), 1.0 / math.sqrt(D))
    ref_t = torch.from_numpy(ref)
    err = (out.float() - ref_t).abs()
    assert bool((err <= out_bound(ref_t, torch.bfloat16)).all()), f"max err {float(err.max())}"


def test_pageable_inputs_and_repeat_calls():
    (q, k, v, m), (hq, hk, hv, hm) = _host_inputs("c4", B=1, H=4, seed=2, pin=False)
    ref = sparse_attention(q, k, v, m).cpu()
    for _ in range(2):
        out = sparse_attention_from_host(hq, hk, hv, hm, slices=2)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_empty_problem():
    hq = torch.empty(0, 2, 64, 64, dtype=torch.float16)
    hm = torch.empty(0, 2, 64, 64, dtype=torch.bool)
    out = sparse_attention_from_host(hq, hq, hq, hm)
    assert out.shape == hq.shape
