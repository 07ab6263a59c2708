"""The backward kernel (sma_attn_bwd) against the reference's backward
formulas: golden fixtures made by the reference's own CPU backward
(python/sparse_attention.py:97-111), and the oracle restatement of it on
workload-shaped inputs.  The forward's out and lse come from this library's
forward kernel, as they do in training.

Tolerance: max |grad - FP32 reference| <= tol * max |FP32 reference| per
gradient, tol = 1.5e-2 (fp16) / 4e-2 (bf16).  P and dS are rounded to the
input dtype for the tensor-core products (as in the forward) and the output
gradients to the input dtype; the reference works in FP32 throughout."""

import math

import numpy as np
import pytest
import torch

from conftest import golden_ids, golden_paths, load_golden
from oracle import oracle
from python import pack_mask, sparse_attention, sparse_attn_cuda, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = {torch.float16: 1.5e-2, torch.bfloat16: 4e-2}


def fwd_bwd(q, k, v, m, dout):
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    packed = pack_mask(m)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=q.device, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, scale, True)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    sparse_attn_cuda.backward(dout, q, k, v, out, lse, packed, dq, dk, dv, scale)
    sparse_attn_cuda.device_status()
    return dq, dk, dv


def check_grads(got, want, dtype, mask):
    for g, w, name in zip(got, want, ("dq", "dk", "dv")):
        g = g.float().cpu()
        w = torch.as_tensor(w).float()
        scale = max(float(w.abs().max()), 1e-6)
        err = float((g - w).abs().max())
        assert err <= TOL[dtype] * scale, f"{name}: max abs err {err:.3e} vs max |ref| {scale:.3e}"
        assert torch.isfinite(g).all(), f"{name} has non-finite values"
    m = torch.as_tensor(mask)
    empty_rows = ~m.any(dim=-1)
    empty_cols = ~m.any(dim=-2)
    assert torch.all(got[0].float().cpu()[empty_rows] == 0), "rows with no kept key get dq = 0"
    assert torch.all(got[1].float().cpu()[empty_cols] == 0), "keys no row attends get dk = 0"
    assert torch.all(got[2].float().cpu()[empty_cols] == 0), "keys no row attends get dv = 0"


@pytest.mark.parametrize("path", golden_paths("bwd"), ids=golden_ids("bwd"))
def test_golden(path):
    case = load_golden(path)
    q, k, v, dout, m = (case[x].to(DEV) for x in ("q", "k", "v", "dout", "mask"))
    got = fwd_bwd(q, k, v, m, dout)
    check_grads(got, (case["dq"], case["dk"], case["dv"]), case["dtype"], case["mask"])


@pytest.mark.parametrize("name,kw", [("c1", dict(B=2)), ("c4", dict(B=1, H=2)), ("c2", dict(B=4, dtype=torch.bfloat16)),
                                     ("c3", dict(B=1, H=2)), ("c3", dict(B=1, H=1, N=700, dtype=torch.float16))])
def test_workload_vs_oracle(name, kw):
    q, k, v, m = workloads.make_inputs(name, seed=11, device=DEV, **kw)
    g = torch.Generator(device=DEV).manual_seed(12)
    dout = torch.randn(q.shape, generator=g, device=DEV).to(q.dtype)
    got = fwd_bwd(q, k, v, m, dout)
    D = q.shape[-1]
    want = oracle.attention_backward(*(x.float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / math.sqrt(D), dout.float().cpu().numpy())
    check_grads(got, want, q.dtype, m.cpu())


def test_autograd_through_public_api():
    """loss.backward() through sparse_attention() gives the oracle's gradients."""
    q, k, v, m = workloads.make_inputs("c1", seed=13, device=DEV, B=1, H=2)
    q, k, v = (x.clone().requires_grad_(True) for x in (q, k, v))
    g = torch.Generator(device=DEV).manual_seed(14)
    w = torch.randn(q.shape, generator=g, device=DEV).to(q.dtype)
    out = sparse_attention(q, k, v, m)
    (out.float() * w.float()).sum().backward()
    want = oracle.attention_backward(*(x.detach().float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / math.sqrt(q.shape[-1]), w.float().cpu().numpy())
    check_grads((q.grad, k.grad, v.grad), want, q.dtype, m.cpu())


def test_autograd_head_dim_128():
    q, k, v, m = workloads.make_inputs("c3", seed=18, device=DEV, B=1, H=2)
    q, k, v = (x.clone().requires_grad_(True) for x in (q, k, v))
    g = torch.Generator(device=DEV).manual_seed(19)
    w = torch.randn(q.shape, generator=g, device=DEV).to(q.dtype)
    out = sparse_attention(q, k, v, m)
    (out.float() * w.float()).sum().backward()
    want = oracle.attention_backward(*(x.detach().float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / math.sqrt(128), w.float().cpu().numpy())
    check_grads((q.grad, k.grad, v.grad), want, q.dtype, m.cpu())


def test_fp32_inputs_backward():
    """fp32 q/k/v run in bf16 like the forward; gradients come back in fp32."""
    q, k, v, m = workloads.make_inputs("c2", seed=15, device=DEV, B=1, H=2)
    q, k, v = (x.float().requires_grad_(True) for x in (q, k, v))
    out = sparse_attention(q, k, v, m)
    out.sum().backward()
    assert q.grad.dtype == torch.float32 and torch.isfinite(q.grad).all()
    want = oracle.attention_backward(*(x.detach().bfloat16().float().cpu().numpy() for x in (q, k, v)),
                                     m.cpu().numpy(), 1 / 8.0, np.ones(q.shape, np.float32))
    check_grads((q.grad, k.grad, v.grad), want, torch.bfloat16, m.cpu())


def test_all_masked_gives_zero_gradients():
    N = 256
    g = torch.Generator(device=DEV).manual_seed(16)
    q, k, v, dout = (torch.randn(1, 2, N, 64, generator=g, device=DEV).half() for _ in range(4))
    m = torch.zeros(1, 2, N, N, dtype=torch.bool, device=DEV)
    dq, dk, dv = fwd_bwd(q, k, v, m, dout)
    assert not dq.any() and not dk.any() and not dv.any()


def test_long_sequence_backward():
    """N = 3000 (ragged tiles, 24 key tiles), checked on sampled rows of dq
    and sampled keys of dk/dv against the oracle."""
    N, H = 3000, 1
    g = torch.Generator(device=DEV).manual_seed(17)
    q, k, v, dout = (torch.randn(1, H, N, 64, generator=g, device=DEV).half() for _ in range(4))
    m = torch.rand(1, H, N, N, generator=g, device=DEV) < 0.05
    m[..., 100:300, :] = False
    dq, dk, dv = fwd_bwd(q, k, v, m, dout)
    want = oracle.attention_backward(*(x.float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / 8.0, dout.float().cpu().numpy())
    check_grads((dq, dk, dv), want, torch.float16, m.cpu())


@pytest.mark.parametrize("N,D,dtype", [(5000, 64, torch.float16), (8320, 128, torch.bfloat16)])
def test_long_banded_backward(N, D, dtype):
    """Long rows whose 128x128 tiles are mostly dead: a band around the
    diagonal plus scattered 256x256 blocks, so each key tile's list of live
    query tiles spans several 32-tile words with gaps.  Checked against the
    oracle."""
    g = torch.Generator(device=DEV).manual_seed(23)
    q, k, v, dout = (torch.randn(1, 1, N, D, generator=g, device=DEV).to(dtype) for _ in range(4))
    i = torch.arange(N, device=DEV)
    band = (i[:, None] - i[None, :]).abs() < 300
    nb = (N + 255) // 256
    blocks = torch.rand(nb, nb, generator=g, device=DEV) < 0.04
    blocks = blocks.repeat_interleave(256, 0).repeat_interleave(256, 1)[:N, :N]
    m = (band | (blocks & (torch.rand(N, N, generator=g, device=DEV) < 0.3)))[None, None]
    dq, dk, dv = fwd_bwd(q, k, v, m, dout)
    want = oracle.attention_backward(*(x.float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / math.sqrt(D), dout.float().cpu().numpy())
    check_grads((dq, dk, dv), want, dtype, m.cpu())


@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (128, torch.bfloat16)])
def test_backward_skipped_tiles_do_not_touch_garbage(D, dtype):
    """K / V of key tiles no row attends and Q / dO of query tiles with no kept
    key hold NaN; the backward never reads them, so the gradients match the
    run with clean inputs bit for bit and hold no NaN."""
    N = 512
    g = torch.Generator(device=DEV).manual_seed(29)
    q, k, v, dout = (torch.randn(1, 2, N, D, generator=g, device=DEV).to(dtype) for _ in range(4))
    m = torch.zeros(1, 2, N, N, dtype=torch.bool, device=DEV)
    m[..., 128:384, 128:256] = torch.rand(1, 2, 256, 128, generator=g, device=DEV) < 0.3
    clean = fwd_bwd(q, k, v, m, dout)
    qb, kb, vb, db = (x.clone() for x in (q, k, v, dout))
    for t in (kb, vb):
        t[..., :128, :] = float("nan")
        t[..., 256:, :] = float("nan")
    for t in (qb, db):
        t[..., :128, :] = float("nan")
        t[..., 384:, :] = float("nan")
    dirty = fwd_bwd(qb, kb, vb, m, db)
    live_q = slice(128, 384)
    live_k = slice(128, 256)
    assert torch.equal(dirty[0][..., live_q, :], clean[0][..., live_q, :])
    assert torch.equal(dirty[1][..., live_k, :], clean[1][..., live_k, :])
    assert torch.equal(dirty[2][..., live_k, :], clean[2][..., live_k, :])
    for x in dirty:
        assert not torch.isnan(x).any()


@pytest.mark.parametrize("empty_rounds", [(1,), (1, 2, 3)])
def test_items_without_live_tiles_between_live_items(empty_rounds):
    """Backward work items (batch*head, 128-key tile) that no query row
    attends, between live ones.  CTA c of G takes items c, c + G, c + 2G, ...,
    so emptying whole rounds of items gives every CTA one or three empty
    items in a row; their lists are published by the scanner warp while the
    other warps are still on the live item before them."""
    q, k, v, m = workloads.make_inputs("c1", seed=21, device=DEV)
    B, H, N, D = q.shape
    BH, KT = B * H, N // 128
    G = min(BH * KT, torch.cuda.get_device_properties(0).multi_processor_count)
    m = m.reshape(BH, N, N)
    for rnd in empty_rounds:
        for j in range(G * rnd, min(G * (rnd + 1), BH * KT)):
            bh, kt = j // KT, j % KT
            m[bh, :, kt * 128:(kt + 1) * 128] = False
    m = m.reshape(B, H, N, N)
    g = torch.Generator(device=DEV).manual_seed(22)
    dout = torch.randn(q.shape, generator=g, device=DEV).to(q.dtype)
    got = fwd_bwd(q, k, v, m, dout)
    heads = torch.arange(0, BH, 7, device=DEV)
    sub = [x.reshape(BH, N, D)[heads].unsqueeze(0) for x in got]
    qf, kf, vf, df = (x.reshape(BH, N, D)[heads].unsqueeze(0).float().cpu().numpy() for x in (q, k, v, dout))
    mf = m.reshape(BH, N, N)[heads].unsqueeze(0).cpu()
    want = oracle.attention_backward(qf, kf, vf, mf.numpy(), 1 / math.sqrt(D), df)
    check_grads(sub, want, q.dtype, mf)


def test_backward_after_forward_split_along_keys():
    """Few long items: the forward splits each along keys and merges (O and
    LSE from the merge); the backward consumes them.  Gradients against the
    oracle."""
    B, H, N, D, dtype = 1, 1, 4096, 128, torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(31)
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV).to(dtype) for _ in range(3))
    m = torch.rand(B, H, N, N, generator=g, device=DEV) < 0.05
    m[..., 3, :] = False  # a fully masked row
    dout = torch.randn(q.shape, generator=g, device=DEV).to(dtype)
    got = fwd_bwd(q, k, v, m, dout)
    want = oracle.attention_backward(*(x.float().cpu().numpy() for x in (q, k, v)), m.cpu().numpy(),
                                     1 / math.sqrt(D), dout.float().cpu().numpy())
    check_grads(got, want, dtype, m.cpu())
