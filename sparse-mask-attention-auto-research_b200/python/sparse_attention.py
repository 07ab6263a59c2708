"""Sparse-mask attention: the reference's Python API on the B200 kernels.

Mirrors python/sparse_attention.py of yulangz/sparse-mask-attention-auto-research:

    sparse_attention(q, k, v, mask)       -> out        (:122-156)
    sparse_attention_func(q, k, v, mask)  -> out        (:159-181, no autograd)
    pack_mask(mask)                       -> int32 bits (:189-206)
    SparseAttentionFunction                              (:52-114)

Inputs are q, k, v [B, H, N, D] (fp16 / bf16, or fp32 which is computed in
bf16 and cast back, as the reference does) and a bool mask [B, H, N, N]
(True = attend).  The softmax scale is 1/sqrt(D).  Rows whose mask is all
False produce 0.

Differences from the reference, all deliberate:
  * CUDA tensors only.  The reference silently falls back to an FP32 PyTorch
    computation for CPU tensors or a missing extension; here both raise
    RuntimeError (the FP32 reference lives in the test oracle, not here).
  * ``sparse_attention_func`` works (the reference passes lse=None to a
    binding that rejects it).
  * ``SparseAttentionFunction.backward`` runs the backward kernel; the
    reference's CUDA backward is an unbound stub (AttributeError when
    called) and its CPU formulas define the result.
  * ``sparse_attention`` builds the autograd node only when an input
    requires a gradient; otherwise it runs the same forward (O and the LSE)
    directly, which saves the node's host cost (same results).
  * ``sparse_attention`` / ``sparse_attention_func`` pack long or large
    masks with the fused packer, which also writes the per-query-tile map of
    live key tiles the attention kernel then uses (same results, no
    re-scan); see ``_pack_for_attention``.
"""

import math

import torch
from torch.autograd import Function

from . import sparse_attn_cuda


class SparseAttentionFunction(Function):
    """Autograd wrapper; forward writes O and the FP32 log-sum-exp like the
    reference (python/sparse_attention.py:52-80, is_training=True)."""

    @staticmethod
    def forward(ctx, q, k, v, mask_packed, mask_bool, scale, seq_len, occupancy=None):
        B, H, N, D = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(B, H, N, device=q.device, dtype=torch.float32)
        sparse_attn_cuda.forward(q, k, v, mask_packed, out, lse, scale, True, occupancy=occupancy)
        ctx.save_for_backward(q, k, v, out, lse, mask_packed, mask_bool)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dout):
        """dq, dk, dv through the backward kernel (reference :82-114; its
        CUDA entry is unbound, its CPU formulas define the result)."""
        q, k, v, out, lse, mask_packed, mask_bool = ctx.saved_tensors
        dout = dout.contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        sparse_attn_cuda.backward(dout, q, k, v, out, lse, mask_packed, dq, dk, dv, ctx.scale)
        return dq, dk, dv, None, None, None, None, None


def _pack_for_attention(mask, head_dim):
    """Packs the mask for the attention kernel; returns (packed, occupancy or None).

    The fused packer's occupancy map lets the head-dim-64 kernel skip its own
    scan of the packed rows.  The map costs the packer about 2 us and saves
    the kernel more than that when the scan is expensive: long rows
    (N >= 1024) or a mask too large to stay in L2 (> 64 MB of bools).  On
    B200 it gains 1-3 us at N = 1024 (causal) and ~40 us at B256 H16 N512,
    and loses ~1 us at B16 H12 N512 and B64 H12 N128, so it is used where it
    wins.  Results are identical either way.
    """
    N = mask.shape[-1]
    if head_dim == 64 and (N >= 1024 or mask.numel() > (64 << 20)):
        return sparse_attn_cuda.pack_mask_occupancy(mask)
    return pack_mask(mask), None


def _check_inputs(q, k, v, mask):
    assert q.shape == k.shape == v.shape, "q/k/v must have the same shape"
    assert q.device == k.device == v.device == mask.device, "all tensors must be on the same device"
    assert mask.dtype == torch.bool, "mask must be a bool tensor"
    if not q.is_cuda:
        raise RuntimeError("sparse_attention requires CUDA tensors (no CPU fallback)")


def sparse_attention(q, k, v, mask):
    """Masked-softmax attention; returns [B, H, N, D] in the input dtype."""
    _check_inputs(q, k, v, mask)
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    orig_dtype = q.dtype
    if orig_dtype == torch.float32:
        q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    mask_packed, occupancy = _pack_for_attention(mask, D)
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        out = SparseAttentionFunction.apply(q, k, v, mask_packed, mask, scale, N, occupancy)
    else:
        # Nothing to differentiate: the same forward (O and the LSE) without
        # the autograd node.
        out = torch.empty_like(q)
        lse = torch.empty(B, H, N, device=q.device, dtype=torch.float32)
        sparse_attn_cuda.forward(q, k, v, mask_packed, out, lse, scale, True, occupancy=occupancy)
    if orig_dtype == torch.float32:
        out = out.float()
    return out


def sparse_attention_func(q, k, v, mask):
    """Inference variant without autograd and without the LSE output."""
    _check_inputs(q, k, v, mask)
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    orig_dtype = q.dtype
    if orig_dtype == torch.float32:
        q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    with torch.no_grad():
        mask_packed, occupancy = _pack_for_attention(mask, D)
        out = torch.empty_like(q)
        sparse_attn_cuda.forward(q, k, v, mask_packed, out, None, scale, False, occupancy=occupancy)
    if orig_dtype == torch.float32:
        out = out.float()
    return out


def pack_mask(mask: torch.Tensor) -> torch.Tensor:
    """bool [B, H, N, N] -> int32 [B, H, N, ceil(N/32)], bit b of word w =
    mask[..., 32*w + b]; bits past N are 0.  Bit-identical to the reference."""
    return sparse_attn_cuda.pack_mask(mask)
