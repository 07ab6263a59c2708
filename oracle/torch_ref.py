"""ORACLE — test and measurement infrastructure only; nothing in the product
imports it.

The reference's own CPU path for the hot path, restated in torch so that it
can be timed on the host cores with every thread torch is given:

    sparse_attention(q, k, v, mask) on CPU tensors
        python/sparse_attention.py:122-156 (the CPU branch, :150-151)
        -> sparse_attention_ref(q.float(), k.float(), v.float(), mask).to(dtype)
           python/sparse_attention.py:26-44
    log-sum-exp of the scaled masked scores, the fallback of
        SparseAttentionFunction.forward, python/sparse_attention.py:72-76
        (-inf for rows with no kept key; the CUDA path writes -FLT_MAX)

The numpy oracle (oracle/oracle.py) is the checker the tests pin against
the golden fixtures; this module is the same arithmetic in the reference's
own library, used as the CPU baseline and the reference arm of bench.py.
"""

import math

import torch


def sparse_attention_ref(q, k, v, mask):
    """FP32 dense masked softmax attention (python/sparse_attention.py:26-44)."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    scores = scores.masked_fill(~mask, float("-inf"))
    attn = torch.softmax(scores, dim=-1)
    attn = torch.nan_to_num(attn, nan=0.0)
    return torch.matmul(attn, v)


def sparse_attention_cpu(q, k, v, mask):
    """The reference's sparse_attention() for CPU tensors (:138-156): fp32
    inputs go through bf16 as on the CUDA path, the FP32 reference runs on
    the (possibly rounded) inputs, and the result is cast back."""
    orig = q.dtype
    if orig == torch.float32:
        q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out = sparse_attention_ref(q.float(), k.float(), v.float(), mask).to(q.dtype)
    return out.float() if orig == torch.float32 else out


def lse_ref(q, k, mask):
    """Natural-log LSE of the scaled masked scores (python/sparse_attention.py:72-76)."""
    D = q.shape[-1]
    scores = torch.matmul(q.float(), k.float().transpose(-2, -1)) / math.sqrt(D)
    scores = scores.masked_fill(~mask, float("-inf"))
    return torch.logsumexp(scores, dim=-1)
