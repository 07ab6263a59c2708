"""Sparse attention over host-resident inputs, streamed through the GPU.

``sparse_attention_from_host(q, k, v, mask)`` takes q, k, v [B, H, N, D]
(fp16 / bf16) and the bool mask [B, H, N, N] in host memory and returns the
output [B, H, N, D] in pinned host memory.  The batch*head range crosses
PCIe in contiguous slices on a copy-in stream; each slice is packed and
attended on the current stream as soon as its inputs have landed, and its
output goes back on a copy-out stream, the slices shrinking along the range.
PCIe carries both directions at once
(measured on a B200 host: 88 MB in alone 1.600 ms, with a 12.6 MB read back at the same
time 1.630 ms), so every slice's kernels and read-back except the last
slice's hide under the input copies that follow them.

The results equal ``sparse_attention`` on the same inputs on the device,
slice by slice: every (batch, head) is independent, and a slice is computed
by the same kernels as the whole.  Inputs should be pinned
(``tensor.pin_memory()``) for the copies to overlap; pageable inputs still
give the right result, with the copies serialised.
"""

import math
import threading

import torch

from . import sparse_attn_cuda

_streams = {}
_streams_lock = threading.Lock()


def _copy_streams(device):
    """The copy-in and copy-out streams of `device` (made once, reused)."""
    key = device.index
    s = _streams.get(key)
    if s is None:
        with _streams_lock:
            s = _streams.get(key)
            if s is None:
                s = (torch.cuda.Stream(device), torch.cuda.Stream(device))
                _streams[key] = s
    return s


_SLICE_BYTES = 20 << 20  # input bytes per slice, on average
_MAX_SLICES = 8


def default_slices(bh, input_bytes):
    """Slices for `bh` heads whose inputs (q, k, v and the bool mask) take
    `input_bytes`: about 20 MB each on average, at most 8, at most one per
    head.  On a B200 host the best counts measured were 4 for 88 MB (B16 H12
    N512 D64) and 92 MB (B4 H16 N1024 D64, causal), 2-3 for 50 MB (B64 H12
    N128) and 6-8 for 469 MB (B8 H32 N1024 D128); more, smaller slices pay
    more per-copy and per-launch overhead than they hide."""
    return max(1, min(bh, _MAX_SLICES, input_bytes // _SLICE_BYTES))


def slice_bounds(bh, slices):
    """Bounds of `slices` contiguous parts of range(bh), in decreasing sizes
    (weights slices, slices - 1, ..., 1): only the last part's kernels and
    read-back are not hidden under later copies, so it is the smallest."""
    total = slices * (slices + 1) // 2
    bounds, acc = [0], 0
    for i in range(slices):
        acc += slices - i
        bounds.append(bh * acc // total)
    return bounds


def sparse_attention_from_host(q, k, v, mask, slices=None, out=None):
    """Masked-softmax attention (scale 1/sqrt(D)) of host tensors, computed on
    the current CUDA device; returns the output in pinned host memory.

    q, k, v: [B, H, N, D] fp16 or bf16 in host memory; mask: bool
    [B, H, N, N] in host memory (True = attend).  ``slices``: parts of the
    batch*head range streamed one after another (``default_slices`` when
    None).  ``out``: an optional pinned host tensor of q's shape and dtype to
    write into.

    Like a non_blocking copy, the call returns once the work is queued: the
    current stream waits for the last read-back, so read the result after
    synchronizing that stream (or the device).
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("mask", mask)):
        if t.is_cuda:
            raise RuntimeError(f"{name} must be in host memory (use sparse_attention for device tensors)")
    if q.dim() != 4:
        raise RuntimeError("q must be 4D")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("Unsupported dtype, need BF16 or FP16")
    if not (k.shape == q.shape and v.shape == q.shape and k.dtype == q.dtype and v.dtype == q.dtype):
        raise RuntimeError("q/k/v must have the same shape and dtype")
    B, H, N, D = q.shape
    if mask.dtype != torch.bool or tuple(mask.shape) != (B, H, N, N):
        raise RuntimeError(f"mask must be a bool tensor of shape {(B, H, N, N)}")
    if out is not None and (out.is_cuda or out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous()):
        raise RuntimeError("out must be a contiguous host tensor of q's shape and dtype")
    BH = B * H
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    if BH == 0 or N == 0:
        return out
    if slices is None:
        slices = default_slices(BH, 3 * q.numel() * q.element_size() + mask.numel())
    slices = max(1, min(int(slices), BH))
    scale = 1.0 / math.sqrt(D)
    dev = torch.device("cuda", torch.cuda.current_device())
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _copy_streams(dev)

    qh, kh, vh = (t.contiguous().view(BH, N, D) for t in (q, k, v))
    mh = mask.contiguous().view(BH, N, N)
    oh = out.view(BH, N, D)
    dq, dk, dv, do = (torch.empty((BH, N, D), dtype=q.dtype, device=dev) for _ in range(4))
    dm = torch.empty((BH, N, N), dtype=torch.bool, device=dev)

    # Everything queued on the current stream before this call comes first.
    start = torch.cuda.Event()
    start.record(cur)
    s_in.wait_event(start)
    bounds = slice_bounds(BH, slices)
    parts = [(bounds[i], bounds[i + 1]) for i in range(slices) if bounds[i + 1] > bounds[i]]
    # Every slice's input copies are queued first, so the copy engine never
    # waits on the host for the next one.
    landed = []
    with torch.cuda.stream(s_in):
        for lo, hi in parts:
            for dst, src in ((dm, mh), (dq, qh), (dk, kh), (dv, vh)):
                dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
            landed.append(ev)
    for (lo, hi), ev in zip(parts, landed):
        n = hi - lo
        cur.wait_event(ev)
        packed = sparse_attn_cuda.pack_mask(dm[lo:hi].view(1, n, N, N))
        sparse_attn_cuda.forward(dq[lo:hi].view(1, n, N, D), dk[lo:hi].view(1, n, N, D), dv[lo:hi].view(1, n, N, D),
                                 packed, do[lo:hi].view(1, n, N, D), None, scale, False)
        done = torch.cuda.Event()
        done.record(cur)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            oh[lo:hi].copy_(do[lo:hi], non_blocking=True)
    # The current stream (and so every later allocation from it, and the
    # caller's synchronisation) comes after the last read-back; the device
    # buffers above are only reused by work ordered after it.
    back = torch.cuda.Event()
    back.record(s_out)
    cur.wait_event(back)
    return out
