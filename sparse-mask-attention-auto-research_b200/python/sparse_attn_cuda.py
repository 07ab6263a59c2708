"""Drop-in for the reference's compiled extension module ``sparse_attn_cuda``.

Same two functions with the same signatures as the pybind module
(csrc/binding.cpp:68-71), implemented over the C ABI of libsma.so:

    forward(q, k, v, mask_packed, out, lse, scale, is_training) -> None
    pack_mask(mask) -> torch.int32 tensor [B, H, N, ceil(N/32)]

Error behaviour follows the reference's TORCH_CHECKs (RuntimeError for
non-CUDA or non-4-D inputs and for dtypes other than fp16/bf16) and adds
the checks the reference leaves out (matching shapes, contiguity, packed
mask geometry), since the raw kernels would otherwise read out of bounds.
``lse`` may be None when ``is_training`` is False (the reference's
``sparse_attention_func`` passes None there and fails to bind it).

Beyond the reference: ``forward_mask(q, k, v, mask, mask_packed, out, lse,
scale, is_training)`` is the pack + forward pair in one launch: the attention
kernel reads the bool mask, writes the packed words into ``mask_packed`` (for
the backward) and computes ``out`` / ``lse`` exactly as ``forward`` does on
them.  ``forward_mask_supported(mask)`` says when it applies.
``pack_mask_occupancy(mask)`` packs and also returns
the per-(batch*head, 128-row query tile) map of live 128-key tiles, and
``forward(..., occupancy=map)`` lets the kernel skip dead tiles from that
map instead of scanning the packed rows (same results).

Work is enqueued on the current CUDA stream of the tensors' device,
asynchronously, like the reference.
"""

import contextlib

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.SMA_DTYPE_FP16, torch.bfloat16: _lib.SMA_DTYPE_BF16}


# The current stream's handle without building a torch.cuda.Stream object
# (0.1 against 2.3 us per call, measured on a B200 host); the public call where torch
# lacks it.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device):
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _device_guard(device):
    """Makes `device` current for the C call; a no-op when it already is (the common case)."""
    if device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_forward_args(q, k, v, mask_packed, out, lse, is_training):
    """The reference binding's checks plus shape / contiguity; returns the lse pointer."""
    _require(q.is_cuda, "q must be CUDA tensor")
    _require(q.dim() == 4, "q must be 4D")
    _require(q.dtype in _DTYPES, "Unsupported dtype, need BF16 or FP16")
    shape, dtype, device = q.shape, q.dtype, q.device
    B, H, N, D = shape
    for name, t in (("k", k), ("v", v), ("out", out)):
        if not (t.shape == shape and t.dtype == dtype and t.device == device and t.is_contiguous()):
            _require(t.device == device, f"{name} must be on the same device as q")
            _require(t.shape == shape, f"{name} must have the shape of q {tuple(shape)}")
            _require(t.dtype == dtype, f"{name} must have the dtype of q")
            _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(q.is_contiguous(), "q must be contiguous")
    n_words = (N + 31) // 32
    _require(mask_packed.device == q.device, "mask_packed must be on the same device as q")
    _require(mask_packed.dtype in (torch.int32, torch.uint32), "mask_packed must be int32/uint32")
    _require(
        tuple(mask_packed.shape) == (B, H, N, n_words),
        f"mask_packed must have shape {(B, H, N, n_words)}, got {tuple(mask_packed.shape)}",
    )
    _require(mask_packed.is_contiguous(), "mask_packed must be contiguous")
    if not is_training:
        return None
    _require(lse is not None, "lse is required when is_training is true")
    _require(lse.device == q.device, "lse must be on the same device as q")
    _require(lse.dtype == torch.float32, "lse must be float32")
    _require(tuple(lse.shape) == (B, H, N), f"lse must have shape {(B, H, N)}")
    _require(lse.is_contiguous(), "lse must be contiguous")
    return lse.data_ptr()


def forward_mask_supported(mask):
    """True when forward_mask takes this bool mask: N % 32 == 0, contiguous,
    16-byte aligned."""
    N = mask.shape[-1]
    return N % 32 == 0 and mask.is_contiguous() and mask.data_ptr() % 16 == 0


def forward_mask(q, k, v, mask, mask_packed, out, lse, scale, is_training):
    """pack_mask(mask) into ``mask_packed`` and forward(q, k, v, mask_packed,
    out, lse, scale, is_training) in one launch: the attention kernel reads
    the bool mask itself.  ``mask_packed`` ([B, H, N, N/32] int32, 16-byte
    aligned) receives exactly what pack_mask returns; out and lse are those
    forward writes.  Needs forward_mask_supported(mask)."""
    lse_ptr = _check_forward_args(q, k, v, mask_packed, out, lse, is_training)
    B, H, N, D = q.shape
    _require(mask.device == q.device, "mask must be on the same device as q")
    _require(mask.dtype == torch.bool, "mask must be a bool tensor")
    _require(tuple(mask.shape) == (B, H, N, N), f"mask must have shape {(B, H, N, N)}, got {tuple(mask.shape)}")
    _require(forward_mask_supported(mask), "forward_mask needs N % 32 == 0 and a contiguous 16-byte aligned mask")
    _require(mask_packed.data_ptr() % 16 == 0, "mask_packed must be 16-byte aligned")
    lib = _lib.load()
    with _device_guard(q.device):
        _lib.check(
            lib.sma_attn_fwd_mask(
                _DTYPES[q.dtype], q.data_ptr(), k.data_ptr(), v.data_ptr(), mask.data_ptr(), mask_packed.data_ptr(),
                out.data_ptr(), lse_ptr, B, H, N, D, float(scale), _stream_ptr(q.device),
            )
        )


def forward(q, k, v, mask_packed, out, lse, scale, is_training, occupancy=None):
    """Sparse attention forward (reference csrc/binding.cpp:9-47).  The optional
    ``occupancy`` is the map returned by pack_mask_occupancy for this mask."""
    lse_ptr = _check_forward_args(q, k, v, mask_packed, out, lse, is_training)
    B, H, N, D = q.shape
    lib = _lib.load()
    if occupancy is not None:
        q_tiles = (N + 127) // 128
        _require(occupancy.device == q.device, "occupancy must be on the same device as q")
        _require(occupancy.dtype in (torch.int32, torch.uint32), "occupancy must be int32/uint32")
        _require(
            tuple(occupancy.shape) == (B, H, q_tiles, 2),
            f"occupancy must have shape {(B, H, q_tiles, 2)}, got {tuple(occupancy.shape)}",
        )
        _require(occupancy.is_contiguous(), "occupancy must be contiguous")
        with _device_guard(q.device):
            _lib.check(
                lib.sma_attn_fwd_occupancy(
                    _DTYPES[q.dtype], q.data_ptr(), k.data_ptr(), v.data_ptr(), mask_packed.data_ptr(),
                    occupancy.data_ptr(), out.data_ptr(), lse_ptr, B, H, N, D, float(scale),
                    _stream_ptr(q.device),
                )
            )
        return
    with _device_guard(q.device):
        _lib.check(
            lib.sma_attn_fwd(
                _DTYPES[q.dtype],
                q.data_ptr(),
                k.data_ptr(),
                v.data_ptr(),
                mask_packed.data_ptr(),
                out.data_ptr(),
                lse_ptr,
                B,
                H,
                N,
                D,
                float(scale),
                _stream_ptr(q.device),
            )
        )


def backward(dout, q, k, v, out, lse, mask_packed, dq, dk, dv, scale):
    """Sparse attention backward with the signature the reference calls
    (python/sparse_attention.py:93-96; never bound by its csrc/binding.cpp).
    Writes dq, dk, dv (shape and dtype of q) from the forward's out and lse.
    Head dims 64 and 128; the FP32 scratch it needs is allocated here."""
    _require(q.is_cuda, "q must be CUDA tensor")
    _require(q.dim() == 4, "q must be 4D")
    _require(q.dtype in _DTYPES, "Unsupported dtype, need BF16 or FP16")
    B, H, N, D = q.shape
    for name, t in (("k", k), ("v", v), ("out", out), ("dout", dout), ("dq", dq), ("dk", dk), ("dv", dv)):
        _require(t.device == q.device, f"{name} must be on the same device as q")
        _require(t.shape == q.shape, f"{name} must have the shape of q {tuple(q.shape)}")
        _require(t.dtype == q.dtype, f"{name} must have the dtype of q")
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(q.is_contiguous(), "q must be contiguous")
    _require(lse.device == q.device and lse.dtype == torch.float32, "lse must be float32 on the device of q")
    _require(tuple(lse.shape) == (B, H, N) and lse.is_contiguous(), f"lse must be contiguous with shape {(B, H, N)}")
    n_words = (N + 31) // 32
    _require(mask_packed.device == q.device, "mask_packed must be on the same device as q")
    _require(mask_packed.dtype in (torch.int32, torch.uint32), "mask_packed must be int32/uint32")
    _require(
        tuple(mask_packed.shape) == (B, H, N, n_words) and mask_packed.is_contiguous(),
        f"mask_packed must be contiguous with shape {(B, H, N, n_words)}",
    )
    dq_accum = torch.empty((B, H, N, D), dtype=torch.float32, device=q.device)
    delta = torch.empty((B, H, N), dtype=torch.float32, device=q.device)
    lib = _lib.load()
    with _device_guard(q.device):
        _lib.check(
            lib.sma_attn_bwd(
                _DTYPES[q.dtype], q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
                lse.data_ptr(), mask_packed.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                dq_accum.data_ptr(), delta.data_ptr(), B, H, N, D, float(scale), _stream_ptr(q.device),
            )
        )


def pack_mask(mask):
    """bool [B, H, N, N] -> int32 [B, H, N, ceil(N/32)] (reference csrc/binding.cpp:49-66)."""
    _require(mask.is_cuda, "mask must be CUDA tensor")
    _require(mask.dim() == 4, "mask must be 4D [B, H, N, N]")
    _require(mask.dtype == torch.bool, "mask must be a bool tensor")
    B, H, N, N2 = mask.shape
    _require(N == N2, f"mask must be square in its last two dims, got {tuple(mask.shape)}")
    mask = mask.contiguous()
    packed = torch.empty((B, H, N, (N + 31) // 32), dtype=torch.int32, device=mask.device)
    lib = _lib.load()
    with _device_guard(mask.device):
        _lib.check(lib.sma_pack_mask(mask.data_ptr(), packed.data_ptr(), B, H, N, _stream_ptr(mask.device)))
    return packed


def occupancy_supported(mask):
    """True when pack_mask_occupancy can handle this mask's geometry."""
    N = mask.shape[-1]
    return N % 32 == 0 and N <= _lib.SMA_MAX_SEQ_LEN_OCCUPANCY and mask.data_ptr() % 16 == 0


def pack_mask_occupancy(mask):
    """bool [B, H, N, N] -> (int32 packed [B, H, N, ceil(N/32)], int32 occupancy
    [B, H, ceil(N/128), 2] or None).  One pass over the mask; bit t of the
    occupancy pair of query tile qt says whether key tile t has a set bit in
    rows 128qt .. 128qt+127.  Shapes the fused packer does not take (N not a
    multiple of 32, N above the maximum) fall back to pack_mask and None."""
    _require(mask.is_cuda, "mask must be CUDA tensor")
    _require(mask.dim() == 4, "mask must be 4D [B, H, N, N]")
    _require(mask.dtype == torch.bool, "mask must be a bool tensor")
    B, H, N, N2 = mask.shape
    _require(N == N2, f"mask must be square in its last two dims, got {tuple(mask.shape)}")
    mask = mask.contiguous()
    if not occupancy_supported(mask):
        return pack_mask(mask), None
    packed = torch.empty((B, H, N, (N + 31) // 32), dtype=torch.int32, device=mask.device)
    occupancy = torch.empty((B, H, (N + 127) // 128, 2), dtype=torch.int32, device=mask.device)
    lib = _lib.load()
    with _device_guard(mask.device):
        _lib.check(
            lib.sma_pack_mask_occupancy(
                mask.data_ptr(), packed.data_ptr(), occupancy.data_ptr(), B, H, N, _stream_ptr(mask.device)
            )
        )
    return packed, occupancy


def device_status(clear=True, device=None):
    """Synchronise and raise SmaError if a device-side wait of this library
    timed out on ``device`` (default: current device) since the last clear."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(lib.sma_device_status(_stream_ptr(dev), 1 if clear else 0))


def set_wait_timeout_ns(ns):
    """Upper bound (ns) of every device-side wait in later launches."""
    _lib.check(_lib.load().sma_set_wait_timeout_ns(int(ns)))


def debug_wait_probe(timeout_ns, device=None):
    """Launch the bounded-wait probe (a wait nothing satisfies); see
    include/sma_capi.h.  Follow with device_status() to observe the timeout."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(lib.sma_debug_wait_probe(int(timeout_ns), _stream_ptr(dev)))
