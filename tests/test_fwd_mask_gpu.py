"""The one-launch forward (sma_attn_fwd_mask): the attention kernel reads the
bool mask itself and packs it while it scans each query tile.  Its packed
output must equal the mask packer's bit for bit, and its out / lse must equal
those of the two-launch path (pack_mask, then forward on the packed words)
bit for bit: the tile loop is the same code on the same words.  The oracle
checks come from the two-launch path's own tests (test_attn_gpu.py).
sparse_attention() itself keeps the two launches, which are faster on B200."""

import math

import pytest
import torch

from python import pack_mask, sparse_attn_cuda, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def two_launch(q, k, v, m):
    B, H, N, D = q.shape
    packed = pack_mask(m)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=q.device, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, 1.0 / math.sqrt(D), True)
    sparse_attn_cuda.device_status()
    return packed, out, lse


def one_launch(q, k, v, m, with_lse=True):
    B, H, N, D = q.shape
    packed = torch.full((B, H, N, N // 32), -1, dtype=torch.int32, device=q.device)  # every word overwritten
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=q.device, dtype=torch.float32) if with_lse else None
    sparse_attn_cuda.forward_mask(q, k, v, m, packed, out, lse, 1.0 / math.sqrt(D), with_lse)
    sparse_attn_cuda.device_status()
    return packed, out, lse


def check_same(q, k, v, m):
    p2, o2, l2 = two_launch(q, k, v, m)
    p1, o1, l1 = one_launch(q, k, v, m)
    assert torch.equal(p1, p2), "packed words differ from pack_mask"
    assert torch.equal(o1, o2), "out differs from the two-launch forward"
    assert torch.equal(l1, l2), "lse differs from the two-launch forward"
    return o1


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_workloads_match_two_launch_path(name):
    q, k, v, m = workloads.make_inputs(name, seed=5, device=DEV)
    check_same(q, k, v, m)


@pytest.mark.parametrize("N", [32, 96, 160, 224, 288, 544, 1056])
@pytest.mark.parametrize("D,dtype", [(64, torch.float16), (128, torch.bfloat16)])
def test_ragged_tiles(N, D, dtype):
    """N a multiple of 32 but not of 128: a partial last query tile (rows past
    N are not packed) and a partial last key tile; W % 4 != 0 takes the
    scalar word path."""
    g = torch.Generator(device=DEV).manual_seed(N + D)
    q, k, v = (torch.randn(2, 3, N, D, generator=g, device=DEV).to(dtype) for _ in range(3))
    m = torch.rand(2, 3, N, N, generator=g, device=DEV) < 0.2
    m[0, 0, 3, :] = False  # an empty row
    m[1, 2, :, :] = False  # an empty head
    check_same(q, k, v, m)


def test_bytes_other_than_0_and_1():
    """A bool tensor viewed from uint8 can hold any byte; non-zero means
    attend, as in the packer.  Mixed batches take the exact packing."""
    g = torch.Generator(device=DEV).manual_seed(3)
    B, H, N, D = 2, 4, 512, 64
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV).half() for _ in range(3))
    raw = torch.randint(0, 256, (B, H, N, N), generator=g, device=DEV, dtype=torch.uint8)
    raw[raw > 160] = 0  # some zeros, the rest spread over 1..160
    raw[0, 1] = (raw[0, 1] != 0).to(torch.uint8)  # one head of plain 0/1 bytes
    raw[1, :, :, 256:] = 0x80  # high-bit-only bytes
    m = raw.view(torch.bool)
    check_same(q, k, v, m)


def test_empty_items_and_tiles():
    """Whole query tiles with no set bit between live ones, dead key tiles
    (never loaded: their K and V hold NaN) and a zero mask."""
    g = torch.Generator(device=DEV).manual_seed(9)
    B, H, N, D = 8, 40, 512, 64
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV).half() for _ in range(3))
    m = torch.rand(B, H, N, N, generator=g, device=DEV) < 0.25
    m[:, :, 128:384, :] = False           # query tiles 1 and 2 of every head empty
    m[:, ::3, :, 256:384] = False         # key tile 2 dead in every third head
    m[2] = False                          # a zero batch
    k[:, ::3, 256:384] = float("nan")
    v[:, ::3, 256:384] = float("nan")
    out = check_same(q, k, v, m)
    assert not torch.isnan(out).any()


@pytest.mark.parametrize("N,D,dtype", [(8320, 64, torch.float16), (16384, 128, torch.bfloat16)])
def test_long_rows(N, D, dtype):
    """Rows longer than one scan batch many times over, with the L2 prefetch
    of a row issued late (the rows of a round do not fit L2)."""
    g = torch.Generator(device=DEV).manual_seed(N)
    q, k, v = (torch.randn(1, 2, N, D, generator=g, device=DEV).to(dtype) for _ in range(3))
    m = torch.rand(1, 2, N, N, generator=g, device=DEV) < 0.01
    m[..., :128, 2048:6000] = False
    check_same(q, k, v, m)


def test_inference_without_lse():
    q, k, v, m = workloads.make_inputs("c2", seed=2, device=DEV, B=4)
    _, o2, _ = two_launch(q, k, v, m)
    p1, o1, _ = one_launch(q, k, v, m, with_lse=False)
    assert torch.equal(o1, o2)
    assert torch.equal(p1, pack_mask(m))


def test_rejects_unsupported_masks():
    q = torch.randn(1, 1, 48, 64, device=DEV).half()
    m = torch.ones(1, 1, 48, 48, dtype=torch.bool, device=DEV)
    assert not sparse_attn_cuda.forward_mask_supported(m)
    packed = torch.empty(1, 1, 48, 2, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="N % 32"):
        sparse_attn_cuda.forward_mask(q, q, q, m, packed, torch.empty_like(q), None, 0.125, False)


def test_first_cuda_call_of_a_thread():
    """A host thread whose first CUDA work is a call into the library (as the
    autograd worker's is when the backward comes first): the entry points
    bind the device's context themselves before they encode tensor maps."""
    import threading

    q, k, v, m = workloads.make_inputs("c1", seed=6, device=DEV, B=1, H=4)
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    packed = pack_mask(m)
    outs = {name: torch.empty_like(q) for name in ("main", "thread")}
    lses = {name: torch.empty(B, H, N, device=DEV, dtype=torch.float32) for name in outs}
    grads = {name: [torch.empty_like(q) for _ in range(3)] for name in outs}
    dout = torch.randn(q.shape, device=DEV).half()
    torch.cuda.synchronize()

    def run(name):
        sparse_attn_cuda.forward(q, k, v, packed, outs[name], lses[name], scale, True)
        sparse_attn_cuda.backward(dout, q, k, v, outs[name], lses[name], packed, *grads[name], scale)
        sparse_attn_cuda.device_status()

    errors = []

    def body():
        try:
            run("thread")
        except Exception as e:  # reported on the main thread
            errors.append(e)

    t = threading.Thread(target=body)
    t.start()
    t.join()
    assert not errors, errors
    run("main")
    assert torch.equal(outs["thread"], outs["main"])
    (dq_t, dk_t, dv_t), (dq_m, dk_m, dv_m) = grads["thread"], grads["main"]
    assert torch.equal(dk_t, dk_m) and torch.equal(dv_t, dv_m)
    assert (dq_t.float() - dq_m.float()).abs().max() <= 1e-3 * dq_m.float().abs().max()
