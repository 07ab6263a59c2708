"""Host-side behaviour of the Python API without a GPU: the reference's
argument checks, the refusal to run on CPU tensors (no fallback), and the
workload generators / roofline arithmetic."""

import math

import pytest
import torch

import python as sma  # noqa: E402
from python import sparse_attn_cuda, workloads


def _qkvm(N=64, D=64, dtype=torch.float16):
    q = torch.randn(1, 2, N, D).to(dtype)
    return q, q.clone(), q.clone(), torch.rand(1, 2, N, N) < 0.5


def test_cpu_tensors_raise_instead_of_falling_back():
    q, k, v, m = _qkvm()
    with pytest.raises(RuntimeError, match="CUDA"):
        sma.sparse_attention(q, k, v, m)
    with pytest.raises(RuntimeError, match="CUDA"):
        sma.sparse_attention_func(q, k, v, m)


def test_reference_assertions():
    q, k, v, m = _qkvm()
    with pytest.raises(AssertionError):
        sma.sparse_attention(q, k[:, :1], v, m)
    with pytest.raises(AssertionError):
        sma.sparse_attention(q, k, v, m.int())


def test_binding_checks_mirror_reference():
    q, k, v, m = _qkvm()
    with pytest.raises(RuntimeError, match="q must be CUDA tensor"):
        sparse_attn_cuda.forward(q, k, v, m, q, None, 0.125, False)
    with pytest.raises(RuntimeError, match="mask must be CUDA tensor"):
        sparse_attn_cuda.pack_mask(m)


def test_make_inputs_deterministic_and_sliceable():
    q, k, v, m = workloads.make_inputs("c2", seed=3, B=2, H=3)
    q2, k2, v2, m2 = workloads.make_inputs("c2", seed=3, B=2, H=3)
    assert torch.equal(q, q2) and torch.equal(m, m2)
    assert q.shape == (2, 3, 128, 64) and m.shape == (2, 3, 128, 128) and q.dtype == torch.float16
    # A shard is exactly the slice of the flattened B*H range.
    qs, ks, vs, ms = workloads.make_inputs("c2", seed=3, B=2, H=3, heads=(1, 5))
    assert torch.equal(qs[0], q.reshape(6, 128, 64)[1:5])
    assert torch.equal(ms[0], m.reshape(6, 128, 128)[1:5])
    assert torch.equal(vs[0], v.reshape(6, 128, 64)[1:5])


@pytest.mark.parametrize("name", ["c3", "c4"])
def test_mask_recipes(name):
    q, k, v, m = workloads.make_inputs(name, seed=0, B=1, H=2)
    N = m.shape[-1]
    assert m[..., torch.arange(N), torch.arange(N)].all(), "diagonal forced"
    if name == "c4":
        assert not torch.triu(m, diagonal=1).any()
        assert abs(m.float().mean().item() - 0.25) < 0.01
    else:
        # 64x64 blocks are either empty or roughly half full
        blocks = m.reshape(1, 2, 16, 64, 16, 64).float().mean(dim=(3, 5))
        off = ~torch.eye(16, dtype=torch.bool)
        vals = blocks[..., off]
        assert ((vals == 0) | ((vals > 0.35) & (vals < 0.65))).all()
        assert abs(m.float().mean().item() - 0.076) < 0.02


@pytest.mark.parametrize("N,num_prev", [(64, 16), (96, 200), (40, 39)])
def test_prefix_random_mask(N, num_prev):
    """The reference sweep's mask (run.py:181-203): row i keeps every key
    j >= i and exactly min(num_prev, i) keys before it, chosen at random."""
    cfg = dict(B=1, H=3, N=N, D=64, dtype=torch.float16, mask="prefix_random", num_prev=num_prev)
    m = workloads.make_inputs(cfg, seed=2)[3][0]
    i = torch.arange(N)
    assert m[:, i[:, None] <= i[None, :]].all(), "every key j >= i is kept"
    before = (m & (i[None, :] < i[:, None])).sum(-1)
    assert torch.equal(before, torch.clamp(i, max=num_prev).expand_as(before))
    if num_prev < N - 1:
        assert not torch.equal(m[0], m[1]), "heads draw their own random keys"


def test_sweep_shapes_follow_the_reference():
    """run.py:497-540: B = 16 up to N = 1024, 4 up to 4096, 2 at 8192, 1 at
    16384; then B 1..64 at N = 512; H12 D64 fp16, num_prev 2048."""
    shapes = dict(workloads.sweep_shapes())
    assert [c["B"] for n, c in shapes.items() if n.startswith("seq")] == [16, 16, 16, 16, 16, 4, 4, 2, 1]
    assert [c["N"] for n, c in shapes.items() if n.startswith("seq")] == [64, 128, 256, 512, 1024, 2048, 4096,
                                                                         8192, 16384]
    assert [c["B"] for n, c in shapes.items() if n.startswith("batch")] == [1, 4, 8, 16, 32, 64]
    assert all(c["H"] == 12 and c["D"] == 64 and c["num_prev"] == 2048 and c["dtype"] == torch.float16
               for c in shapes.values())


def test_roofline_arithmetic():
    assert workloads.dense_flops(16, 12, 512, 64) == 4 * 16 * 12 * 512 * 512 * 64
    b = workloads.attn_bytes(16, 12, 512, 64)
    assert b == 4 * 192 * 512 * 64 * 2 + 192 * 512 * 16 * 4 + 192 * 512 * 4
    assert workloads.pack_bytes(16, 12, 512) == 192 * 512 * 512 + 192 * 512 * 16 * 4
    m = torch.zeros(1, 1, 256, 256, dtype=torch.bool)
    m[0, 0, 0, 200] = True
    assert workloads.live_tile_fraction(m, 128, 128) == 0.25
    assert workloads.live_tile_fraction(m, 128, 64) == 1 / 8
    assert math.isclose(workloads.live_flops(1, 1, 256, 64, 0.25), 4 * 128 * 128 * 64)
