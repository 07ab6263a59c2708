"""The fused packer (pack + occupancy map) on the GPU: its packed words are
the reference's bits, its map equals the oracle's live (query tile, key tile)
blocks, and attention driven by the map gives bitwise the same output and
LSE as attention that scans the packed rows itself."""

import math

import numpy as np
import pytest
import torch

from conftest import golden_paths, load_golden
from oracle import oracle
from python import pack_mask, sparse_attention, sparse_attn_cuda, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _occ_cases():
    out = []
    for path in golden_paths("pack") + golden_paths("attn"):
        n = load_golden(path)["mask"].shape[-1]
        if n % 32 == 0:
            out.append(path)
    return out


@pytest.mark.parametrize("path", _occ_cases(), ids=lambda p: p.split("/")[-1][:-4])
def test_fused_pack_golden(path):
    case = load_golden(path)
    packed, occ = sparse_attn_cuda.pack_mask_occupancy(case["mask"].to(DEV))
    assert occ is not None
    assert torch.equal(packed.cpu(), case["packed"])
    assert np.array_equal(occ.cpu().numpy(), oracle.occupancy(case["mask"].numpy()))


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_fused_pack_full_workload(name):
    heads = (0, 512) if name == "c5" else None
    _, _, _, m = workloads.make_inputs(name, seed=5, device=DEV, heads=heads)
    packed, occ = sparse_attn_cuda.pack_mask_occupancy(m)
    assert torch.equal(packed, pack_mask(m))
    assert np.array_equal(occ.cpu().numpy(), oracle.occupancy(m.cpu().numpy()))


def test_unsupported_shapes_fall_back():
    m = torch.rand(1, 2, 100, 100, device=DEV) < 0.3
    packed, occ = sparse_attn_cuda.pack_mask_occupancy(m)
    assert occ is None
    assert torch.equal(packed, pack_mask(m))


def _fwd(q, k, v, packed, occ):
    B, H, N, D = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=DEV, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, 1.0 / math.sqrt(D), True, occupancy=occ)
    return out, lse


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_attention_with_map_is_identical(name):
    heads = (0, 512) if name == "c5" else None
    q, k, v, m = workloads.make_inputs(name, seed=9, device=DEV, heads=heads)
    packed, occ = sparse_attn_cuda.pack_mask_occupancy(m)
    o1, l1 = _fwd(q, k, v, packed, None)
    o2, l2 = _fwd(q, k, v, packed, occ)
    sparse_attn_cuda.device_status()
    assert torch.equal(o1, o2)
    assert torch.equal(l1, l2)


def test_sparse_blocks_and_empty_items():
    # Whole query tiles without a set bit, and key tiles dead for some query tiles only.
    g = torch.Generator(device=DEV).manual_seed(3)
    B, H, N, D = 2, 3, 640, 64
    q, k, v = (torch.randn(B, H, N, D, generator=g, device=DEV).half() for _ in range(3))
    m = torch.rand(B, H, N, N, generator=g, device=DEV) < 0.2
    m[:, :, 128:256, :] = False        # query tile 1: empty item
    m[:, :, :, 384:512] = False        # key tile 3 dead everywhere
    m[0, 1, 512:, :128] = False        # key tile 0 dead for query tile 4 of one head
    packed, occ = sparse_attn_cuda.pack_mask_occupancy(m)
    assert np.array_equal(occ.cpu().numpy(), oracle.occupancy(m.cpu().numpy()))
    o1, l1 = _fwd(q, k, v, packed, None)
    o2, l2 = _fwd(q, k, v, packed, occ)
    sparse_attn_cuda.device_status()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    assert torch.count_nonzero(o2[:, :, 128:256]) == 0


@pytest.mark.parametrize("name", ["c1", "c4"])
def test_public_api_matches_the_scan_path(name):
    # c4 (N = 1024) goes through the fused packer and the map, c1 through the plain packer.
    from python.sparse_attention import _pack_for_attention

    q, k, v, m = workloads.make_inputs(name, seed=2, device=DEV, heads=(0, 4))
    assert (_pack_for_attention(m, q.shape[-1])[1] is not None) == (name == "c4")
    o1, _ = _fwd(q, k, v, pack_mask(m), None)
    assert torch.equal(sparse_attention(q, k, v, m), o1)
