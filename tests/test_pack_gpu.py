"""pack_mask on the GPU is bit-exact against the reference (golden fixtures
from the reference's CPU packer) and against the oracle on every workload's
mask at full size."""

import numpy as np
import pytest
import torch

from conftest import golden_ids, golden_paths, load_golden
from oracle import oracle
from python import pack_mask, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("path", golden_paths("pack") + golden_paths("attn"), ids=golden_ids("pack") + golden_ids("attn"))
def test_pack_golden_bit_exact(path):
    case = load_golden(path)
    got = pack_mask(case["mask"].to(DEV)).cpu()
    assert got.dtype == torch.int32
    assert torch.equal(got, case["packed"])


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_pack_full_workload_vs_oracle(name):
    _, _, _, m = workloads.make_inputs(name, seed=11, device=DEV)
    got = pack_mask(m).cpu().numpy()
    want = oracle.pack_mask_parallel(m.cpu().numpy())
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [1, 5, 31, 33, 63, 95, 127, 129, 1000])
def test_pack_ragged_n(n):
    g = torch.Generator(device=DEV).manual_seed(n)
    m = torch.rand(2, 3, n, n, generator=g, device=DEV) < 0.4
    got = pack_mask(m).cpu().numpy()
    assert np.array_equal(got, oracle.pack_mask(m.cpu().numpy()))


def test_pack_non_contiguous_and_expanded():
    g = torch.Generator(device=DEV).manual_seed(0)
    base = torch.rand(1, 1, 128, 128, generator=g, device=DEV) < 0.5
    expanded = base.expand(2, 3, 128, 128)
    got = pack_mask(expanded).cpu().numpy()
    assert np.array_equal(got, oracle.pack_mask(expanded.cpu().numpy()))
    transposed = base.transpose(-1, -2)
    assert np.array_equal(pack_mask(transposed).cpu().numpy(), oracle.pack_mask(transposed.cpu().numpy()))


def test_pack_misaligned_storage():
    # A view starting one byte into its storage takes the general path.
    g = torch.Generator(device=DEV).manual_seed(1)
    flat = torch.rand(1 + 2 * 64 * 64, generator=g, device=DEV) < 0.5
    view = flat[1:].view(1, 2, 64, 64)
    assert np.array_equal(pack_mask(view).cpu().numpy(), oracle.pack_mask(view.cpu().numpy()))


def test_pack_nonzero_bytes_count_as_true():
    raw = torch.tensor([0, 1, 2, 128, 255, 0, 7, 0] * 8, dtype=torch.uint8, device=DEV)
    m = raw.view(torch.bool).view(1, 1, 8, 8)
    want = oracle.pack_mask((raw.cpu().numpy() != 0).reshape(1, 1, 8, 8))
    got = pack_mask(m).cpu().numpy()
    assert np.array_equal(got, want)
