"""Generate the golden fixtures in tests/golden/ by running the reference's
own CPU code (yulangz/sparse-mask-attention-auto-research, python/sparse_attention.py).

Run in a container where the reference is mounted, naming its root:

    python tests/golden/make_golden.py --reference <reference root>
    (or SMA_REFERENCE_ROOT=<reference root> python tests/golden/make_golden.py)

The reference module is imported read-only; with no compiled extension it
takes its CPU paths:
  pack_mask()                     python/sparse_attention.py:189-206 (CPU fallback)
  sparse_attention_ref()          python/sparse_attention.py:26-44   (FP32 oracle, as run.py:435)
  SparseAttentionFunction.forward python/sparse_attention.py:52-80   (fallback LSE, :67-76)
  generate_random_sparse_mask()   python/sparse_attention.py:209-239 (the reference's own masks)
  SparseAttentionFunction.backward python/sparse_attention.py:82-114 (its CPU formulas; run on FP32
                                  copies of the fp16/bf16 inputs so the gradients stay in FP32)

Each case is one .npz: q/k/v as raw 16-bit patterns plus their dtype name,
the bool mask bit-packed with numpy (little bit order), the reference's FP32
output, its LSE (-inf for rows with no kept key), and for pack cases the
reference's int32 packed words.  Inputs come from torch's CPU generator with
the seed stored in the file.
"""

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _save(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


class _Ctx:
    def save_for_backward(self, *tensors):
        self.saved = tensors


def attention_case(ref, name, q, k, v, mask, seed, note):
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    out = ref.sparse_attention_ref(q.float(), k.float(), v.float(), mask)
    packed = ref.pack_mask(mask)
    ctx = _Ctx()
    ref.SparseAttentionFunction.forward(ctx, q, k, v, packed, mask, scale, N)
    lse = ctx.saved[4]
    meta = dict(kind="attention", name=name, shape=[B, H, N, D], dtype=str(q.dtype).replace("torch.", ""),
                seed=seed, scale=scale, note=note,
                reference=["python/sparse_attention.py:26-44", "python/sparse_attention.py:67-76",
                           "python/sparse_attention.py:189-206"])
    _save(name, q=_bits16(q), k=_bits16(k), v=_bits16(v),
          mask=np.packbits(mask.numpy(), axis=-1, bitorder="little"), n=np.int64(N),
          out=out.numpy().astype(np.float32), lse=lse.numpy().astype(np.float32),
          packed=packed.numpy().astype(np.int32), meta=json.dumps(meta))
    print(f"{name}: {meta['shape']} {meta['dtype']} density={mask.float().mean().item():.4f}")


def backward_case(ref, name, q, k, v, mask, dout, seed, note):
    """The reference's backward formulas (python/sparse_attention.py:97-111)
    on FP32 copies of the 16-bit inputs, so dq/dk/dv are its FP32 results."""
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    qf, kf, vf, dof = q.float(), k.float(), v.float(), dout.float()
    packed = ref.pack_mask(mask)
    ctx = _Ctx()
    ref.SparseAttentionFunction.forward(ctx, qf, kf, vf, packed, mask, scale, N)
    lse = ctx.saved[4]
    ctx.saved_tensors = ctx.saved
    ctx.scale = scale
    dq, dk, dv = ref.SparseAttentionFunction.backward(ctx, dof)[:3]
    meta = dict(kind="backward", name=name, shape=[B, H, N, D], dtype=str(q.dtype).replace("torch.", ""),
                seed=seed, scale=scale, note=note,
                reference=["python/sparse_attention.py:82-114", "python/sparse_attention.py:26-44",
                           "python/sparse_attention.py:67-76"])
    _save(name, q=_bits16(q), k=_bits16(k), v=_bits16(v), dout=_bits16(dout),
          mask=np.packbits(mask.numpy(), axis=-1, bitorder="little"), n=np.int64(N),
          lse=lse.numpy().astype(np.float32), dq=dq.numpy().astype(np.float32),
          dk=dk.numpy().astype(np.float32), dv=dv.numpy().astype(np.float32), meta=json.dumps(meta))
    print(f"{name}: {meta['shape']} {meta['dtype']} backward density={mask.float().mean().item():.4f}")


def pack_case(ref, name, mask, seed, note):
    packed = ref.pack_mask(mask)
    meta = dict(kind="pack", name=name, shape=list(mask.shape), seed=seed, note=note,
                reference=["python/sparse_attention.py:189-206"])
    _save(name, mask=np.packbits(mask.numpy(), axis=-1, bitorder="little"), n=np.int64(mask.shape[-1]),
          packed=packed.numpy().astype(np.int32), meta=json.dumps(meta))
    print(f"{name}: {list(mask.shape)} density={mask.float().mean().item():.4f}")


def qkv(gen, B, H, N, D, dtype, mult=1.0):
    q = (torch.randn(B, H, N, D, generator=gen) * mult).to(dtype)
    k = (torch.randn(B, H, N, D, generator=gen) * mult).to(dtype)
    v = torch.randn(B, H, N, D, generator=gen).to(dtype)
    return q, k, v


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SMA_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $SMA_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference root with --reference or SMA_REFERENCE_ROOT")
    sys.path.insert(0, args.reference)
    import importlib

    ref = importlib.import_module("python.sparse_attention")  # the reference module, CPU paths

    assert not ref.HAS_CUDA_EXT, "expected the reference's CPU fallback paths"

    # ---------------------------------------------------------------- pack cases
    seed = 1
    gen = torch.Generator().manual_seed(seed)
    for n in (1, 7, 8, 31, 32, 33, 40, 64, 100, 128, 255, 512):
        for dens in (0.0, 0.25, 0.75, 1.0):
            m = torch.rand(1, 2, n, n, generator=gen) < dens
            pack_case(ref, f"pack_N{n}_d{int(dens * 100)}", m, seed, "Bernoulli mask")
    m = torch.zeros(1, 1, 64, 64, dtype=torch.bool)
    m[..., 31] = True
    m[..., 63] = True
    pack_case(ref, "pack_bit31", m, 0, "only columns 31 and 63 set: sign bit of each word")

    # ---------------------------------------------------------------- attention cases
    # The reference's correctness cases (run.py:416-456): B2 H4 D64 fp16, seed
    # 42, masks from its own generator (all-True for N <= 2049).
    for n in (64, 128):
        gen = torch.Generator().manual_seed(42)
        q, k, v = qkv(gen, 2, 4, n, 64, torch.float16)
        mask = ref.generate_random_sparse_mask(2, 4, n, num_random_prev=2048, device="cpu")
        attention_case(ref, f"attn_refcase_N{n}", q, k, v, mask, 42, "run.py:416-456 shapes; reference mask generator")

    # Fully-masked row (run.py:458-467).
    gen = torch.Generator().manual_seed(7)
    q, k, v = qkv(gen, 1, 1, 8, 64, torch.float16)
    mask = torch.ones(1, 1, 8, 8, dtype=torch.bool)
    mask[:, :, 0, :] = False
    attention_case(ref, "attn_masked_row_N8", q, k, v, mask, 7, "run.py:458-467: row 0 fully masked")

    def bern(gen, B, H, N, keep):
        return torch.rand(B, H, N, N, generator=gen) < keep

    cases = []
    # Reduced-size versions of the five benchmark workloads' mask recipes.
    gen = torch.Generator().manual_seed(101)
    q, k, v = qkv(gen, 1, 2, 512, 64, torch.float16)
    cases.append(("attn_c1_mini", q, k, v, bern(gen, 1, 2, 512, 0.25), 101, "c1 recipe, B1 H2"))
    gen = torch.Generator().manual_seed(102)
    q, k, v = qkv(gen, 2, 3, 128, 64, torch.float16)
    cases.append(("attn_c2_mini", q, k, v, bern(gen, 2, 3, 128, 0.25), 102, "c2 recipe, B2 H3"))
    gen = torch.Generator().manual_seed(103)
    q, k, v = qkv(gen, 1, 1, 1024, 128, torch.bfloat16)
    alive = (torch.rand(1, 1, 16, 16, generator=gen) >= 0.85).repeat_interleave(64, 2).repeat_interleave(64, 3)
    m = alive & (torch.rand(1, 1, 1024, 1024, generator=gen) < 0.5)
    m |= torch.eye(1024, dtype=torch.bool)
    cases.append(("attn_c3_mini", q, k, v, m, 103, "c3 recipe (64x64 dead tiles), B1 H1"))
    gen = torch.Generator().manual_seed(104)
    q, k, v = qkv(gen, 1, 1, 1024, 64, torch.float16)
    i = torch.arange(1024)
    m = (i[None, :] <= i[:, None]) & (torch.rand(1, 1, 1024, 1024, generator=gen) < 0.5)
    m |= torch.eye(1024, dtype=torch.bool)
    cases.append(("attn_c4_mini", q, k, v, m, 104, "c4 recipe (causal), B1 H1"))

    # Ragged sequence lengths (partial query and key tiles).
    gen = torch.Generator().manual_seed(105)
    q, k, v = qkv(gen, 1, 2, 40, 128, torch.bfloat16)
    m = bern(gen, 1, 2, 40, 0.5)
    m[0, 1, 5, :] = False
    cases.append(("attn_N40_bf16_D128", q, k, v, m, 105, "N=40, one fully masked row"))
    gen = torch.Generator().manual_seed(106)
    q, k, v = qkv(gen, 2, 1, 100, 64, torch.float16)
    cases.append(("attn_N100_fp16_D64", q, k, v, bern(gen, 2, 1, 100, 0.3), 106, "N=100"))
    gen = torch.Generator().manual_seed(107)
    q, k, v = qkv(gen, 1, 1, 200, 128, torch.float16)
    cases.append(("attn_N200_fp16_D128", q, k, v, bern(gen, 1, 1, 200, 0.25), 107, "N=200, D=128 fp16"))
    gen = torch.Generator().manual_seed(108)
    q, k, v = qkv(gen, 1, 2, 256, 64, torch.bfloat16)
    cases.append(("attn_N256_bf16_D64", q, k, v, bern(gen, 1, 2, 256, 0.25), 108, "bf16, D=64"))

    # Tile-skip invariants.
    gen = torch.Generator().manual_seed(109)
    q, k, v = qkv(gen, 1, 2, 256, 64, torch.float16)
    cases.append(("attn_zero_mask_N256", q, k, v, torch.zeros(1, 2, 256, 256, dtype=torch.bool), 109,
                  "all rows masked: every key tile skipped"))
    gen = torch.Generator().manual_seed(110)
    q, k, v = qkv(gen, 1, 1, 300, 64, torch.float16)
    cols = torch.randint(0, 300, (300,), generator=gen)
    m = torch.zeros(1, 1, 300, 300, dtype=torch.bool)
    m[0, 0, torch.arange(300), cols] = True
    cases.append(("attn_single_bit_N300", q, k, v, m, 110, "one kept key per row: out row = that v row"))
    gen = torch.Generator().manual_seed(111)
    q, k, v = qkv(gen, 1, 1, 512, 64, torch.float16)
    m = torch.zeros(1, 1, 512, 512, dtype=torch.bool)
    m[0, 0, 128:256, 256:320] = torch.rand(128, 64, generator=gen) < 0.5
    cases.append(("attn_one_live_tile_N512", q, k, v, m, 111, "a single live (query tile, key tile) block"))

    # Large score range: q, k ~ N(0, 64) so the running max jumps between tiles.
    gen = torch.Generator().manual_seed(112)
    q, k, v = qkv(gen, 1, 2, 512, 64, torch.float16, mult=8.0)
    cases.append(("attn_large_scores_N512", q, k, v, bern(gen, 1, 2, 512, 0.25), 112, "q,k scaled by 8"))
    gen = torch.Generator().manual_seed(113)
    q, k, v = qkv(gen, 1, 1, 1024, 128, torch.bfloat16, mult=4.0)
    i = torch.arange(1024)
    m = (i[None, :] >= i[:, None]) & (torch.rand(1, 1, 1024, 1024, generator=gen) < 0.3)
    cases.append(("attn_anticausal_bf16_D128", q, k, v, m, 113, "upper-triangular, last row has one key"))

    for name, q, k, v, m, seed, note in cases:
        attention_case(ref, name, q, k, v, m, seed, note)

    # ---------------------------------------------------------------- backward cases
    bcases = []
    gen = torch.Generator().manual_seed(201)
    q, k, v = qkv(gen, 1, 2, 512, 64, torch.float16)
    bcases.append(("bwd_c1_mini", q, k, v, bern(gen, 1, 2, 512, 0.25), 201, "c1 recipe, B1 H2"))
    gen = torch.Generator().manual_seed(202)
    q, k, v = qkv(gen, 2, 1, 100, 64, torch.float16)
    m = bern(gen, 2, 1, 100, 0.3)
    m[1, 0, 7, :] = False
    bcases.append(("bwd_N100_fp16", q, k, v, m, 202, "N=100 (partial tiles), one fully masked row"))
    gen = torch.Generator().manual_seed(203)
    q, k, v = qkv(gen, 1, 2, 256, 64, torch.bfloat16)
    bcases.append(("bwd_N256_bf16", q, k, v, bern(gen, 1, 2, 256, 0.25), 203, "bf16"))
    gen = torch.Generator().manual_seed(204)
    q, k, v = qkv(gen, 1, 1, 1024, 64, torch.float16)
    i = torch.arange(1024)
    m = (i[None, :] <= i[:, None]) & (torch.rand(1, 1, 1024, 1024, generator=gen) < 0.5)
    m |= torch.eye(1024, dtype=torch.bool)
    bcases.append(("bwd_c4_mini", q, k, v, m, 204, "c4 recipe (causal): dead blocks above the diagonal"))
    gen = torch.Generator().manual_seed(205)
    q, k, v = qkv(gen, 1, 1, 512, 64, torch.float16, mult=4.0)
    m = torch.zeros(1, 1, 512, 512, dtype=torch.bool)
    m[0, 0, 128:384, 256:448] = torch.rand(256, 192, generator=gen) < 0.4
    bcases.append(("bwd_block_N512", q, k, v, m, 205, "live block only; larger scores; zero rows and columns"))
    gen = torch.Generator().manual_seed(206)
    q, k, v = qkv(gen, 1, 1, 200, 128, torch.bfloat16)
    bcases.append(("bwd_N200_bf16_D128", q, k, v, bern(gen, 1, 1, 200, 0.3), 206, "D=128 (oracle only)"))
    for name, q, k, v, m, seed, note in bcases:
        g2 = torch.Generator().manual_seed(seed + 1000)
        dout = torch.randn(q.shape, generator=g2).to(q.dtype)
        backward_case(ref, name, q, k, v, m, dout, seed, note)


if __name__ == "__main__":
    main()
