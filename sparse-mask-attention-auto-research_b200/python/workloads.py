"""The five benchmark workloads and their seeded synthetic inputs, plus the
per-workload roofline arithmetic.

Workloads (q, k, v ~ N(0, 1); scale 1/sqrt(D); True = attend):
  c1  B16  H12 N512  D64  fp16  Bernoulli keep 0.25                   (headline)
  c2  B64  H12 N128  D64  fp16  Bernoulli keep 0.25                   (short sequences)
  c3  B8   H32 N1024 D128 bf16  64x64 tiles dead w.p. 0.85, keep 0.5 inside, diagonal kept
  c4  B4   H16 N1024 D64  fp16  causal AND Bernoulli keep 0.5, diagonal kept
  c5  B256 H16 N512  D64  fp16  Bernoulli keep 0.25                   (multi-GPU sweep)

Inputs are generated per head from a seed so that any slice of the flattened
B*H range (a multi-GPU shard) is exactly the slice of the global tensors.

The reference's performance sweep (run.py:483-540) uses a further mask,
"prefix_random" (run.py:181-203): row i attends every key j >= i plus
min(num_prev, i) keys j < i drawn uniformly without replacement
(num_prev = 2048, H12 D64 fp16); sweep_shapes() lists its shapes.
"""

import math

import torch

CONFIGS = {
    "c1": dict(B=16, H=12, N=512, D=64, dtype=torch.float16, mask="bernoulli", keep=0.25),
    "c2": dict(B=64, H=12, N=128, D=64, dtype=torch.float16, mask="bernoulli", keep=0.25),
    "c3": dict(B=8, H=32, N=1024, D=128, dtype=torch.bfloat16, mask="block", tile=64, dead=0.85, keep=0.5),
    "c4": dict(B=4, H=16, N=1024, D=64, dtype=torch.float16, mask="causal", keep=0.5),
    "c5": dict(B=256, H=16, N=512, D=64, dtype=torch.float16, mask="bernoulli", keep=0.25),
}

# Heads generated per RNG draw; seeds are per block so shards are slices.
_HEAD_BLOCK = 16


def describe(name):
    c = CONFIGS[name]
    dt = {torch.float16: "fp16", torch.bfloat16: "bf16"}[c["dtype"]]
    return f"B{c['B']}H{c['H']}N{c['N']}D{c['D']} {dt} mask={c['mask']}"


def _mask_block(cfg, nh, N, gen, device):
    kind = cfg["mask"]
    if kind == "bernoulli":
        return torch.rand(nh, N, N, generator=gen, device=device) < cfg["keep"]
    if kind == "block":
        t = cfg["tile"]
        nt = (N + t - 1) // t
        alive = torch.rand(nh, nt, nt, generator=gen, device=device) >= cfg["dead"]
        alive = alive.repeat_interleave(t, 1).repeat_interleave(t, 2)[:, :N, :N]
        m = alive & (torch.rand(nh, N, N, generator=gen, device=device) < cfg["keep"])
        m |= torch.eye(N, dtype=torch.bool, device=device)
        return m
    if kind == "prefix_random":
        # Keys j >= i, plus the num_prev lowest of uniform scores among j < i
        # (all of them when i <= num_prev), one head at a time to bound memory.
        i = torch.arange(N, device=device)
        later = i[None, :] >= i[:, None]
        k = min(cfg["num_prev"], N - 1)
        if k >= N - 1:
            return torch.ones(nh, N, N, dtype=torch.bool, device=device)
        heads = []
        for _ in range(nh):
            scores = torch.rand(N, N, generator=gen, device=device)
            scores.masked_fill_(later, float("inf"))
            idx = torch.topk(scores, k, dim=-1, largest=False).indices
            del scores
            m = torch.zeros(N, N, dtype=torch.bool, device=device)
            m.scatter_(-1, idx, True)
            m &= ~later
            m |= later
            heads.append(m)
        return torch.stack(heads)
    if kind == "causal":
        i = torch.arange(N, device=device)
        causal = i[None, :] <= i[:, None]
        m = causal & (torch.rand(nh, N, N, generator=gen, device=device) < cfg["keep"])
        m |= torch.eye(N, dtype=torch.bool, device=device)
        return m
    raise ValueError(kind)


def sweep_shapes():
    """The reference's performance sweep (run.py:497-540): sequence-length
    scaling with B chosen by N, and batch scaling at N = 512; H12 D64 fp16,
    prefix_random masks with num_prev 2048.  Returns (name, cfg) pairs."""
    base = dict(H=12, D=64, dtype=torch.float16, mask="prefix_random", num_prev=2048)
    out = []
    for N in (64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384):
        B = 16 if N <= 1024 else 4 if N <= 4096 else 2 if N <= 8192 else 1
        out.append((f"seq N{N} B{B}", dict(base, B=B, N=N)))
    for B in (1, 4, 8, 16, 32, 64):
        out.append((f"batch B{B} N512", dict(base, B=B, N=512)))
    return out


def make_inputs(name_or_cfg, seed=0, device="cpu", heads=None, **overrides):
    """Seeded q, k, v [B', H', N, D] and bool mask [B', H', N, N].

    ``heads=(lo, hi)`` selects a contiguous slice of the flattened B*H range
    (returned with shape [1, hi-lo, N, D]); without it the full [B, H, ...]
    tensors are returned.  ``overrides`` replace config fields (e.g. B=2 for
    a reduced-size variant with the same mask recipe).
    """
    cfg = dict(CONFIGS[name_or_cfg]) if isinstance(name_or_cfg, str) else dict(name_or_cfg)
    cfg.update(overrides)
    B, H, N, D, dtype = cfg["B"], cfg["H"], cfg["N"], cfg["D"], cfg["dtype"]
    BH = B * H
    lo, hi = (0, BH) if heads is None else heads
    device = torch.device(device)
    qs, ks, vs, ms = [], [], [], []
    b0 = lo // _HEAD_BLOCK
    b1 = (hi + _HEAD_BLOCK - 1) // _HEAD_BLOCK
    for blk in range(b0, b1):
        h0 = blk * _HEAD_BLOCK
        nh = min(_HEAD_BLOCK, BH - h0)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed * 1_000_003 + blk)
        q = torch.randn(nh, N, D, generator=gen, device=device).to(dtype)
        k = torch.randn(nh, N, D, generator=gen, device=device).to(dtype)
        v = torch.randn(nh, N, D, generator=gen, device=device).to(dtype)
        m = _mask_block(cfg, nh, N, gen, device)
        s0 = max(lo, h0) - h0
        s1 = min(hi, h0 + nh) - h0
        qs.append(q[s0:s1])
        ks.append(k[s0:s1])
        vs.append(v[s0:s1])
        ms.append(m[s0:s1])
    q, k, v, m = (torch.cat(x) for x in (qs, ks, vs, ms))
    if heads is None:
        shape = (B, H)
    else:
        shape = (1, hi - lo)
    return (
        q.reshape(*shape, N, D).contiguous(),
        k.reshape(*shape, N, D).contiguous(),
        v.reshape(*shape, N, D).contiguous(),
        m.reshape(*shape, N, N).contiguous(),
    )


# ------------------------------------------------------------------ roofline


def dense_flops(B, H, N, D):
    """Dense-equivalent FLOPs of one forward, 4*B*H*N^2*D (reference run.py:232-237)."""
    return 4.0 * B * H * N * N * D


def attn_bytes(B, H, N, D, elem=2, with_lse=True):
    """Algorithmic HBM bytes of the attention kernel: read Q, K, V and the
    packed mask once, write O (and the FP32 LSE)."""
    bh = B * H
    qkvo = 4 * bh * N * D * elem
    packed = bh * N * ((N + 31) // 32) * 4
    lse = bh * N * 4 if with_lse else 0
    return qkvo + packed + lse


def backward_flops(B, H, N, D):
    """Dense-equivalent FLOPs of one backward: five N x N x D products
    (S, dP, dV, dK, dQ), 10*B*H*N^2*D."""
    return 10.0 * B * H * N * N * D


def backward_bytes(B, H, N, D, elem=2):
    """Algorithmic HBM bytes of the backward: read Q, K, V, O, dO, the packed
    mask and the LSE once, write dQ, dK, dV.  (The FP32 dQ accumulator adds
    a clear, the partial sums and a final read on top.)"""
    bh = B * H
    return 8 * bh * N * D * elem + bh * N * ((N + 31) // 32) * 4 + bh * N * 4


def pack_bytes(B, H, N):
    """Algorithmic HBM bytes of pack_mask: read N^2 bytes, write N^2/8."""
    bh = B * H
    return bh * N * N + bh * N * ((N + 31) // 32) * 4


def live_tile_fraction(mask, bm=128, bn=128):
    """Fraction of (query tile, key tile) blocks with at least one set bit."""
    B, H, N, _ = mask.shape
    qt = (N + bm - 1) // bm
    kt = (N + bn - 1) // bn
    m = torch.zeros(B, H, qt * bm, kt * bn, dtype=torch.bool, device=mask.device)
    m[:, :, :N, :N] = mask
    blocks = m.view(B, H, qt, bm, kt, bn).any(dim=5).any(dim=3)
    return blocks.float().mean().item()


def live_flops(B, H, N, D, live_frac, bm=128, bn=128):
    """MMA FLOPs the kernel issues: 4*bm*bn*D per live tile pair."""
    qt = (N + bm - 1) // bm
    kt = (N + bn - 1) // bn
    return 4.0 * bm * bn * D * B * H * qt * kt * live_frac


def kernel_tile(D):
    """(BM, BN) of the attention kernel for head dim D."""
    return (128, 128) if D == 64 else (128, 64)


def scale_for(D):
    return 1.0 / math.sqrt(D)
