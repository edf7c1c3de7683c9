"""Seeded synthetic workloads (Qwen layer-0 FFN shapes; no real weights here).

Each generator is deterministic for its seed.  Small tensors use a CPU
``torch.Generator``; the large weight arrays are drawn on the target device
(a CUDA generator is far faster than drawing 267M values on the host), so
the same seed gives the same weights on the same GPU/torch build.

* decode (``decode_layer``): hidden 5120, intermediate 17408, weights
  ~ N(0, 0.02^2) drawn directly in neuron-major packed form (every element is
  iid, so this is the same distribution as packing three separately drawn
  matrices), x ~ N(0, 1), ids = sort(randperm(N, seed=1000+token)[:K]).
* selector (``selector_scores``): fp32 scores ~ Laplace(0, 1) per token; a
  hot 10% of neurons (seeded permutation) gets boost c*(i+1)^-1.1, c = 8, for
  the i-th hot neuron (Zipf(1.1)-ranked).
* offload (``offload_hot_set`` / ``offload_token_ids``): 25% of the
  intermediate neurons (seeded permutation) are "hot" and stay in HBM; per
  token K = ceil(0.1 N) ids, token 0 drawing 80% of them from the hot set and
  20% from the cold rest; every later token keeps a seeded 50% of the
  previous token's ids and draws the rest 80/20 hot/cold, without
  replacement, from neurons it does not already hold.  Ids sorted.
* oracle layer (``oracle_layer``): hidden 1024, intermediate 3072, fp32,
  gate/up [N,H] and down [H,N] ~ N(0, 0.02^2) drawn in that order from seed 0,
  64 tokens x ~ N(0,1) RMS-normalised as x / sqrt(mean(x^2) + 1e-6).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

DECODE_HIDDEN = 5120
DECODE_INTERMEDIATE = 17408
WEIGHT_STD = 0.02


def retention_k(intermediate: int, retention: float) -> int:
    return max(1, math.ceil(intermediate * retention))


@dataclass
class PackedLayer:
    packed: torch.Tensor   # [N, 3H] neuron-major records
    hidden: int
    intermediate: int

    def gate(self) -> torch.Tensor:
        return self.packed[:, :self.hidden]

    def up(self) -> torch.Tensor:
        return self.packed[:, self.hidden:2 * self.hidden]

    def down(self) -> torch.Tensor:
        """[H, N] view of the down projection (the reference's layout)."""
        return self.packed[:, 2 * self.hidden:3 * self.hidden].t()


def decode_layer(hidden: int = DECODE_HIDDEN, intermediate: int = DECODE_INTERMEDIATE,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda", seed: int = 0,
                 record_range: tuple[int, int] | None = None) -> PackedLayer:
    """Packed layer with iid N(0, 0.02^2) weights.  ``record_range`` draws only
    records [begin, end) of the full layer (an intermediate-dimension shard):
    record n is drawn from its own seed block, so shards of one seed agree with
    the unsharded layer."""
    if hidden % 8:
        raise ValueError("decode_layer draws packed records directly and needs hidden % 8 == 0")
    begin, end = record_range if record_range is not None else (0, intermediate)
    device = torch.device(device)
    packed = torch.empty((end - begin, 3 * hidden), dtype=dtype, device=device)
    block = 1024  # records per seeded block
    for b0 in range(begin - begin % block, end, block):
        gen = torch.Generator(device=device).manual_seed(seed * 1_000_003 + b0 // block)
        rows = torch.randn((block, 3 * hidden), generator=gen, device=device, dtype=torch.float32)
        rows.mul_(WEIGHT_STD)
        lo, hi = max(b0, begin), min(b0 + block, end)
        packed[lo - begin:hi - begin].copy_(rows[lo - b0:hi - b0])
    return PackedLayer(packed, hidden, end - begin)


def decode_x(batch: int = 1, hidden: int = DECODE_HIDDEN, dtype: torch.dtype = torch.bfloat16, seed: int = 1) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn((batch, hidden), generator=gen).to(dtype)


def decode_ids(intermediate: int, k: int, token: int = 0) -> torch.Tensor:
    """sort(randperm(N, seed=1000+token)[:K]) as int32 (CPU)."""
    gen = torch.Generator().manual_seed(1000 + token)
    return torch.randperm(intermediate, generator=gen)[:k].sort().values.to(torch.int32)


def selector_scores(batch: int, intermediate: int = DECODE_INTERMEDIATE, seed: int = 7, hot_fraction: float = 0.1,
                    boost: float = 8.0, zipf: float = 1.1) -> torch.Tensor:
    """[batch, N] fp32 Laplace(0,1) scores with a Zipf-boosted hot subset (CPU)."""
    gen = torch.Generator().manual_seed(seed)
    u = torch.rand((batch, intermediate), generator=gen, dtype=torch.float64) - 0.5
    scores = -torch.sign(u) * torch.log1p(-2 * u.abs())
    hot = torch.randperm(intermediate, generator=gen)[:max(1, int(round(hot_fraction * intermediate)))]
    ranks = torch.arange(1, hot.numel() + 1, dtype=torch.float64)
    scores[:, hot] += boost * ranks.pow(-zipf)
    return scores.to(torch.float32)


def oracle_layer(hidden: int = 1024, intermediate: int = 3072, tokens: int = 64, seed: int = 0):
    """(gate [N,H], up [N,H], down [H,N], x [T,H]) fp32 on CPU."""
    gen = torch.Generator().manual_seed(seed)
    gate = torch.randn((intermediate, hidden), generator=gen) * WEIGHT_STD
    up = torch.randn((intermediate, hidden), generator=gen) * WEIGHT_STD
    down = torch.randn((hidden, intermediate), generator=gen) * WEIGHT_STD
    x = torch.randn((tokens, hidden), generator=gen)
    x = x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
    return gate, up, down, x


def decode_bytes(k: int, hidden: int = DECODE_HIDDEN, esize: int = 2, batch: int = 1, index_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one decode call: K records + x + ids + y."""
    return k * 3 * hidden * esize + batch * hidden * esize + k * index_bytes + batch * hidden * esize


def offload_hot_set(intermediate: int = DECODE_INTERMEDIATE, hot_fraction: float = 0.25, seed: int = 11) -> torch.Tensor:
    """Sorted int64 ids of the always-resident neurons of a layer."""
    gen = torch.Generator().manual_seed(seed)
    n_hot = int(round(hot_fraction * intermediate))
    return torch.randperm(intermediate, generator=gen)[:n_hot].sort().values


def offload_token_ids(intermediate: int, k: int, hot: torch.Tensor, tokens: int, hot_pick: float = 0.8,
                      reuse: float = 0.5, seed: int = 12) -> list[torch.Tensor]:
    """Per-token sorted int32 id sets with hot-set bias and temporal reuse (CPU)."""
    gen = torch.Generator().manual_seed(seed)
    is_hot = torch.zeros(intermediate, dtype=torch.bool)
    is_hot[hot] = True

    def draw(count: int, exclude: torch.Tensor) -> torch.Tensor:
        want_hot = int(round(hot_pick * count))
        hot_pool = torch.nonzero(is_hot & ~exclude).flatten()
        cold_pool = torch.nonzero(~is_hot & ~exclude).flatten()
        want_hot = min(want_hot, hot_pool.numel())
        want_cold = min(count - want_hot, cold_pool.numel())
        picked = [hot_pool[torch.randperm(hot_pool.numel(), generator=gen)[:want_hot]],
                  cold_pool[torch.randperm(cold_pool.numel(), generator=gen)[:want_cold]]]
        return torch.cat(picked)

    out = []
    prev = None
    for _ in range(tokens):
        taken = torch.zeros(intermediate, dtype=torch.bool)
        if prev is None:
            ids = draw(k, taken)
        else:
            keep = prev[torch.randperm(prev.numel(), generator=gen)[:int(round(reuse * k))]]
            taken[keep] = True
            ids = torch.cat([keep, draw(k - keep.numel(), taken)])
        ids = ids.sort().values
        out.append(ids.to(torch.int32))
        prev = ids.long()
    return out


PREFILL_TOKENS = 512
PREFILL_TILE = 128
PREFILL_BLOCK = 64


def prefill_tile_blocks(intermediate: int = DECODE_INTERMEDIATE, tokens: int = PREFILL_TOKENS, density: float = 0.3,
                        hot_fraction: float = 0.2, seed: int = 21) -> tuple[torch.Tensor, list[torch.Tensor]]:
    """Block selections of a block-sparse prefill: (hot block ids, per-tile sorted block ids).

    Records form blocks of 64.  A seeded ``hot_fraction`` of the blocks is on
    for every 128-token tile; every other block is on per tile with
    probability p chosen so that the expected fraction of blocks per tile is
    ``density`` (p = (density * blocks - hot) / (blocks - hot)).
    """
    n_blocks = (intermediate + PREFILL_BLOCK - 1) // PREFILL_BLOCK
    n_tiles = (tokens + PREFILL_TILE - 1) // PREFILL_TILE
    gen = torch.Generator().manual_seed(seed)
    n_hot = int(round(hot_fraction * n_blocks))
    order = torch.randperm(n_blocks, generator=gen)
    hot = order[:n_hot].sort().values
    cold = order[n_hot:]
    p = max(0.0, (density * n_blocks - n_hot) / max(1, n_blocks - n_hot))
    tiles = []
    for _ in range(n_tiles):
        on = torch.rand(cold.numel(), generator=gen) < p
        tiles.append(torch.cat([hot, cold[on]]).sort().values.to(torch.int32))
    return hot, tiles


def prefill_x(tokens: int = PREFILL_TOKENS, hidden: int = DECODE_HIDDEN, dtype: torch.dtype = torch.bfloat16,
              seed: int = 22, device: str | torch.device = "cpu") -> torch.Tensor:
    """x ~ N(0, 1) of a prefill, [tokens, hidden]."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(tokens, hidden, generator=gen).to(dtype).to(device)


def prefill_flops(tile_blocks: list[torch.Tensor], hidden: int = DECODE_HIDDEN, intermediate: int | None = None,
                  tile: int = PREFILL_TILE) -> int:
    """Algorithmic FLOPs: per tile 2 * 128 * 3 * hidden * (records of its blocks)."""
    total = 0
    for blocks in tile_blocks:
        records = blocks.numel() * PREFILL_BLOCK
        if intermediate is not None and blocks.numel() and int(blocks.max()) == (intermediate - 1) // PREFILL_BLOCK:
            records -= (int(blocks.max()) + 1) * PREFILL_BLOCK - intermediate
        total += 2 * tile * 3 * hidden * records
    return total


def prefill_unique_bytes(tile_blocks: list[torch.Tensor], hidden: int = DECODE_HIDDEN, tokens: int = PREFILL_TOKENS,
                         esize: int = 2) -> int:
    """Bytes a block-major prefill must move: each used block once, plus x and y."""
    used = torch.unique(torch.cat([b.to(torch.int64) for b in tile_blocks])).numel()
    return used * PREFILL_BLOCK * 3 * hidden * esize + 2 * tokens * hidden * esize
