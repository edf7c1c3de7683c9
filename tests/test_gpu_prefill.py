"""Block-sparse prefill (qcc_indexed_ffn_prefill) against the oracle.

The reference runs each 128-token tile through TorchDynamicSparseFFN
(runtime/ffn.py:20-39) on the expansion of the tile's blocks
(clustering/block_layout.py:61-64); the oracle does the same in float64
(``oracle.ffn.sparse_ffn_f64``) and with the reference's own bf16 / fp16
rounding sequence (``oracle.ffn.dynamic_sparse_ffn``).  The tensor-core path
must agree within the north-star tolerance (rel-L2 1e-2 for 16-bit weights).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import TOL
from oracle import ffn as offn
from qcc_b200 import _lib
from qcc_b200 import workloads
from qcc_b200.runtime.packing import pack_neuron_major
from qcc_b200.runtime.prefill import BLOCK_RECORDS, TILE_TOKENS, BlockSparsePrefill, blocks_of_ids, tile_block_lists

PREFILL_TOL = TOL["bfloat16"]


def expand(blocks: torch.Tensor, n_records: int) -> torch.Tensor:
    """clustering/block_layout.py:61-64 (expand_block_indices) for one tile."""
    ids = [r for b in blocks.tolist() for r in range(b * BLOCK_RECORDS, min((b + 1) * BLOCK_RECORDS, n_records))]
    return torch.tensor(sorted(ids), dtype=torch.int64)


def oracle_prefill(x, tiles, gate, up, down):
    n = gate.shape[0]
    y = np.zeros((x.shape[0], gate.shape[1]))
    for t, blocks in enumerate(tiles):
        rows = slice(t * TILE_TOKENS, min((t + 1) * TILE_TOKENS, x.shape[0]))
        ids = expand(blocks, n)
        if ids.numel():
            y[rows] = offn.sparse_ffn_f64(x[rows], ids, gate, up, down)
    return y


def random_tiles(n_blocks, n_tiles, gen, density):
    tiles = []
    for _ in range(n_tiles):
        on = torch.rand(n_blocks, generator=gen) < density
        tiles.append(torch.nonzero(on).flatten().to(torch.int32)[torch.randperm(int(on.sum()), generator=gen)])
    return tiles


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,hidden,n,dtype,density", [
    (128, 256, 512, torch.bfloat16, 0.5),
    (100, 200, 130, torch.bfloat16, 0.7),      # partial tile, hidden not a multiple of 64, partial last block
    (300, 1024, 1024, torch.float16, 0.3),
    (640, 512, 768, torch.bfloat16, 0.4),      # two groups of tiles
    (1, 64, 64, torch.bfloat16, 1.0),
    (257, 5120, 2048, torch.bfloat16, 0.3),
])
def test_prefill_matches_oracle(tokens, hidden, n, dtype, density):
    gen = torch.Generator().manual_seed(tokens * 7 + hidden + n)
    gate = (torch.randn(n, hidden, generator=gen) * 0.05).to(dtype)
    up = (torch.randn(n, hidden, generator=gen) * 0.05).to(dtype)
    down = (torch.randn(hidden, n, generator=gen) * 0.05).to(dtype)
    x = torch.randn(tokens, hidden, generator=gen).to(dtype)
    n_blocks = (n + BLOCK_RECORDS - 1) // BLOCK_RECORDS
    tiles = random_tiles(n_blocks, (tokens + TILE_TOKENS - 1) // TILE_TOKENS, gen, density)
    dev = torch.device("cuda", 0)
    weights = pack_neuron_major(gate.to(dev), up.to(dev), down.to(dev))
    engine = BlockSparsePrefill(weights)
    y = engine(x.to(dev), tiles)
    torch.cuda.synchronize()
    engine.check()
    expected = oracle_prefill(x, tiles, gate, up, down)
    assert offn.rel_l2(y.double().cpu().numpy(), expected) <= PREFILL_TOL
    # Second call on the same workspace: identical result.
    y2 = engine(x.to(dev), tiles)
    assert torch.equal(y, y2)


@pytest.mark.gpu
def test_prefill_reference_rounding_and_fp32_output():
    """Against the reference's own bf16 sequence per tile, with an fp32 y."""
    hidden, n, tokens = 512, 1024, 256
    gen = torch.Generator().manual_seed(5)
    gate = (torch.randn(n, hidden, generator=gen) * 0.05).bfloat16()
    up = (torch.randn(n, hidden, generator=gen) * 0.05).bfloat16()
    down = (torch.randn(hidden, n, generator=gen) * 0.05).bfloat16()
    x = torch.randn(tokens, hidden, generator=gen).bfloat16()
    tiles = random_tiles(n // BLOCK_RECORDS, 2, gen, 0.4)
    dev = torch.device("cuda", 0)
    engine = BlockSparsePrefill(pack_neuron_major(gate.to(dev), up.to(dev), down.to(dev)))
    y = engine(x.to(dev), tiles, out_dtype=torch.float32)
    assert y.dtype == torch.float32
    ref = torch.cat([offn.dynamic_sparse_ffn(x[t * 128:(t + 1) * 128], expand(b, n), gate, up, down)
                     for t, b in enumerate(tiles)])
    assert offn.rel_l2(y.double().cpu().numpy(), ref.double().numpy()) <= PREFILL_TOL


def tf32(a: np.ndarray) -> np.ndarray:
    """fp32 values cut to tf32 (10 explicit mantissa bits, the low 13 bits dropped)."""
    return (np.asarray(a, dtype=np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def oracle_prefill_tf32(x, tiles, gate, up, down):
    """The prefill in float64 on tf32 operands, the activations cut to tf32 again before the down product."""
    n = gate.shape[0]
    xs, g, u, d = (tf32(t.numpy()).astype(np.float64) for t in (x, gate, up, down))
    y = np.zeros((x.shape[0], gate.shape[1]))
    for t, blocks in enumerate(tiles):
        rows = slice(t * TILE_TOKENS, min((t + 1) * TILE_TOKENS, x.shape[0]))
        ids = expand(blocks, n).numpy()
        if ids.size:
            gv, uv = xs[rows] @ g[ids].T, xs[rows] @ u[ids].T
            a = (gv / (1.0 + np.exp(-gv)) * uv).astype(np.float32)
            y[rows] = tf32(a).astype(np.float64) @ d[:, ids].T
    return y


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,hidden,n,density", [
    (128, 256, 512, 0.5),
    (100, 200, 130, 0.7),      # partial tile, hidden not a multiple of 32, partial last block
    (300, 1024, 1024, 0.3),
    (640, 512, 768, 0.4),      # two groups of tiles
    (257, 5120, 2048, 0.3),
])
def test_prefill_fp32_records_on_tf32(tokens, hidden, n, density):
    """fp32 records run on kind::tf32, which reads the tf32 part of each fp32
    operand (the low 13 mantissa bits dropped, not rounded).

    * Against float64 on the same tf32 operands: rel-L2 <= 1e-4.  What remains
      is the fp32 accumulation, and activations within an fp32 rounding of a
      tf32 boundary that the kernel and float64 cut to neighbouring tf32 values.
    * Against the exact fp32 layer: rel-L2 <= 5e-3 (measured 2.2e-3 to 2.3e-3),
      the tf32 cut of three operand streams.
    """
    gen = torch.Generator().manual_seed(tokens * 5 + hidden + n)
    gate = torch.randn(n, hidden, generator=gen) * 0.05
    up = torch.randn(n, hidden, generator=gen) * 0.05
    down = torch.randn(hidden, n, generator=gen) * 0.05
    x = torch.randn(tokens, hidden, generator=gen)
    n_blocks = (n + BLOCK_RECORDS - 1) // BLOCK_RECORDS
    tiles = random_tiles(n_blocks, (tokens + TILE_TOKENS - 1) // TILE_TOKENS, gen, density)
    dev = torch.device("cuda", 0)
    engine = BlockSparsePrefill(pack_neuron_major(gate.to(dev), up.to(dev), down.to(dev)))
    y = engine(x.to(dev), tiles)
    torch.cuda.synchronize()
    engine.check()
    assert y.dtype == torch.float32
    got = y.double().cpu().numpy()
    assert offn.rel_l2(got, oracle_prefill_tf32(x, tiles, gate, up, down)) <= 1e-4
    assert offn.rel_l2(got, oracle_prefill(x, tiles, gate, up, down)) <= 5e-3
    assert torch.equal(engine(x.to(dev), tiles), y)


@pytest.mark.gpu
def test_prefill_empty_tiles_and_out_of_range_blocks():
    hidden, n, tokens = 256, 512, 384
    gen = torch.Generator().manual_seed(9)
    gate = (torch.randn(n, hidden, generator=gen) * 0.05).bfloat16()
    up = (torch.randn(n, hidden, generator=gen) * 0.05).bfloat16()
    down = (torch.randn(hidden, n, generator=gen) * 0.05).bfloat16()
    x = torch.randn(tokens, hidden, generator=gen).bfloat16()
    dev = torch.device("cuda", 0)
    engine = BlockSparsePrefill(pack_neuron_major(gate.to(dev), up.to(dev), down.to(dev)))
    tiles = [torch.tensor([], dtype=torch.int32), torch.tensor([3, 1], dtype=torch.int32),
             torch.tensor([0, 7], dtype=torch.int32)]
    y = engine(x.to(dev), tiles).cpu()
    assert torch.count_nonzero(y[:128]) == 0
    assert offn.rel_l2(y.double().numpy(), oracle_prefill(x, tiles, gate, up, down)) <= PREFILL_TOL
    bad = [torch.tensor([0], dtype=torch.int32), torch.tensor([1, 99], dtype=torch.int32),
           torch.tensor([-1, 2], dtype=torch.int32)]
    y = engine(x.to(dev), bad).cpu()
    with pytest.raises(ValueError, match="range"):
        engine.check()
    good = [torch.tensor([0]), torch.tensor([1]), torch.tensor([2])]
    assert offn.rel_l2(y.double().numpy(), oracle_prefill(x, good, gate, up, down)) <= PREFILL_TOL


@pytest.mark.gpu
def test_prefill_tiles_equal_decode_engine():
    """Each tile of the prefill equals the fused decode kernel on the tile's expanded ids."""
    from qcc_b200.runtime.engine import IndexedSparseFFN
    hidden, n, tokens = 1024, 1536, 256
    dev = torch.device("cuda", 0)
    layer = workloads.decode_layer(hidden, n, device=dev, seed=4)
    from qcc_b200.runtime.packing import PackedFFNWeights
    weights = PackedFFNWeights(layer.packed, hidden, n)
    x = workloads.prefill_x(tokens, hidden, device=dev, seed=3)
    _, tiles = workloads.prefill_tile_blocks(n, tokens, seed=5)
    y = BlockSparsePrefill(weights)(x, tiles)
    decode = IndexedSparseFFN(weights)
    for t, blocks in enumerate(tiles):
        ids = expand(blocks, n).to(torch.int32).to(dev)
        rows = x[t * 128:(t + 1) * 128]
        ref = decode(rows, ids)
        assert offn.rel_l2(y[t * 128:(t + 1) * 128].double().cpu().numpy(), ref.double().cpu().numpy()) <= 1e-2


@pytest.mark.gpu
def test_prefill_full_size_against_torch_fp32():
    """The 512-token, hidden 5120, N 17408 prefill against an fp32 cuBLAS formulation."""
    dev = torch.device("cuda", 0)
    layer = workloads.decode_layer(device=dev, seed=2)
    from qcc_b200.runtime.packing import PackedFFNWeights
    weights = PackedFFNWeights(layer.packed, layer.hidden, layer.intermediate)
    x = workloads.prefill_x(device=dev)
    _, tiles = workloads.prefill_tile_blocks()
    flat, offsets = tile_block_lists(tiles, dev)
    y = BlockSparsePrefill(weights)(x, (flat, offsets))
    torch.cuda.synchronize()
    g, u, d = layer.gate(), layer.up(), layer.down()
    for t, blocks in enumerate(tiles):
        ids = expand(blocks, layer.intermediate).to(dev)
        xt = x[t * 128:(t + 1) * 128].float()
        a = torch.nn.functional.silu(xt @ g[ids].float().t()) * (xt @ u[ids].float().t())
        ref = a @ d[:, ids].float().t()
        err = (y[t * 128:(t + 1) * 128].float() - ref).norm() / ref.norm()
        assert float(err) <= PREFILL_TOL


def test_blocks_of_ids_round_trip():
    n = 17408
    blocks = torch.tensor([0, 5, 271])
    assert torch.equal(blocks_of_ids(expand(blocks, n), n_records=n), blocks)
    n = 130  # partial last block of 2 records
    assert torch.equal(blocks_of_ids(expand(torch.tensor([2]), n), n_records=n), torch.tensor([2]))
    with pytest.raises(ValueError, match="complete blocks"):
        blocks_of_ids(torch.arange(10))


def test_tile_block_lists_offsets():
    flat, offsets = tile_block_lists([torch.tensor([3, 1]), torch.tensor([], dtype=torch.int32),
                                      torch.tensor([7])], torch.device("cpu"))
    assert flat.tolist() == [3, 1, 7]
    assert offsets.tolist() == [0, 2, 2, 3]
    assert flat.dtype == torch.int32 and offsets.dtype == torch.int32


def test_prefill_workload_density():
    hot, tiles = workloads.prefill_tile_blocks()
    assert hot.numel() == 54 and len(tiles) == 4
    for t in tiles:
        assert set(hot.tolist()) <= set(t.tolist())
        assert torch.equal(t, t.sort().values)
    density = sum(t.numel() for t in tiles) / (4 * 272)
    assert 0.25 <= density <= 0.35
    flops = workloads.prefill_flops(tiles)
    assert flops == sum(2 * 128 * 3 * 5120 * 64 * t.numel() for t in tiles)


def test_prefill_abi_rejects_bad_dtypes_and_shapes():
    lib = _lib.library()
    dummy = 256
    status = lib.qcc_indexed_ffn_prefill(dummy, 64, 4, 64, dummy, 64, 99, dummy, dummy, dummy, 1 << 20,
                                         dummy, 64, _lib.DTYPE_F32, None)
    assert status == _lib.ERR_DTYPE
    status = lib.qcc_indexed_ffn_prefill(dummy, 64, 4, 64, dummy, 64, _lib.DTYPE_F32, dummy, dummy, dummy, 1 << 20,
                                         dummy, 64, 99, None)
    assert status == _lib.ERR_DTYPE
    status = lib.qcc_indexed_ffn_prefill(dummy, 32, 4, 64, dummy, 64, _lib.DTYPE_BF16, dummy, dummy, dummy, 1 << 20,
                                         dummy, 64, _lib.DTYPE_BF16, None)
    assert status == _lib.ERR_SHAPE
