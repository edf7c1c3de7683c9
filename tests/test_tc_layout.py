"""Operand-layout arithmetic of the tensor-core decode kernel, emulated on the CPU.

The kernel (csrc/decode_tc.cuh) feeds tcgen05.mma with no-swizzle shared-memory
operands built from 128-byte core matrices.  For both majors SBO is the byte
distance between core matrices adjacent in M (or N) and LBO the distance
between core matrices adjacent in K; within a core matrix a K-major operand
holds 8 M rows of 8 K elements (rows 16 bytes apart), an MN-major one 8 K rows
of 8 M elements.  These tests replay the kernel's descriptors (start offsets,
LBO, SBO), its diagonal extraction and its TMEM-to-hidden index map with numpy
in float64 and check that they compute the gated FFN:

* gate / up: records staged 2 KB apart read as "8 rows per record" (K-major),
  token rows read as the matching B operand; the dot product is the sum of
  the diagonal D[(r, i), (t, i)] over i;
* down: the records' down parts as an MN-major A operand, a block-diagonal B
  (a[t, r] on the diagonal of an 8x8 block per record and token) in a high and
  a low 16-bit part; lane (g, m) of tile j, column (t, kk) = y_t[1024 j + 64 g
  + 8 kk + m].
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

GROUP, CHUNK, TILE = 16, 1024, 1024  # records per group, gate|up elements per stage, hidden elements per y tile


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).bfloat16().float().double().numpy()


def _kmajor(buf: np.ndarray, start: int, lbo: int, sbo: int, rows: int) -> np.ndarray:
    """[rows, 16] elements of a K-major no-swizzle operand (16-bit elements, byte addresses)."""
    m = np.arange(rows)[:, None]
    k = np.arange(16)[None, :]
    addr = start + (m // 8) * sbo + (k // 8) * lbo + (m % 8) * 16 + (k % 8) * 2
    return buf[addr // 2]


def _mnmajor(buf: np.ndarray, start: int, lbo: int, sbo: int, rows: int) -> np.ndarray:
    """[rows (M), 16 (K)] elements of an MN-major no-swizzle operand."""
    m = np.arange(rows)[:, None]
    k = np.arange(16)[None, :]
    addr = start + (m // 8) * sbo + (k // 8) * lbo + (k % 8) * 16 + (m % 8) * 2
    return buf[addr // 2]


def _setup(seed, hidden, tokens):
    rng = np.random.default_rng(seed)
    gate = _bf16(rng.standard_normal((GROUP, hidden)) * 0.05)
    up = _bf16(rng.standard_normal((GROUP, hidden)) * 0.05)
    down = _bf16(rng.standard_normal((GROUP, hidden)) * 0.05)  # record r's down part: D[:, r]
    x = _bf16(rng.standard_normal((tokens, hidden)))
    return gate, up, down, x


@pytest.mark.parametrize("hidden", [2048, 3584])
def test_gate_up_diagonal_sums_are_the_dot_products(hidden):
    # 3584: the last gate / up chunk holds 512 elements (four K steps of 128 instead of eight).
    tp = 4
    n = 8 * tp
    gate, up, _, x = _setup(0, hidden, tp)
    xs = x.reshape(-1)  # token rows hidden * 2 bytes apart (the kernel's x staging)
    accs = []
    for part in (gate, up):
        acc = np.zeros((128, n))
        for c in range((hidden + CHUNK - 1) // CHUNK):
            el = min(CHUNK, hidden - c * CHUNK)
            stage = np.full(GROUP * TILE, np.nan)  # record r's chunk at r * 2 KB; the rest is never read
            for r in range(GROUP):
                stage[r * TILE:r * TILE + el] = part[r, c * CHUNK:c * CHUNK + el]
            for k in range(el // 128):
                a = _kmajor(stage, 256 * k, 128, CHUNK * 2, 128)
                b = _kmajor(xs, (c * CHUNK + 128 * k) * 2, 128, hidden * 2, n)
                acc += a @ b.T
        accs.append(acc)
    rows = np.arange(128)
    for t in range(tp):
        # lane 8 r + i holds column 8 t + i; the record's eight lanes sum to the dot product
        diag = [acc[rows, 8 * t + (rows % 8)].reshape(GROUP, 8).sum(axis=1) for acc in accs]
        np.testing.assert_allclose(diag[0], gate @ x[t], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(diag[1], up @ x[t], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("hidden", [2048, 3584])
@pytest.mark.parametrize("rn", [1, 13, 16])
def test_down_tiles_with_split_activations_give_y(hidden, rn):
    # rn records in the group; an odd group's last MMA step repeats its last record with a zero
    # activation.  3584: the last tile holds 512 elements; rows past them read unwritten memory
    # and are not stored.
    tp = 4
    n = 8 * tp
    _, _, down, _ = _setup(1, hidden, tp)
    act = np.random.default_rng(2).standard_normal((tp, GROUP)) * 3.0
    act[:, rn:] = 0.0
    hi = _bf16(act)
    lo = _bf16(act - hi)
    bhi = np.zeros(tp * 1024)
    blo = np.zeros(tp * 1024)
    for t in range(tp):
        for r in range(GROUP):
            for i in range(8):  # element t * 1024 + r * 64 + 9 i: the diagonal of block (t, r)
                bhi[t * 1024 + r * 64 + 9 * i] = hi[t, r]
                blo[t * 1024 + r * 64 + 9 * i] = lo[t, r]
    y = np.full((tp, hidden), np.nan)
    for j in range((hidden + TILE - 1) // TILE):
        el = min(TILE, hidden - j * TILE)
        stage = np.full(GROUP * TILE, np.nan)  # slots past the group and past el stay unwritten
        for s_ in range(rn + (rn & 1)):
            stage[s_ * TILE:s_ * TILE + el] = down[min(s_, rn - 1), j * TILE:j * TILE + el]
        acc = np.zeros((128, n))
        for p in range((rn + 1) // 2):
            a = _mnmajor(stage, p * 2 * TILE * 2, TILE * 2, 128, 128)
            acc += a @ _kmajor(bhi, p * 256, 128, 2048, n).T
            acc += a @ _kmajor(blo, p * 256, 128, 2048, n).T
        lane = np.arange(128)[:, None]
        col = np.arange(n)[None, :]
        h = j * TILE + 64 * (lane // 8) + 8 * (col % 8) + lane % 8
        keep = np.broadcast_to(h < hidden, acc.shape)
        tok = np.broadcast_to(col // 8, acc.shape)
        y[tok[keep], h[keep]] = acc[keep]
    expected = act @ down  # y_t = sum_r a[t, r] D[:, r]
    # The high and low parts carry the activation to ~2^-17 relative.
    np.testing.assert_allclose(y, expected, rtol=0, atol=1e-5 * np.abs(expected).max())
