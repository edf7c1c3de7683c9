"""qcc_indexed_ffn_decode_static: the decode entry point for callers that cannot allocate.

Callers running inside another framework's allocator, plugin hosts that only
pass input and output buffers, or loops that must not call cudaMalloc/cudaFree
use this variant: its scratch is a fixed array inside the library, so the
call itself allocates nothing.  These tests call it through the C ABI and
compare it with qcc_indexed_ffn_decode (caller-provided workspace) on two
calls in a row, which also checks that the scratch left behind by one call
does not disturb the next.  Kept in a file of its own that is collected
last, and self-contained so it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import ffn as offn
from qcc_b200 import _lib
from qcc_b200.runtime.packing import pack_neuron_major

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 4 << 20


def _layer(hidden, intermediate, k, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    gate = (torch.randn(intermediate, hidden, generator=gen) * 0.02).to(dtype)
    up = (torch.randn(intermediate, hidden, generator=gen) * 0.02).to(dtype)
    down = (torch.randn(hidden, intermediate, generator=gen) * 0.02).to(dtype)
    x = torch.randn(1, hidden, generator=gen).to(dtype)
    ids = torch.randperm(intermediate, generator=gen)[:k].sort().values.to(torch.int32)
    return gate, up, down, x, ids


def _decode_with_workspace(lib, weights, x, ids, stream):
    code = _lib.dtype_code(x.dtype)
    nbytes = int(lib.qcc_decode_workspace_bytes(1, weights.hidden, code))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    _lib.check(lib.qcc_workspace_init(ws.data_ptr(), nbytes, stream), "qcc_workspace_init")
    y = torch.empty_like(x)
    status = lib.qcc_indexed_ffn_decode(x.data_ptr(), x.stride(0), 1, weights.hidden, weights.packed.data_ptr(),
                                        weights.n_records, code, ids.data_ptr(), _lib.INDEX_I32, ids.numel(), None,
                                        None, ws.data_ptr(), nbytes, y.data_ptr(), y.stride(0), code, None, 0,
                                        None, 0, stream)
    _lib.check(status, "qcc_indexed_ffn_decode")
    return y


def _decode_static(lib, weights, x, ids, stream):
    code = _lib.dtype_code(x.dtype)
    y = torch.empty_like(x)
    status = lib.qcc_indexed_ffn_decode_static(x.data_ptr(), x.stride(0), 1, weights.hidden,
                                               weights.packed.data_ptr(), weights.n_records, code, ids.data_ptr(),
                                               _lib.INDEX_I32, ids.numel(), None, None, y.data_ptr(), y.stride(0),
                                               code, None, 0, stream)
    _lib.check(status, "qcc_indexed_ffn_decode_static")
    return y


@pytest.mark.parametrize("hidden,intermediate,k,dtype,tol", [
    (5120, 4096, 1024, torch.bfloat16, 1e-2),
    (1024, 600, 150, torch.float32, 1e-5),
])
def test_static_scratch_matches_workspace_entry_point_twice(hidden, intermediate, k, dtype, tol):
    lib = _lib.library()
    device = torch.device("cuda", 0)
    gate, up, down, x, ids = _layer(hidden, intermediate, k, dtype, seed=hidden + k)
    weights = pack_neuron_major(gate.to(device), up.to(device), down.to(device))
    xd, idd = x.to(device), ids.to(device)
    stream = torch.cuda.current_stream(device).cuda_stream
    reference = _decode_with_workspace(lib, weights, xd, idd, stream)
    expected = offn.sparse_ffn_f64(x, ids, gate, up, down)
    # A first call with an id outside the layer leaves a non-zero status word in
    # the shared scratch (out-of-range ids are skipped, not a fault); the calls
    # after it must not be disturbed by what it left behind.
    bad = idd.clone()
    bad[0] = intermediate + 5
    _decode_static(lib, weights, xd, bad, stream)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        y = _decode_static(lib, weights, xd, idd, stream)
        torch.cuda.synchronize(device)
        assert offn.rel_l2(y.double().cpu().numpy(), reference.double().cpu().numpy()) <= tol
        assert offn.rel_l2(y.double().cpu().numpy(), expected) <= tol


def test_static_scratch_rejects_requests_beyond_its_size():
    lib = _lib.library()
    need = int(lib.qcc_decode_workspace_bytes(2, 5120, _lib.DTYPE_BF16))
    assert need > STATIC_SCRATCH_BYTES
    dummy = ctypes.c_void_p(256)
    status = lib.qcc_indexed_ffn_decode_static(dummy, 5120, 2, 5120, dummy, 10, _lib.DTYPE_BF16, dummy,
                                               _lib.INDEX_I32, 4, None, None, dummy, 5120, _lib.DTYPE_BF16, None, 0,
                                               None)
    assert status == _lib.ERR_WORKSPACE
