"""The C-ABI library loads without a GPU and exports what include/qcc_b200.h declares."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
import qcc_b200
from qcc_b200 import _lib

HEADER = ROOT / "include" / "qcc_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^QCC_API\s+[\w\s\*]+?\b(qcc_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("qcc_indexed_ffn_decode", "qcc_select_topk", "qcc_build_union", "qcc_pack_records",
                     "qcc_decode_workspace_bytes", "qcc_workspace_init", "qcc_version"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.library_path()))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_pure_host_queries_without_gpu():
    lib = _lib.library()
    assert lib.qcc_version() == 2
    assert lib.qcc_hidden_pad(5120, _lib.DTYPE_BF16) == 5120
    assert lib.qcc_hidden_pad(5, _lib.DTYPE_F32) == 8
    assert lib.qcc_record_bytes(5120, _lib.DTYPE_BF16) == 30720
    assert lib.qcc_record_bytes(5120, _lib.DTYPE_F32) == 61440
    # 2-8 tokens of 16-bit records with hidden % 128 == 0 run on the tensor cores.
    assert lib.qcc_decode_max_batch(5120, _lib.DTYPE_BF16) == 8
    assert lib.qcc_decode_max_batch(5120, _lib.DTYPE_F16) == 8
    assert lib.qcc_decode_max_batch(2560, _lib.DTYPE_BF16) == 8
    assert lib.qcc_decode_max_batch(8192, _lib.DTYPE_BF16) == 6
    assert lib.qcc_decode_max_batch(10240, _lib.DTYPE_BF16) == 4
    # fp32 records and other sizes: the CUDA-core kernel's limits.
    assert lib.qcc_decode_max_batch(5120, _lib.DTYPE_F32) == 4
    assert lib.qcc_decode_max_batch(5000, _lib.DTYPE_BF16) == 4
    assert lib.qcc_decode_max_batch(8192, _lib.DTYPE_F32) == 1
    assert lib.qcc_decode_max_batch(20480, _lib.DTYPE_BF16) == 0
    # status / counters header + one fp32 partial row per CTA (up to 160 CTAs)
    assert lib.qcc_decode_workspace_bytes(1, 5120, _lib.DTYPE_BF16) == 256 + 160 * 5120 * 4
    assert lib.qcc_workspace_status_offset() == 0
    assert lib.qcc_status_string(_lib.ERR_SHAPE).decode().startswith("inconsistent")


def test_argument_validation_happens_before_any_cuda_call():
    lib = _lib.library()
    dummy = ctypes.c_void_p(16)
    # batch 0 -> shape error; unknown dtype -> dtype error; tiny workspace -> workspace error.
    big = 1 << 30
    args = [dummy, 8, 0, 8, dummy, 4, _lib.DTYPE_BF16, dummy, _lib.INDEX_I32, 2, None, None, dummy, big, dummy, 8,
            _lib.DTYPE_BF16, None, 0, None, 0, None]
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_SHAPE
    args[2] = 1
    args[6] = 9
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_DTYPE
    args[6] = _lib.DTYPE_BF16
    args[13] = 16
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_WORKSPACE
    args[13] = big
    args[4] = ctypes.c_void_p(18)  # packed not 16-byte aligned
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_ALIGNMENT
    args[4] = dummy
    args[8] = _lib.INDEX_I32 | 0x200  # an unknown flag bit in the index type
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_DTYPE
    args[8] = _lib.INDEX_I32 | _lib.IDS_READY
    args[2] = 0
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_SHAPE  # the flag is accepted, batch 0 is not
    # Batches beyond qcc_decode_max_batch: 5 tokens of fp32 records (limit 4), 7 at hidden 8192 (limit 6); more
    # than 8 tokens never fit the token-mask byte.
    args[8] = _lib.INDEX_I32
    args[2], args[3], args[6], args[16] = 5, 5120, _lib.DTYPE_F32, _lib.DTYPE_F32
    args[1], args[15] = 5120, 5120
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_UNSUPPORTED
    args[2], args[3], args[6], args[16] = 7, 8192, _lib.DTYPE_BF16, _lib.DTYPE_BF16
    args[1], args[15] = 8192, 8192
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_UNSUPPORTED
    args[2] = 9
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_SHAPE
    # QCC_MASK_SHIFT(s): the call's tokens must fit bits s .. s + batch - 1 of the mask byte.
    args[2] = 4
    args[8] = _lib.INDEX_I32 | _lib.mask_shift(5)
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_SHAPE
    args[8] = _lib.INDEX_I32 | 0x8000  # the bit above the shift field
    assert lib.qcc_indexed_ffn_decode(*args) == _lib.ERR_DTYPE
    args[2], args[8] = 1, _lib.INDEX_I32
    # Cross-rank sum: the exchange buffers must hold three slots of this batch for every rank.
    need = int(lib.qcc_exchange_bytes(2, 1, 8, _lib.DTYPE_BF16))
    assert need == 256 + 3 * 2 * 2 * 16
    xchg = (ctypes.c_void_p * 2)(16, 32)
    ar = [dummy, 8, 1, 8, dummy, 4, _lib.DTYPE_BF16, dummy, _lib.INDEX_I32, 2, None, None, dummy, big, dummy, 8,
          _lib.DTYPE_BF16, None, 0, 0, 4, xchg, need - 16, 2, 0, None]
    assert lib.qcc_indexed_ffn_decode_allreduce(*ar) == _lib.ERR_WORKSPACE
    ar[2] = 2  # a batch beyond what the buffer was sized for
    ar[22] = need
    assert lib.qcc_indexed_ffn_decode_allreduce(*ar) == _lib.ERR_WORKSPACE
    assert lib.qcc_exchange_init(None, need) == _lib.ERR_INVALID_ARGUMENT
    assert lib.qcc_exchange_set_wait_limit(None, 1000) == _lib.ERR_INVALID_ARGUMENT
    assert lib.qcc_select_topk(dummy, 4, 1, 4, 5, dummy, 5, None) == _lib.ERR_SHAPE  # k > n
    assert lib.qcc_build_union(dummy, 4, 9, 4, 0, 10, dummy, dummy, dummy, None) == _lib.ERR_SHAPE  # batch > 8
    assert lib.qcc_pack_records(dummy, dummy, 4, dummy, 1, 1, 4, 8, _lib.DTYPE_BF16, dummy, None) == _lib.ERR_SHAPE


def test_check_raises_with_status_text():
    with pytest.raises(_lib.QCCError, match="inconsistent shape"):
        _lib.check(_lib.ERR_SHAPE, "qcc_select_topk")


def test_package_import_name():
    assert qcc_b200.__name__ == "qcc_b200"
    assert qcc_b200.library_path().name == "libqcc_b200.so"
