"""Packed-record artefact: layout, manifest checks and failures (host only).

Follows the reference's stream-cache tests (tests/test_freetoken_host_store.py:
a row gather from the host store, a checksum mismatch and a model mismatch)
for the interleaved record file.  The records are compared with the oracle's
restatement of the packed layout.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import ffn as offn
from qcc_b200.runtime import artefact
from qcc_b200.runtime.packing import PackedFFNWeights


def _layer(h=20, n=12, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(n, h, generator=g) * 0.02).to(dtype)
    up = (torch.randn(n, h, generator=g) * 0.02).to(dtype)
    down = (torch.randn(h, n, generator=g) * 0.02).to(dtype)
    return gate, up, down


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_round_trip_matches_oracle_layout(tmp_path, dtype):
    gate, up, down = _layer(dtype=dtype)
    manifest = artefact.write_artefact(tmp_path / "layer", (gate, up, down), source="unit")
    assert manifest["hidden"] == 20 and manifest["hidden_pad"] == 24 and manifest["intermediate"] == 12
    loaded = artefact.load_manifest(tmp_path / "layer", expected_shape=(20, 12))
    artefact.validate_files(tmp_path / "layer", loaded, checksums=True)
    records = artefact.read_records(tmp_path / "layer", loaded)
    want = offn.pack_records(gate.float().numpy(), up.float().numpy(), down.float().numpy())
    assert np.array_equal(records.float().numpy(), want)
    assert records.dtype == dtype


def test_shard_rows_and_transposed_down(tmp_path):
    gate, up, down = _layer(h=16, n=10)
    artefact.write_artefact(tmp_path / "a", (gate, up, down))
    full = artefact.read_records(tmp_path / "a")
    part = artefact.read_records(tmp_path / "a", record_range=(3, 7))
    assert torch.equal(part, full[3:7])
    assert artefact.read_records(tmp_path / "a", record_range=(5, 5)).shape == (0, 48)
    # Packing from the reference's transposed down_t gives the same records.
    assert torch.equal(artefact.pack_records_host(gate, up, down.t().contiguous(), transposed_down=True), full)
    with pytest.raises(ValueError, match="outside"):
        artefact.read_records(tmp_path / "a", record_range=(4, 11))


def test_packed_weights_slice_keeps_offsets(tmp_path):
    gate, up, down = _layer(h=8, n=6)
    packed = artefact.pack_records_host(gate, up, down)
    shard = PackedFFNWeights(packed[2:5], 8, 3, 2, 6)
    m = artefact.write_artefact(tmp_path / "s", shard)
    assert (m["record_offset"], m["total_intermediate"], m["intermediate"]) == (2, 6, 3)
    assert torch.equal(artefact.read_records(tmp_path / "s"), packed[2:5])


def test_checksum_size_and_format_failures(tmp_path):
    gate, up, down = _layer()
    root = tmp_path / "bad"
    artefact.write_artefact(root, (gate, up, down))
    manifest = artefact.load_manifest(root)
    payload = root / artefact.RECORDS_FILE
    raw = bytearray(payload.read_bytes())
    raw[5] ^= 0xFF
    payload.write_bytes(bytes(raw))
    artefact.validate_files(root, manifest, checksums=False)  # size still right
    with pytest.raises(ValueError, match="checksum"):
        artefact.validate_files(root, manifest, checksums=True)
    payload.write_bytes(bytes(raw[:-2]))
    with pytest.raises(ValueError, match="byte-size"):
        artefact.validate_files(root, manifest, checksums=False)
    payload.unlink()
    with pytest.raises(FileNotFoundError, match="payload"):
        artefact.validate_files(root, manifest)
    with pytest.raises(ValueError, match="expected"):
        artefact.load_manifest(root, expected_shape=(5120, 17408))
    text = json.loads((root / artefact.MANIFEST_FILE).read_text())
    for field, value, match in (("format_version", 99, "Unsupported"), ("format", "other", "Unsupported"),
                                ("hidden_pad", 21, "inconsistent"), ("dtype", "int8", "dtype")):
        broken = dict(text, **{field: value})
        (root / artefact.MANIFEST_FILE).write_text(json.dumps(broken))
        with pytest.raises(ValueError, match=match):
            artefact.load_manifest(root)
    broken = dict(text)
    del broken["records"]
    (root / artefact.MANIFEST_FILE).write_text(json.dumps(broken))
    with pytest.raises(ValueError, match="missing required field"):
        artefact.load_manifest(root)
    (root / artefact.MANIFEST_FILE).unlink()
    with pytest.raises(FileNotFoundError, match="manifest"):
        artefact.load_manifest(root)


def test_pack_reference_runtime_weights_file(tmp_path):
    from safetensors.torch import save_file

    gate, up, down = _layer(h=12, n=7)
    src = tmp_path / "layer.safetensors"
    save_file({"gate_proj.weight": gate, "up_proj.weight": up, "down_proj.weight": down}, str(src),
              metadata={"model": "unit-test"})
    manifest = artefact.pack_safetensors_layer(src, tmp_path / "packed")
    assert manifest["metadata"]["model"] == "unit-test"
    assert manifest["metadata"]["runtime_layout"] == "neuron_major_interleaved"
    records = artefact.read_records(tmp_path / "packed")
    assert torch.equal(records, artefact.pack_records_host(gate, up, down))
    save_file({"gate_proj.weight": gate, "up_proj.weight": up}, str(tmp_path / "partial.safetensors"))
    with pytest.raises(ValueError, match="missing"):
        artefact.pack_safetensors_layer(tmp_path / "partial.safetensors", tmp_path / "nope")


def test_load_packed_layer_refuses_cpu(tmp_path):
    artefact.write_artefact(tmp_path / "c", _layer())
    with pytest.raises(RuntimeError, match="CUDA"):
        artefact.load_packed_layer(tmp_path / "c", device="cpu")
